// selftest.cu — an on-device check of the failure path every kernel of this library relies on: a
// bounded wait that runs out.
//
// The GEMM kernels' waits (sm100_common.cuh mbar_wait) give up after KDB_WAIT_NS, record
// KDB_ERR_TIMEOUT and a site id in the device status word, raise the CTA's abort flag, and the CTA
// then frees its tensor memory and returns instead of hanging.  In normal runs no wait ever runs
// out, so this kernel makes one run out on purpose and cheaply: one CTA allocates TMEM like the GEMMs
// do, waits with a short caller-given limit on an mbarrier that nothing arrives on, and tears down
// through the same steps (abort flag, TMEM free, return).  The caller then reads the status word and
// can launch normal work on the same context.  Nothing faults, traps or spins without a limit.
#include "host_util.h"
#include "sm100_common.cuh"

namespace kdb {

constexpr unsigned int kSiteSelfTest = 0x1F0;

__global__ void __launch_bounds__(64, 1) wait_timeout_selftest_kernel(uint64_t limit_ns) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_word;
  volatile int* abort_flag = &abort_word;
  const int warp = warp_id_uniform();
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(&tmem_slot, 32);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = tmem_slot;
  if (threadIdx.x == 0) {
    // phase 0 of a fresh barrier completes only after one arrival, and nothing arrives
    mbar_wait_for(&bar, 0, abort_flag, kSiteSelfTest, limit_ns);
  } else if (warp == 1 && lane_id() == 0) {
    // a second role waiting on the same phase leaves once the first has raised the abort flag
    mbar_wait_for(&bar, 0, abort_flag, kSiteSelfTest + 1, 2 * limit_ns + 1000000ull);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, 32);
  }
}

int selftest_wait_timeout(unsigned long long limit_ns, cudaStream_t s) {
  if (limit_ns < 1000ull || limit_ns > KDB_WAIT_NS) return KDB_ERR_INVALID_ARG;
  wait_timeout_selftest_kernel<<<1, 64, 0, s>>>(static_cast<uint64_t>(limit_ns));
  return cuda_status(cudaGetLastError());
}

}  // namespace kdb

// moe_noalloc.cu — the MoE permutation plan with its scratch in a fixed device array inside the
// library, for callers that cannot allocate device memory.
//
// Who needs it: a caller that owns only the buffers it passes in and has no device allocator of its
// own — for example a serving runtime bound to this library over a C FFI whose memory is reserved
// once at start-up, or code running where cudaMalloc is not permitted (inside a stream capture, under
// a hard memory budget) — cannot provide the workspace kdb_moe_plan asks for.  This entry point runs
// the same plan kernels on a file-scope __device__ array instead.
//
// The array holds kNoallocPlanBytes (1,577,216 bytes, about 1.5 MiB) on every GPU where the library is
// loaded, until the process exits.  Its limits: t * k <= 131072 routed slots, e <= 1024 experts and
// ceil(t / 256) * e <= 65536 chunk cells; larger calls are rejected with KDB_ERR_UNSUPPORTED.
//
// Host code cannot use the array's name as a device address: its device address is resolved once per
// device with cudaGetSymbolAddress, with that device current, the first time this entry point runs on
// it.  That first call therefore makes a runtime call that must not happen inside a stream capture;
// make it once before capturing.  The resolved address is cached for the life of the process: after a
// device reset (cudaDeviceReset, or a primary context torn down and created again) it no longer names
// the array, so a caller that resets a device must not use this entry point on that device again.
//
// Every call shares the array and it keeps the last call's contents.  Nothing in it has to start at
// zero: each call writes every cell it later reads (the per-chunk counts are written for every chunk
// and expert, the bases and m-tile prefix by the scan, the row arrays by the scatter).  Calls whose
// kernels overlap on the GPU — on different streams, or from different host threads — race on the
// array; issue them on one stream or serialise them.
#include <mutex>

#include "host_util.h"
#include "moe.h"

namespace kdb {

namespace {
constexpr long long kNoallocMaxRows = 131072;        // t * k
constexpr long long kNoallocMaxChunkCells = 65536;   // ceil(t / 256) * e
constexpr long long kNoallocMaxExperts = 1024;
// Laid out as moe_plan_only carves it: two chunk tables, the (e + 1) m-tile prefix, two row arrays,
// each rounded up to 256 bytes.
constexpr size_t kNoallocPlanBytes = 2 * (kNoallocMaxChunkCells * 4) + ((kNoallocMaxExperts + 1) * 4 + 255) / 256 * 256 +
                                     2 * (kNoallocMaxRows * 4);
static_assert(kNoallocPlanBytes == 1577216, "documented size of the fixed plan scratch");

static __device__ __align__(256) unsigned char g_noalloc_plan_scratch[kNoallocPlanBytes];

std::mutex g_noalloc_mu;
void* g_noalloc_addr[64] = {nullptr};

int noalloc_scratch(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_status(e);
  if (dev < 0 || dev >= 64) return KDB_ERR_NO_DEVICE;
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_noalloc_addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_plan_scratch);
    if (e != cudaSuccess) return cuda_status(e);
    g_noalloc_addr[dev] = p;
  }
  *out = g_noalloc_addr[dev];
  return KDB_OK;
}
}  // namespace

int moe_plan_noalloc(const int* ids, const float* topk_w, long long T, long long E, long long k, int* counts,
                     int* offsets, int* perm_slot, int* slot_pos, cudaStream_t s) {
  if (T < 0 || E <= 0 || k <= 0 || k > E) return KDB_ERR_INVALID_ARG;
  if (T * k > kNoallocMaxRows || E > kNoallocMaxExperts || ((T + 255) / 256) * E > kNoallocMaxChunkCells)
    return KDB_ERR_UNSUPPORTED;
  if (!ids || !topk_w || !counts || !offsets || !perm_slot || !slot_pos) return KDB_ERR_INVALID_ARG;
  const size_t need = moe_plan_scratch_bytes(T, E, k);
  if (need > kNoallocPlanBytes) return KDB_ERR_UNSUPPORTED;
  void* scratch = nullptr;
  int rc = noalloc_scratch(&scratch);
  if (rc) return rc;
  return moe_plan_only(ids, topk_w, static_cast<int>(T), static_cast<int>(E), static_cast<int>(k), counts, offsets,
                       perm_slot, slot_pos, scratch, kNoallocPlanBytes, s);
}

}  // namespace kdb

// capi.cu — extern "C" entry points of libkdb200.so (declared in include/kdb200.h).
#include <cuda_runtime.h>

#include "../../include/kdb200.h"
#include "kdb_status.h"
#include "host_util.h"
#include "proj.h"
#include "sm100_common.cuh"

namespace kdb {
cudaError_t last_cuda_error();
}  // namespace kdb

extern "C" {

int kdb_abi_version(void) { return KDB200_ABI_VERSION; }

const char* kdb_strerror(int code) {
  switch (code) {
    case KDB_OK: return "ok";
    case KDB_ERR_INVALID_ARG: return "invalid argument (size, null or misaligned pointer, stride)";
    case KDB_ERR_UNSUPPORTED: return "shape not supported by the kernels";
    case KDB_ERR_CUDA: return "CUDA runtime/driver error";
    case KDB_ERR_TIMEOUT: return "a bounded device wait timed out";
    case KDB_ERR_WORKSPACE: return "workspace too small";
    case KDB_ERR_NO_DEVICE: return "no sm_100 device";
    case KDB_ERR_DEVICE_BOUNDS: return "a kernel rejected an out-of-range index";
    default: return "unknown status";
  }
}

int kdb_last_cuda_error(void) { return static_cast<int>(kdb::last_cuda_error()); }

int kdb_status_read(uint32_t out[4], int clear, void* stream) {
  if (!out) return KDB_ERR_INVALID_ARG;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int rc = kdb::cuda_status(cudaMemcpyFromSymbolAsync(out, kdb::g_status, sizeof(unsigned int) * 4, 0,
                                                      cudaMemcpyDeviceToHost, s));
  if (rc) return rc;
  rc = kdb::cuda_status(cudaStreamSynchronize(s));
  if (rc) return rc;
  if (clear) {
    static const unsigned int zero[4] = {0, 0, 0, 0};
    rc = kdb::cuda_status(cudaMemcpyToSymbolAsync(kdb::g_status, zero, sizeof(zero), 0, cudaMemcpyHostToDevice, s));
    if (rc) return rc;
    rc = kdb::cuda_status(cudaStreamSynchronize(s));
  }
  return rc;
}

int kdb_proj_bf16(const void* x, const void* w, void* y, int64_t m, int64_t n, int64_t k, int64_t ldy,
                  void* stream) {
  return kdb::proj_bf16(x, w, y, m, n, k, ldy, 0, static_cast<cudaStream_t>(stream));
}

int kdb_proj_bf16_cfg(const void* x, const void* w, void* y, int64_t m, int64_t n, int64_t k, int64_t ldy,
                      int tile_n, void* stream) {
  return kdb::proj_bf16(x, w, y, m, n, k, ldy, tile_n, static_cast<cudaStream_t>(stream));
}

}  // extern "C"

// host_util.cu — see host_util.h.
#include "host_util.h"

#include <atomic>
#include <mutex>

namespace kdb {

static thread_local cudaError_t t_last_cuda_error = cudaSuccess;

void set_cuda_error(cudaError_t e) { t_last_cuda_error = e; }
cudaError_t last_cuda_error() { return t_last_cuda_error; }

int cuda_status(cudaError_t e) {
  if (e == cudaSuccess) return KDB_OK;
  set_cuda_error(e);
  return KDB_ERR_CUDA;
}

static std::atomic<int> g_sm_budget{0};

int set_sm_budget(int sms) { return g_sm_budget.exchange(sms > 0 ? sms : 0); }
int sm_budget() { return g_sm_budget.load(); }

int num_sms() {
  static int cache[64] = {0};
  int dev = 0;
  int n = 148;
  if (cudaGetDevice(&dev) == cudaSuccess && dev >= 0 && dev < 64) {
    if (cache[dev] == 0) {
      int v = 0;
      if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0) v = 148;
      cache[dev] = v;
    }
    n = cache[dev];
  }
  const int b = g_sm_budget.load(std::memory_order_relaxed);
  return (b > 0 && b < n) ? (b < 2 ? 2 : b) : n;
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

int make_tmap_bf16_2d(CUtensorMap* map, const void* base, uint64_t inner, uint64_t rows, uint64_t ld,
                      uint32_t box_inner, uint32_t box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return KDB_ERR_CUDA;
  if (!aligned16(base) || (ld * 2) % 16 != 0 || inner == 0 || rows == 0) return KDB_ERR_INVALID_ARG;
  const cuuint64_t dims[2] = {inner, rows};
  const cuuint64_t strides[1] = {ld * 2};
  const cuuint32_t box[2] = {box_inner, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? KDB_OK : KDB_ERR_INVALID_ARG;
}

int make_token_maps(TokenMaps* m, const void* rows, uint64_t n_rows, uint64_t k) {
  for (int i = 0; i < 5; ++i) {
    const int rc = make_tmap_bf16_2d(&m->m[i], rows, k, n_rows, k, 64, 16u << i);
    if (rc) return rc;
  }
  return KDB_OK;
}

}  // namespace kdb

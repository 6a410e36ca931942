// capi.cu — extern "C" entry points of libkdb200.so (declared in include/kdb200.h).
#include <cuda_runtime.h>

#include "../../include/kdb200.h"
#include "kdb_status.h"
#include "host_util.h"
#include "moe.h"
#include "proj.h"
#include "sm100_common.cuh"

namespace kdb {
cudaError_t last_cuda_error();
int selftest_wait_timeout(unsigned long long limit_ns, cudaStream_t s);
size_t attn_workspace_bytes(long long B, long long T, long long Hq, long long Hkv, long long max_len,
                            long long window);
int attn_decode_fp8(const void* q, const void* k_new, const void* v_new, void* k_cache, void* v_cache,
                    const int* block_table, const int* seq_lens, float kv_scale, void* out, long long B, long long T,
                    long long Hq, long long Hkv, long long D, long long max_len, long long slots, long long window,
                    void* workspace, size_t workspace_bytes, cudaStream_t s);
}  // namespace kdb

extern "C" {

int kdb_abi_version(void) { return KDB200_ABI_VERSION; }

int kdb_set_sm_budget(int32_t sms) { return kdb::set_sm_budget(sms < 0 ? 0 : sms); }

int kdb_sm_budget(void) { return kdb::sm_budget(); }

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

int kdb_selftest_wait_timeout(uint64_t limit_ns, void* stream) {
  return kdb::selftest_wait_timeout(limit_ns, static_cast<cudaStream_t>(stream));
}

int kdb_proj_bf16(const void* x, const void* w, void* y, int64_t m, int64_t n, int64_t k, int64_t ldy,
                  void* stream) {
  return kdb::proj_bf16(x, w, y, m, n, k, ldy, 0, 0, static_cast<cudaStream_t>(stream));
}

size_t kdb_proj_workspace_bytes(int64_t m, int64_t n, int64_t k) { return kdb::proj_workspace_bytes(m, n, k); }

int kdb_proj_bf16_ws(const void* x, const void* w, void* y, int64_t m, int64_t n, int64_t k, int64_t ldy,
                     void* workspace, size_t workspace_bytes, void* stream) {
  if (workspace && (reinterpret_cast<uintptr_t>(workspace) & 15) != 0) return KDB_ERR_INVALID_ARG;
  return kdb::proj_bf16(x, w, y, m, n, k, ldy, 0, 0, static_cast<cudaStream_t>(stream), workspace, workspace_bytes);
}

int kdb_proj_split_f32(const float* w, void* w_split, int64_t n, int64_t k, void* stream) {
  return kdb::proj_split_f32(w, w_split, n, k, static_cast<cudaStream_t>(stream));
}

size_t kdb_proj_f32w_workspace_bytes(int64_t m, int64_t n, int64_t k) { return kdb::proj_f32w_workspace_bytes(m, n, k); }

int kdb_proj_f32w(const void* x, const void* w_split, float* y, int64_t m, int64_t n, int64_t k, void* workspace,
                  size_t workspace_bytes, void* stream) {
  if (workspace && (reinterpret_cast<uintptr_t>(workspace) & 15) != 0) return KDB_ERR_INVALID_ARG;
  return kdb::proj_f32w(x, w_split, y, m, n, k, workspace, workspace_bytes, static_cast<cudaStream_t>(stream));
}

int kdb_proj_tile_shape(int64_t m, int64_t n, int32_t out[2]) {
  if (!out || m <= 0 || n <= 0) return KDB_ERR_INVALID_ARG;
  int bn = 0, pair = 0;
  kdb::pick_tile(m, n, kdb::num_sms(), &bn, &pair);
  out[0] = bn;
  out[1] = pair;
  return KDB_OK;
}

int kdb_proj_bf16_cfg(const void* x, const void* w, void* y, int64_t m, int64_t n, int64_t k, int64_t ldy,
                      int tile_n, int cta_pair, void* stream) {
  return kdb::proj_bf16(x, w, y, m, n, k, ldy, tile_n, cta_pair, static_cast<cudaStream_t>(stream));
}

static kdb::MoeShape moe_shape(int64_t t, int64_t h, int64_t e, int64_t i, int64_t k, int64_t shared,
                               int64_t shared_i) {
  kdb::MoeShape sh;
  sh.t = t;
  sh.h = h;
  sh.e = e;
  sh.i = i;
  sh.k = k;
  sh.shared = shared;
  sh.shared_i = shared_i;
  return sh;
}

size_t kdb_moe_workspace_bytes(int64_t t, int64_t h, int64_t e, int64_t i, int64_t k, int64_t shared,
                               int64_t shared_i) {
  return kdb::moe_workspace_bytes(moe_shape(t, h, e, i, k, shared, shared_i));
}

int kdb_moe_pack_gate_up(const void* w_gate_up, void* packed, int64_t e, int64_t i, int64_t h, void* stream) {
  if (e < 0 || i <= 0 || h <= 0 || i % 128 != 0 || h % 8 != 0) return KDB_ERR_INVALID_ARG;
  if (e * 2 * i > (1ll << 31)) return KDB_ERR_UNSUPPORTED;
  if (!w_gate_up || !packed || w_gate_up == packed) return KDB_ERR_INVALID_ARG;
  if (!kdb::aligned16(w_gate_up) || !kdb::aligned16(packed)) return KDB_ERR_INVALID_ARG;
  return kdb::moe_pack_gate_up(w_gate_up, packed, (int)e, (int)i, (int)h, static_cast<cudaStream_t>(stream));
}

int kdb_moe_route(const void* x, const float* router_w, const float* router_bias, float* logits, float* topk_w,
                  int32_t* topk_ids, int64_t t, int64_t h, int64_t e, int64_t k, void* stream) {
  if (t < 0 || h <= 0 || e <= 0 || e > 1024 || k <= 0 || k > e || k > 32) return KDB_ERR_INVALID_ARG;
  if (t * e > (1ll << 31) / 4 || t * h > (1ll << 40)) return KDB_ERR_UNSUPPORTED;
  if (t == 0) return KDB_OK;
  if (!x || !router_w || !logits || !topk_w || !topk_ids) return KDB_ERR_INVALID_ARG;
  return kdb::moe_route(x, router_w, router_bias, logits, topk_w, topk_ids, (int)t, (int)h, (int)e, (int)k,
                        static_cast<cudaStream_t>(stream));
}

size_t kdb_moe_plan_workspace_bytes(int64_t t, int64_t e, int64_t k) { return kdb::moe_plan_scratch_bytes(t, e, k); }

int kdb_moe_plan(const int32_t* topk_ids, const float* topk_w, int64_t t, int64_t e, int64_t k, int32_t* counts,
                 int32_t* offsets, int32_t* perm_slot, int32_t* slot_pos, void* workspace, size_t workspace_bytes,
                 void* stream) {
  if (t < 0 || t * k > (1ll << 30)) return KDB_ERR_INVALID_ARG;
  return kdb::moe_plan_only(topk_ids, topk_w, (int)t, (int)e, (int)k, counts, offsets, perm_slot, slot_pos,
                            workspace, workspace_bytes, static_cast<cudaStream_t>(stream));
}

int kdb_moe_plan_noalloc(const int32_t* topk_ids, const float* topk_w, int64_t t, int64_t e, int64_t k,
                         int32_t* counts, int32_t* offsets, int32_t* perm_slot, int32_t* slot_pos, void* stream) {
  return kdb::moe_plan_noalloc(topk_ids, topk_w, t, e, k, counts, offsets, perm_slot, slot_pos,
                               static_cast<cudaStream_t>(stream));
}

int kdb_moe_prepare_router(const float* router_w, void* router_split, float* router_norms, int64_t e, int64_t h,
                           void* stream) {
  if (e <= 0 || h <= 0 || e > 1024 || e * h > (1ll << 31)) return KDB_ERR_INVALID_ARG;
  if (!router_w || !router_split || !router_norms) return KDB_ERR_INVALID_ARG;
  return kdb::router_prepare(router_w, router_split, router_norms, (int)e, (int)h, static_cast<cudaStream_t>(stream));
}

int kdb_moe_router_approx(const void* x, const void* router_split, float* approx, int64_t t, int64_t h, int64_t e,
                          void* stream) {
  if (t < 0 || h <= 0 || e <= 0 || e > 1024 || h % 64 != 0) return KDB_ERR_INVALID_ARG;
  if (t == 0) return KDB_OK;
  if (!x || !router_split || !approx || !kdb::aligned16(x) || !kdb::aligned16(router_split)) return KDB_ERR_INVALID_ARG;
  if (t * e > (1ll << 31) / 4) return KDB_ERR_UNSUPPORTED;
  return kdb::router_approx(x, router_split, approx, (int)t, (int)h, (int)e, static_cast<cudaStream_t>(stream));
}

size_t kdb_moe_route_fast_workspace_bytes(int64_t t, int64_t e) {
  if (t < 0 || e <= 0) return 0;
  return kdb::router_fast_scratch_bytes(t, e);
}

int kdb_moe_route_fast(const void* x, const float* router_w, const float* router_bias, const void* router_split,
                       const float* router_norms, float* topk_w, int32_t* topk_ids, int64_t t, int64_t h, int64_t e,
                       int64_t k, void* workspace, size_t workspace_bytes, void* stream) {
  if (t < 0 || h <= 0 || h % 64 != 0 || e <= 0 || e > 1024 || k <= 0 || k > e || k > 32) return KDB_ERR_INVALID_ARG;
  if (t * e > (1ll << 31) / 4) return KDB_ERR_UNSUPPORTED;
  if (t == 0) return KDB_OK;
  if (!x || !router_w || !router_split || !router_norms || !topk_w || !topk_ids) return KDB_ERR_INVALID_ARG;
  if (!kdb::aligned16(x) || !kdb::aligned16(router_w) || !kdb::aligned16(router_split)) return KDB_ERR_INVALID_ARG;
  if (!workspace || workspace_bytes < kdb::router_fast_scratch_bytes(t, e)) return KDB_ERR_WORKSPACE;
  if ((reinterpret_cast<uintptr_t>(workspace) & 255) != 0) return KDB_ERR_INVALID_ARG;
  return kdb::moe_route_fast(x, router_w, router_bias, router_split, router_norms, topk_w, topk_ids, (int)t, (int)h,
                             (int)e, (int)k, workspace, static_cast<cudaStream_t>(stream));
}

int kdb_moe_gather_rows(const void* x, const int32_t* index, int64_t div, void* out, int64_t rows, int64_t h,
                        int64_t t, void* stream) {
  if (rows < 0 || h <= 0 || h % 8 != 0 || t < 0 || div <= 0 || rows > (1ll << 31) || t > (1ll << 31)) return KDB_ERR_INVALID_ARG;
  if (rows == 0) return KDB_OK;
  if (!x || !index || !out || !kdb::aligned16(x) || !kdb::aligned16(out)) return KDB_ERR_INVALID_ARG;
  return kdb::moe_gather_rows(x, index, out, (int)rows, (int)h, (int)t, static_cast<cudaStream_t>(stream), (int)div);
}

static int expert_gemm_args(const void* a, int64_t a_rows, const void* w, int64_t groups, int64_t i, int64_t h,
                            const int32_t* offsets, const int32_t* mtile_start, const void* out) {
  if (a_rows < 0 || groups <= 0 || i <= 0 || h <= 0 || i % 128 != 0 || h % 8 != 0) return KDB_ERR_INVALID_ARG;
  if ((offsets == nullptr) != (mtile_start == nullptr)) return KDB_ERR_INVALID_ARG;
  if (!offsets && groups != 1) return KDB_ERR_INVALID_ARG;
  if (a_rows > (1ll << 30) || groups * 2 * i > (1ll << 31) || groups * h > (1ll << 31)) return KDB_ERR_UNSUPPORTED;
  if (a_rows == 0) return KDB_OK;
  if (!a || !w || !out || !kdb::aligned16(a) || !kdb::aligned16(w) || !kdb::aligned16(out)) return KDB_ERR_INVALID_ARG;
  return -1;   // arguments fine, work to do
}

int kdb_moe_expert_gate_up(const void* a, int64_t a_rows, const void* w_gate_up_packed, int64_t groups, int64_t i,
                           int64_t h, const int32_t* offsets, const int32_t* mtile_start, void* out, void* stream) {
  const int rc = expert_gemm_args(a, a_rows, w_gate_up_packed, groups, i, h, offsets, mtile_start, out);
  if (rc >= 0) return rc;
  return kdb::moe_gemm_gate_up(a, (int)a_rows, w_gate_up_packed, (int)groups, (int)i, (int)h, offsets, mtile_start,
                               out, static_cast<cudaStream_t>(stream));
}

size_t kdb_moe_expert_down_combine_workspace_bytes(int64_t t, int64_t h) {
  if (t <= 0 || h <= 0 || h % 128 != 0) return 0;
  return static_cast<size_t>(t) * static_cast<size_t>(h / 128) * sizeof(int);
}

int kdb_moe_expert_down_combine(const void* a, int64_t a_rows, const void* w_down, int64_t groups, int64_t i, int64_t h,
                                const int32_t* offsets, const int32_t* mtile_start, const float* row_scale,
                                const int32_t* perm_slot, const int32_t* slot_pos, const void* shared_rows,
                                void* rows_out, void* y, int64_t t, int64_t k, void* workspace,
                                size_t workspace_bytes, void* stream) {
  const int rc = expert_gemm_args(a, a_rows, w_down, groups, i, h, offsets, mtile_start, rows_out);
  if (rc >= 0) return rc;
  if (!offsets || !row_scale || !perm_slot || !slot_pos || !y || t <= 0 || k <= 0 || k > 32) return KDB_ERR_INVALID_ARG;
  if (h % 128 != 0 || t > (1ll << 30) / 32) return KDB_ERR_UNSUPPORTED;
  if (!workspace || workspace_bytes < kdb_moe_expert_down_combine_workspace_bytes(t, h)) return KDB_ERR_WORKSPACE;
  if ((reinterpret_cast<uintptr_t>(workspace) & 3) != 0) return KDB_ERR_INVALID_ARG;
  return kdb::moe_gemm_down_combine(a, (int)a_rows, w_down, (int)groups, (int)i, (int)h, offsets, mtile_start,
                                    row_scale, perm_slot, slot_pos, static_cast<int*>(workspace), shared_rows, rows_out,
                                    y, (int)t, (int)k, static_cast<cudaStream_t>(stream));
}

int kdb_moe_expert_down(const void* a, int64_t a_rows, const void* w_down, int64_t groups, int64_t i, int64_t h,
                        const int32_t* offsets, const int32_t* mtile_start, const float* row_scale, void* out,
                        void* stream) {
  const int rc = expert_gemm_args(a, a_rows, w_down, groups, i, h, offsets, mtile_start, out);
  if (rc >= 0) return rc;
  return kdb::moe_gemm_down(a, (int)a_rows, w_down, (int)groups, (int)i, (int)h, offsets, mtile_start, row_scale, out,
                            static_cast<cudaStream_t>(stream));
}

int kdb_moe_combine(const void* rows, const int32_t* slot_pos, const float* slot_w, const void* shared_rows, void* y,
                    int64_t t, int64_t h, int64_t k, void* stream) {
  if (t < 0 || h <= 0 || h % 8 != 0 || k <= 0 || k > 32 || t * k > (1ll << 31)) return KDB_ERR_INVALID_ARG;
  if (t == 0) return KDB_OK;
  if (!rows || !slot_pos || !y || !kdb::aligned16(rows) || !kdb::aligned16(y)) return KDB_ERR_INVALID_ARG;
  if (shared_rows && !kdb::aligned16(shared_rows)) return KDB_ERR_INVALID_ARG;
  return kdb::moe_combine(rows, slot_pos, shared_rows, y, (int)t, (int)h, (int)k, static_cast<cudaStream_t>(stream),
                          slot_w);
}

size_t kdb_moe_ep_regroup_workspace_bytes(int64_t p, int64_t er) {
  if (p <= 0 || er <= 0 || er > 1024 || p > 1024) return 0;
  return kdb::moe_ep_regroup_scratch_bytes((int)p, (int)er);
}

int kdb_moe_ep_regroup(const int32_t* counts, int64_t p, int64_t er, int to_expert_major, const void* in, void* out,
                       int64_t h, int32_t* offsets, int32_t* mtile_start, void* workspace, size_t workspace_bytes,
                       void* stream) {
  if (p <= 0 || p > 1024 || er <= 0 || er > 1024 || h <= 0 || h % 8 != 0) return KDB_ERR_INVALID_ARG;
  if (!counts || !offsets || !mtile_start) return KDB_ERR_INVALID_ARG;
  if ((in == nullptr) != (out == nullptr)) return KDB_ERR_INVALID_ARG;
  if (in && (!kdb::aligned16(in) || !kdb::aligned16(out) || in == out)) return KDB_ERR_INVALID_ARG;
  if (!workspace || workspace_bytes < kdb::moe_ep_regroup_scratch_bytes((int)p, (int)er)) return KDB_ERR_WORKSPACE;
  if ((reinterpret_cast<uintptr_t>(workspace) & 255) != 0) return KDB_ERR_INVALID_ARG;
  return kdb::moe_ep_regroup(counts, (int)p, (int)er, to_expert_major, in, out, (int)h, offsets, mtile_start,
                             workspace, static_cast<cudaStream_t>(stream));
}

int kdb_moe_forward(const void* x, const float* router_w, const float* router_bias, const void* router_split,
                    const float* router_norms, const void* w_gate_up_packed,
                    const void* w_down, const void* shared_gate_up_packed, const void* shared_down, void* y,
                    float* topk_w, int32_t* topk_ids, int64_t t, int64_t h, int64_t e, int64_t i, int64_t k,
                    int64_t shared, int64_t shared_i, void* workspace, size_t workspace_bytes, void* stream) {
  return kdb::moe_forward(x, router_w, router_bias, router_split, router_norms, w_gate_up_packed, w_down,
                          shared_gate_up_packed, shared_down, y,
                          topk_w, topk_ids, moe_shape(t, h, e, i, k, shared, shared_i), workspace, workspace_bytes,
                          static_cast<cudaStream_t>(stream));
}

size_t kdb_moe_w4a16_workspace_bytes(int64_t t, int64_t h, int64_t i, int64_t local, int64_t e_total, int64_t k) {
  return kdb::moe_w4a16_workspace_bytes(t, h, i, local, e_total, k);
}

int kdb_moe_w4a16_forward(const void* x, const int32_t* topk_ids, const float* topk_w, const void* w13_blocks,
                          const float* w13_gscale, const void* w2_blocks, const float* w2_gscale, const float* pw1,
                          void* y, int64_t t, int64_t h, int64_t i, int64_t local, int64_t e_total, int64_t k,
                          void* workspace, size_t workspace_bytes, void* stream) {
  return kdb::moe_w4a16_forward(x, topk_ids, topk_w, w13_blocks, w13_gscale, w2_blocks, w2_gscale, pw1, y, t, h, i,
                                local, e_total, k, workspace, workspace_bytes, static_cast<cudaStream_t>(stream));
}

size_t kdb_attn_decode_workspace_bytes(int64_t batch, int64_t q_len, int64_t q_heads, int64_t kv_heads,
                                       int64_t max_len, int64_t window) {
  return kdb::attn_workspace_bytes(batch, q_len, q_heads, kv_heads, max_len, window);
}

int kdb_attn_decode_fp8(const void* q, const void* k_new, const void* v_new, void* k_cache, void* v_cache,
                        const int32_t* block_table, const int32_t* seq_lens, float kv_scale, void* out,
                        int64_t batch, int64_t q_len, int64_t q_heads, int64_t kv_heads, int64_t head_dim,
                        int64_t max_len, int64_t slots, int64_t window, void* workspace, size_t workspace_bytes,
                        void* stream) {
  return kdb::attn_decode_fp8(q, k_new, v_new, k_cache, v_cache, block_table, seq_lens, kv_scale, out, batch, q_len,
                              q_heads, kv_heads, head_dim, max_len, slots, window, workspace, workspace_bytes,
                              static_cast<cudaStream_t>(stream));
}

}  // extern "C"

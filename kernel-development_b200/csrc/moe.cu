// moe.cu — the fused MoE layer forward: route -> plan -> gather -> grouped gate_up (SwiGLU) ->
// [shared expert] -> grouped down (x routing weight) -> combine.  Every stage is a kernel launched on
// the caller's stream; all scratch is carved from the caller's workspace, so the forward never
// allocates or synchronises and can be captured in a CUDA graph.
//
// Reference counterpart: the whole `up_moe` engine (okc-challenge/engines/x3_h.cu:311-663), which
// fuses plan, gate_up, SwiGLU, down and combine for M <= 8 tokens on an H200; here the stages are
// separate persistent kernels sized for T up to 16384 tokens.
#include "host_util.h"
#include "moe.h"

namespace kdb {

namespace {
constexpr size_t kAlign = 256;
inline size_t up(size_t v) { return (v + kAlign - 1) / kAlign * kAlign; }
constexpr int kChunk = 256;   // tokens per plan chunk (moe_route.cu)

struct Carve {
  size_t logits, chunk_counts, chunk_base, counts, offsets, mtile_start, perm_slot, slot_pos, perm_token, perm_w,
      xy_perm, hbuf, hshared, yshared, total;
};

Carve carve(const MoeShape& sh) {
  Carve c{};
  const size_t T = sh.t, H = sh.h, E = sh.e, I = sh.i, K = sh.k;
  const size_t R = T * K;
  const size_t C = (T + kChunk - 1) / kChunk;
  size_t o = 0;
  c.logits = o;       o += router_fast_scratch_bytes(T, E);   // exact logits, or approx + candidates
  c.chunk_counts = o; o += up(sizeof(int) * C * E);
  c.chunk_base = o;   o += up(sizeof(int) * C * E);
  c.counts = o;       o += up(sizeof(int) * E);
  c.offsets = o;      o += up(sizeof(int) * (E + 1));
  c.mtile_start = o;  o += up(sizeof(int) * (E + 1));
  c.perm_slot = o;    o += up(sizeof(int) * R);
  c.slot_pos = o;     o += up(sizeof(int) * R);
  c.perm_token = o;   o += up(sizeof(int) * R);
  c.perm_w = o;       o += up(sizeof(float) * R);
  c.xy_perm = o;      o += up(2 * R * H);          // x_perm, later reused for the per-slot down output
  c.hbuf = o;         o += up(2 * R * I);
  c.hshared = o;      o += sh.shared ? up(2 * T * sh.shared_i) : 0;
  c.yshared = o;      o += sh.shared ? up(2 * T * H) : 0;
  c.total = o;
  return c;
}
}  // namespace

int moe_check_shape(const MoeShape& sh) {
  if (sh.t < 0 || sh.h <= 0 || sh.e <= 0 || sh.i <= 0 || sh.k <= 0) return KDB_ERR_INVALID_ARG;
  if (sh.k > sh.e || sh.k > 32) return KDB_ERR_UNSUPPORTED;
  if (sh.e > 1024) return KDB_ERR_UNSUPPORTED;
  if (sh.h % 8 != 0) return KDB_ERR_UNSUPPORTED;          // TMA rows and 16-byte vectors
  if (sh.i % 128 != 0) return KDB_ERR_UNSUPPORTED;        // gate/up packing in 128-row halves
  if (sh.shared < 0 || sh.shared > 1) return KDB_ERR_UNSUPPORTED;
  if (sh.shared && (sh.shared_i <= 0 || sh.shared_i % 128 != 0)) return KDB_ERR_UNSUPPORTED;
  if (sh.t * sh.k > (1ll << 30) || sh.t * sh.e > (1ll << 31) / 4) return KDB_ERR_UNSUPPORTED;
  return KDB_OK;
}

size_t moe_workspace_bytes(const MoeShape& sh) {
  if (moe_check_shape(sh) != KDB_OK) return 0;
  return carve(sh).total;
}

size_t moe_plan_scratch_bytes(long long t, long long e, long long k) {
  if (t < 0 || e <= 0 || k <= 0) return 0;
  const size_t C = (static_cast<size_t>(t) + kChunk - 1) / kChunk, R = static_cast<size_t>(t) * k;
  return 2 * up(sizeof(int) * C * e) + up(sizeof(int) * (e + 1)) + up(sizeof(int) * R) + up(sizeof(float) * R);
}

int moe_plan_only(const int* ids, const float* topk_w, int T, int E, int k, int* counts, int* offsets,
                  int* perm_slot, int* slot_pos, void* workspace, size_t workspace_bytes, cudaStream_t s) {
  if (T < 0 || E <= 0 || E > 1024 || k <= 0 || k > E) return KDB_ERR_INVALID_ARG;
  if (!ids || !topk_w || !counts || !offsets || !perm_slot || !slot_pos) return KDB_ERR_INVALID_ARG;
  const size_t need = moe_plan_scratch_bytes(T, E, k);
  if (!workspace || workspace_bytes < need) return KDB_ERR_WORKSPACE;
  if ((reinterpret_cast<uintptr_t>(workspace) & (kAlign - 1)) != 0) return KDB_ERR_INVALID_ARG;
  const size_t C = (static_cast<size_t>(T) + kChunk - 1) / kChunk, R = static_cast<size_t>(T) * k;
  char* ws = static_cast<char*>(workspace);
  int* chunk_counts = reinterpret_cast<int*>(ws);
  int* chunk_base = reinterpret_cast<int*>(ws + up(sizeof(int) * C * E));
  int* mtile_start = reinterpret_cast<int*>(ws + 2 * up(sizeof(int) * C * E));
  int* perm_token = reinterpret_cast<int*>(ws + 2 * up(sizeof(int) * C * E) + up(sizeof(int) * (E + 1)));
  float* perm_w = reinterpret_cast<float*>(ws + 2 * up(sizeof(int) * C * E) + up(sizeof(int) * (E + 1)) +
                                           up(sizeof(int) * R));
  return moe_plan(ids, topk_w, T, E, k, chunk_counts, chunk_base, counts, offsets, mtile_start, perm_slot, slot_pos,
                  perm_token, perm_w, s);
}

int moe_forward(const void* x, const float* router_w, const float* router_bias, const void* router_split,
                const float* router_norms, const void* w_gate_up_packed,
                const void* w_down, const void* shared_gate_up_packed, const void* shared_down, void* y,
                float* topk_w, int* topk_ids, const MoeShape& sh, void* workspace, size_t workspace_bytes,
                cudaStream_t s) {
  int rc = moe_check_shape(sh);
  if (rc) return rc;
  if (sh.t == 0) return KDB_OK;   // nothing to route (empty tensors may carry null pointers)
  if (!x || !router_w || !w_gate_up_packed || !w_down || !y || !topk_w || !topk_ids) return KDB_ERR_INVALID_ARG;
  if (sh.shared && (!shared_gate_up_packed || !shared_down)) return KDB_ERR_INVALID_ARG;
  if (!aligned16(x) || !aligned16(y) || !aligned16(w_gate_up_packed) || !aligned16(w_down)) return KDB_ERR_INVALID_ARG;
  const Carve c = carve(sh);
  if (!workspace || workspace_bytes < c.total) return KDB_ERR_WORKSPACE;
  if ((reinterpret_cast<uintptr_t>(workspace) & (kAlign - 1)) != 0) return KDB_ERR_INVALID_ARG;
  char* ws = static_cast<char*>(workspace);
  auto F = [&](size_t off) { return reinterpret_cast<float*>(ws + off); };
  auto Ip = [&](size_t off) { return reinterpret_cast<int*>(ws + off); };

  const int T = static_cast<int>(sh.t), H = static_cast<int>(sh.h), E = static_cast<int>(sh.e);
  const int I = static_cast<int>(sh.i), K = static_cast<int>(sh.k);
  const int R = T * K;

  // Routing: the tensor-core pre-pass with exact re-evaluation of the candidates when the router has
  // been prepared (kdb_moe_prepare_router) and H is a multiple of 64; otherwise every logit in the
  // fixed fp64 order.  Both give identical ids and weights.
  if (router_split && router_norms && H % 64 == 0 && aligned16(router_w) && aligned16(router_split))
    rc = moe_route_fast(x, router_w, router_bias, router_split, router_norms, topk_w, topk_ids, T, H, E, K,
                        ws + c.logits, s);
  else
    rc = moe_route(x, router_w, router_bias, F(c.logits), topk_w, topk_ids, T, H, E, K, s);
  if (rc) return rc;
  rc = moe_plan(topk_ids, topk_w, T, E, K, Ip(c.chunk_counts), Ip(c.chunk_base), Ip(c.counts), Ip(c.offsets),
                Ip(c.mtile_start), Ip(c.perm_slot), Ip(c.slot_pos), Ip(c.perm_token), F(c.perm_w), s);
  if (rc) return rc;
  void* xy_perm = ws + c.xy_perm;
  void* hbuf = ws + c.hbuf;
  rc = moe_gather_rows(x, Ip(c.perm_token), xy_perm, R, H, T, s);
  if (rc) return rc;
  // a token picks an expert at most once: no group holds more than T rows
  rc = moe_gemm_gate_up(xy_perm, R, w_gate_up_packed, E, I, H, Ip(c.offsets), Ip(c.mtile_start), hbuf, s, T);
  if (rc) return rc;
  // the shared expert first: the routed down's combine reads its rows
  void* yshared = nullptr;
  if (sh.shared) {
    const int Is = static_cast<int>(sh.shared_i);
    void* hs = ws + c.hshared;
    yshared = ws + c.yshared;
    rc = moe_gemm_gate_up(x, T, shared_gate_up_packed, 1, Is, H, nullptr, nullptr, hs, s);
    if (rc) return rc;
    rc = moe_gemm_down(hs, T, shared_down, 1, Is, H, nullptr, nullptr, nullptr, yshared, s);
    if (rc) return rc;
  }
  // x_perm is dead once gate_up has run (stream order): its buffer takes the per-slot down output.  The
  // combine runs as its own kernel: the down GEMM with the combine merged into its epilogue
  // (moe_gemm_down_combine, kdb_moe_expert_down_combine) measured slower on B200 at every layer size tried.
  rc = moe_gemm_down(hbuf, R, w_down, E, I, H, Ip(c.offsets), Ip(c.mtile_start), F(c.perm_w), xy_perm, s, T);
  if (rc) return rc;
  return moe_combine(xy_perm, Ip(c.slot_pos), yshared, y, T, H, K, s);
}

}  // namespace kdb

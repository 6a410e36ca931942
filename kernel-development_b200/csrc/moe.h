// moe.h — internal launchers of the MoE layer (C-ABI wrappers in capi.cu).
#pragma once
#include <cstddef>
#include <cuda_runtime.h>

namespace kdb {

// Tokens of one grouped-GEMM tile: the plan's tile prefix mtile_start[g] counts ceil(count_g / kMoeTokenTile).
constexpr int kMoeTokenTile = 512;

int moe_route(const void* x, const float* wr, const float* bias, float* logits, float* topk_w, int* topk_ids,
              int T, int H, int E, int k, cudaStream_t s);
int moe_plan(const int* ids, const float* topk_w, int T, int E, int k, int* chunk_counts, int* chunk_base,
             int* counts, int* offsets, int* mtile_start, int* perm_slot, int* slot_pos, int* perm_token,
             float* perm_w, cudaStream_t s);
int moe_gather_rows(const void* x, const int* perm_token, void* x_perm, int R, int H, int T, cudaStream_t s,
                    int div = 1);
int moe_combine(const void* yperm, const int* slot_pos, const void* yshared, void* y, int T, int H, int k,
                cudaStream_t s, const float* slot_w = nullptr);
// Expert-parallel regroup (moe_ep.cu): rows held as blocks (source rank s, local expert e) in
// source-major order <-> expert-major order.  counts: int32 [P, Er] on the device.
int moe_ep_regroup(const int* counts, int P, int Er, int to_expert_major, const void* in, void* out, int H,
                   int* offsets, int* mtile_start, void* scratch, cudaStream_t s);
size_t moe_ep_regroup_scratch_bytes(int P, int Er);
int moe_pack_gate_up(const void* w, void* packed, int E, int I, int H, cudaStream_t s);
// Grouped expert GEMMs (moe_gemm.cu).  max_group_tokens: an upper bound on any group's row count that the
// caller guarantees (0 = none known; a_rows is used); a bound <= 64 selects the weight-streaming variant.
int moe_gemm_gate_up(const void* a, int a_rows, const void* w_packed, int groups, int I, int H, const int* offsets,
                     const int* mtile_start, void* out, cudaStream_t s, int max_group_tokens = 0);
int moe_gemm_down(const void* a, int a_rows, const void* w_down, int groups, int I, int H, const int* offsets,
                  const int* mtile_start, const float* row_scale, void* out, cudaStream_t s, int max_group_tokens = 0);
// Grouped down (CTA-pair path) with the weighted combine fused into its epilogue: rows_out receives the
// scaled per-slot rows, y[t] the combine of token t's k slot rows (+ yshared[t]); arrivals: int32
// [T, H / 128] scratch, zeroed here.  H % 128 == 0.
int moe_gemm_down_combine(const void* a, int a_rows, const void* w_down, int groups, int I, int H,
                          const int* offsets, const int* mtile_start, const float* row_scale, const int* perm_slot,
                          const int* slot_pos, int* arrivals, const void* yshared, void* rows_out, void* y, int T,
                          int k, cudaStream_t s);

// NVFP4 w4a16 layer of one expert-parallel rank (moe_w4a16.cu).
size_t moe_w4a16_workspace_bytes(long long T, long long H, long long I, long long L, long long E, long long k);
int moe_w4a16_forward(const void* x, const int* ids, const float* tw, const void* w13_blocks, const float* w13_gscale,
                      const void* w2_blocks, const float* w2_gscale, const float* pw1,
                      void* y, long long T, long long H, long long I, long long L, long long E, long long k,
                      void* workspace, size_t workspace_bytes, cudaStream_t s);

struct MoeShape {
  long long t, h, e, i, k, shared, shared_i;
};

// Validates a layer shape; KDB_OK or an error code.
int moe_check_shape(const MoeShape& sh);

// Workspace bytes of moe_forward for a shape (0 on an invalid shape).
size_t moe_workspace_bytes(const MoeShape& sh);

// Scratch bytes of moe_plan_only (chunk counts/bases, m-tile prefix, row tokens, row weights).
size_t moe_plan_scratch_bytes(long long t, long long e, long long k);

// The routing plan alone (for composition and tests): counts[E], offsets[E + 1], perm_slot[T*k],
// slot_pos[T*k] from topk ids/weights; scratch from `workspace`.
int moe_plan_only(const int* ids, const float* topk_w, int T, int E, int k, int* counts, int* offsets,
                  int* perm_slot, int* slot_pos, void* workspace, size_t workspace_bytes, cudaStream_t s);

// kdb_moe_plan_noalloc: the plan with scratch in a fixed device array (moe_noalloc.cu).
int moe_plan_noalloc(const int* ids, const float* topk_w, long long T, long long E, long long k, int* counts,
                     int* offsets, int* perm_slot, int* slot_pos, cudaStream_t s);

// Fast router (moe_router_fast.cu): prepare splits the fp32 router into [bf16 hi | bf16 mid] and row norms.
int router_prepare(const float* wr, void* wcat, float* norms, int E, int H, cudaStream_t s);
int router_approx(const void* x, const void* wcat, float* approx, int T, int H, int E, cudaStream_t s);
size_t router_fast_scratch_bytes(long long T, long long E);
int moe_route_fast(const void* x, const float* wr, const float* bias, const void* wcat, const float* norms,
                   float* topk_w, int* topk_ids, int T, int H, int E, int k, void* scratch, cudaStream_t s);

int moe_forward(const void* x, const float* router_w, const float* router_bias, const void* router_split,
                const float* router_norms, const void* w_gate_up_packed,
                const void* w_down, const void* shared_gate_up_packed, const void* shared_down, void* y,
                float* topk_w, int* topk_ids, const MoeShape& sh, void* workspace, size_t workspace_bytes,
                cudaStream_t s);

}  // namespace kdb

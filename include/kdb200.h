/*
 * kdb200.h — C ABI of libkdb200.so, the B200 (sm_100a) kernels behind the bf16 projection and the
 * fused Mixture-of-Experts layer.
 *
 * Every entry point takes plain device pointers, sizes in elements, and a cudaStream_t passed as
 * `void*` (NULL = legacy default stream).  Entry points never allocate device memory and never
 * synchronise: scratch comes from a caller-provided workspace, so each call is capturable in a CUDA
 * graph.  They return KDB_OK (0) or one of the KDB_ERR_* codes in kdb_status.h; asynchronous device
 * errors (a bounded wait that timed out, a kernel's own bounds check) land in the device status
 * word read by kdb_status_read().  Two entry points depart from this, each described at its
 * declaration: kdb_status_read synchronises the stream it is given, and kdb_moe_plan_noalloc takes
 * its scratch from a fixed array inside the library (not from a workspace) and resolves that array's
 * address with a runtime call on its first use per device, which must not happen inside a capture.
 *
 * The reference reaches these paths only through its problem-adapter boundary: the submission's
 * `prepare(weights) -> state` and `kernel_fn(data, state) -> out`, called by
 * kdev `OkcAdapter.prepare/call` (src/kdev/adapters/okc.py:501-515, 534-537).  The Python host
 * layer (kernel-development_b200/kdb200) exposes exactly those two functions on top of this ABI.
 */
#ifndef KDB200_H
#define KDB200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define KDB200_ABI_VERSION 2   /* 2: kdb_moe_w4a16_forward takes pw1 */

/* Tokens of one grouped expert-GEMM tile; the routing plan's mtile_start counts ceil(count / this). */
#define KDB_MOE_TOKEN_TILE 512

/* ---------------------------------------------------------------------------------------------- */
/* Library and status                                                                              */
/* ---------------------------------------------------------------------------------------------- */

/* ABI version (KDB200_ABI_VERSION). */
int kdb_abi_version(void);

/*
 * Process-wide cap on the SMs the persistent kernels launched after this call size their grids for
 * (0 = all SMs; values below 2 act as 2).  Returns the previous cap.  Use: leave SMs free for a
 * collective (NCCL all-to-all) that runs alongside the expert GEMMs; results do not depend on it.
 */
int kdb_set_sm_budget(int32_t sms);
int kdb_sm_budget(void);

/* Static string for a KDB_* status code. */
const char* kdb_strerror(int code);

/* The last CUDA error code recorded by a failing entry point on this host thread (0 if none). */
int kdb_last_cuda_error(void);

/*
 * Reads (and, if `clear` != 0, clears) the current device's status word: out[0] = first error code
 * (0 = none), out[1] = site id, out[2] = block index, out[3] = number of reports.  Synchronises the
 * given stream; call it outside timed regions.  Replaces the reference's debug-counter read-back of
 * its bounded spins (okc-challenge/engines/sc_h.cu:75-90), without the trap.
 */
int kdb_status_read(uint32_t out[4], int clear, void* stream);

/*
 * Self-test of the device failure path: one CTA waits, with a limit of limit_ns of global time
 * (1 us .. 2 s), on a barrier nothing arrives on, records KDB_ERR_TIMEOUT at site 0x1F0 in the device
 * status word, frees its tensor memory and returns, exactly as any kernel of the library does when
 * one of its bounded waits runs out.  Read the result with kdb_status_read.  No counterpart in the
 * reference, whose bounded spins count timeouts into a debug buffer (okc-challenge/engines/
 * sc_h.cu:75-90) that its tests never make run out.
 */
int kdb_selftest_wait_timeout(uint64_t limit_ns, void* stream);

/* ---------------------------------------------------------------------------------------------- */
/* bf16 dense projection                                                                           */
/* ---------------------------------------------------------------------------------------------- */

/*
 * Y[m, n] = sum_k X[m, k] * W[n, k]   (Y = X · Wᵀ), bf16 inputs, fp32 accumulation, bf16 output
 * rounded to nearest-even.
 *   x: bf16 [m, k] row-major, 16-byte aligned;  w: bf16 [n, k] row-major, 16-byte aligned;
 *   y: bf16 [m, n] with row stride ldy >= n elements (a column slice of a wider matrix is allowed).
 *   k % 8 == 0 (TMA row-stride rule).  m, n, k <= 2^30.  k == 0 writes zeros.
 * Replaces the body of `kernel_fn(data, state)` for the reference's `muse_bf16_proj` problem
 * (src/kdev/adapters/okc.py:534-537; src/kdev/adapters/okc_problems/muse_bf16_proj.toml:1-8).
 */
int kdb_proj_bf16(const void* x, const void* w, void* y, int64_t m, int64_t n, int64_t k, int64_t ldy,
                  void* stream);

/* Workspace bytes kdb_proj_bf16_ws can use for this shape: 0 for every shape.  Small-M (m <= 128,
 * weight-streaming) shapes split K over the CTAs of a thread-block cluster and sum the fp32 partials in
 * slice order through distributed shared memory inside the one launch, so no workspace is needed. */
size_t kdb_proj_workspace_bytes(int64_t m, int64_t n, int64_t k);

/* kdb_proj_bf16 with a workspace argument, kept for callers of the earlier two-launch K split; the
 * workspace is not used (results are deterministic either way). */
int kdb_proj_bf16_ws(const void* x, const void* w, void* y, int64_t m, int64_t n, int64_t k, int64_t ldy,
                     void* workspace, size_t workspace_bytes, void* stream);

/*
 * Projection with fp32 weights and fp32 output, for the reference's router layer ("fp32 weights and
 * output (BF16 hi+lo pair with FP32 accumulation allowed)", src/kdev/adapters/okc_problems/
 * muse_bf16_proj.toml:371; probe rows exact to 0.1%, :376).  Prepare once with kdb_proj_split_f32:
 * w fp32 [n, k] -> w_split bf16 [n, 2k] = [bf16(W) | bf16(W - bf16(W))] per row (each weight kept to
 * 2^-16 relative).  Then Y fp32 [m, n] (contiguous) = X · W_hiᵀ + X · W_midᵀ with fp32 accumulation;
 * k % 64 == 0, x and w_split 16-byte aligned.  m <= 128 runs the in-launch cluster K split of
 * kdb_proj_bf16; the workspace arguments are not used (kdb_proj_f32w_workspace_bytes is 0).
 */
int kdb_proj_split_f32(const float* w, void* w_split, int64_t n, int64_t k, void* stream);
size_t kdb_proj_f32w_workspace_bytes(int64_t m, int64_t n, int64_t k);
int kdb_proj_f32w(const void* x, const void* w_split, float* y, int64_t m, int64_t n, int64_t k, void* workspace,
                  size_t workspace_bytes, void* stream);

/* The output tile kdb_proj_bf16 picks for an m x n output on the current device: out[0] = tile width,
 * out[1] = 1 for 256-row tiles on CTA pairs, 0 for 128-row single-CTA tiles.  Host-only. */
int kdb_proj_tile_shape(int64_t m, int64_t n, int32_t out[2]);

/* As kdb_proj_bf16 with the output tile forced: tile_n 64, 128, 192, 224 or 256 with cta_pair 0
 * (128-row tiles, one CTA each), or tile_n 192, 224, 256 with cta_pair 1 (256-row tiles computed by
 * 2-CTA clusters); tile_n 0 with cta_pair 0 chooses automatically. */
int kdb_proj_bf16_cfg(const void* x, const void* w, void* y, int64_t m, int64_t n, int64_t k, int64_t ldy,
                      int tile_n, int cta_pair, void* stream);

/* ---------------------------------------------------------------------------------------------- */
/* Fused MoE layer                                                                                 */
/* ---------------------------------------------------------------------------------------------- */
/*
 * Layer:  logits = x · Wrᵀ (+ bias) (fp32);  ids = top-k(logits);  w = renormalised softmax over the
 * k picks;  y[t] = Σ_j w[t,j] · down_e( bf16( silu(x[t]·Wg_eᵀ) * (x[t]·Wu_eᵀ) ) ) (+ shared expert)
 * with e = ids[t,j].  Replaces the body of kernel_fn(data, state) for the reference's fused MoE
 * problem (`muse_moe_w4a16`: src/kdev/adapters/okc_problems/muse_moe_w4a16.toml; reference engines
 * okc-challenge/engines/sc_h.cu:189, x3_h.cu:311, x7_h.cu:310), for the bf16 SwiGLU layer with an
 * fp32 router inside the layer.
 *
 * Shapes: t tokens, h hidden (h % 8 == 0), e experts (k <= e <= 1024), i intermediate
 * (i % 128 == 0), k top-k (k <= 32), shared in {0, 1} always-on experts of intermediate shared_i
 * (shared_i % 128 == 0).  Weights: router fp32 [e, h], optional router_bias fp32 [e],
 * w_gate_up bf16 [e, 2i, h] (gate rows then up rows per expert) packed once with
 * kdb_moe_pack_gate_up, w_down bf16 [e, h, i], shared_* likewise with e = 1.
 */

/* Workspace bytes kdb_moe_forward needs for this shape (0 if the shape is unsupported). */
size_t kdb_moe_workspace_bytes(int64_t t, int64_t h, int64_t e, int64_t i, int64_t k, int64_t shared,
                               int64_t shared_i);

/*
 * One-time weight re-layout (the problem's `prepare(weights)`, okc.py:501-515): packed[e] holds, for
 * every 128-wide block b of the intermediate dimension, the 128 gate rows of block b followed by the
 * 128 up rows of block b, so one 256-wide GEMM tile carries matching gate and up columns.  Lossless
 * (a row permutation).  w_gate_up and packed: bf16 [e, 2i, h], distinct buffers.
 */
int kdb_moe_pack_gate_up(const void* w_gate_up, void* packed, int64_t e, int64_t i, int64_t h, void* stream);

/*
 * Router stage alone: logits fp32 [t, e] (each the fixed-order fp64 dot product rounded once to
 * fp32, plus bias), topk_ids int32 [t, k] (descending logit; ties -> lower expert), topk_w fp32
 * [t, k] renormalised softmax weights.  Routing plan counterpart: x3_h.cu:346-385.
 */
int kdb_moe_route(const void* x, const float* router_w, const float* router_bias, float* logits, float* topk_w,
                  int32_t* topk_ids, int64_t t, int64_t h, int64_t e, int64_t k, void* stream);

/* Scratch bytes of kdb_moe_plan. */
size_t kdb_moe_plan_workspace_bytes(int64_t t, int64_t e, int64_t k);

/*
 * Permutation plan alone: counts int32 [e], offsets int32 [e + 1] (exclusive scan), perm_slot int32
 * [t*k] (slot t*k + j held by each permuted row; rows grouped by expert, tokens ascending within an
 * expert), slot_pos int32 [t*k] (inverse).  Counterpart of the per-expert mask/popc/scan plan of
 * x3_h.cu:346-385, for any t.
 */
int kdb_moe_plan(const int32_t* topk_ids, const float* topk_w, int64_t t, int64_t e, int64_t k, int32_t* counts,
                 int32_t* offsets, int32_t* perm_slot, int32_t* slot_pos, void* workspace, size_t workspace_bytes,
                 void* stream);

/*
 * The permutation plan of kdb_moe_plan without a caller workspace.  No counterpart in the
 * reference: an addition for callers that cannot allocate device memory (a runtime that reserves
 * all memory at start-up and reaches this library through a C FFI, or code that must not call
 * cudaMalloc), who pass only their inputs and outputs.  Its scratch is a fixed 1,577,216-byte array
 * inside the library (held on every GPU that loads it until exit); limits t*k <= 131072,
 * e <= 1024, ceil(t/256)*e <= 65536, else KDB_ERR_UNSUPPORTED.  The first call on a device resolves
 * the array's address (a runtime call): make it before any stream capture.  The address is cached for
 * the life of the process; a caller that resets a device (cudaDeviceReset, or tearing down and
 * re-creating its primary context) must not call this entry point on that device afterwards.  Calls
 * share the array: calls that overlap on the GPU race, so issue them on one stream.  Outputs as
 * kdb_moe_plan.
 */
int kdb_moe_plan_noalloc(const int32_t* topk_ids, const float* topk_w, int64_t t, int64_t e, int64_t k,
                         int32_t* counts, int32_t* offsets, int32_t* perm_slot, int32_t* slot_pos, void* stream);

/*
 * One-time router preparation for the tensor-core routing path: router_split bf16 [e, 2h] receives
 * [bf16(W) | bf16(W - bf16(W))] per expert row and router_norms fp32 [e] an upper bound of each
 * row's 2-norm.  Lossless for the layer (router_w itself stays the source of the exact logits).
 */
int kdb_moe_prepare_router(const float* router_w, void* router_split, float* router_norms, int64_t e, int64_t h,
                           void* stream);

/* approx fp32 [t, e] = x · [W_hi | W_mid]ᵀ on the tensor cores (h % 64 == 0): the routing pre-pass. */
int kdb_moe_router_approx(const void* x, const void* router_split, float* approx, int64_t t, int64_t h, int64_t e,
                          void* stream);

/* Scratch bytes of kdb_moe_route_fast. */
size_t kdb_moe_route_fast_workspace_bytes(int64_t t, int64_t e);

/*
 * Router stage on the tensor-core path: ids and weights identical to kdb_moe_route (the candidates
 * of a rigorous error bound around the k-th approximate logit are recomputed in the fixed fp64
 * order), without computing every fp64 logit.  h % 64 == 0.  Counterpart of the routing plan's
 * top-k read (x3_h.cu:346-365) with the router inside the layer.
 */
int kdb_moe_route_fast(const void* x, const float* router_w, const float* router_bias, const void* router_split,
                       const float* router_norms, float* topk_w, int32_t* topk_ids, int64_t t, int64_t h, int64_t e,
                       int64_t k, void* workspace, size_t workspace_bytes, void* stream);

/* ---- Stage entry points (composition, expert parallelism) ----------------------------------- */

/* out[r, :] = x[index[r] / div, :] for r < rows (x bf16 [t, h], h % 8 == 0); a bad index is reported
 * in the device status word (KDB_ERR_DEVICE_BOUNDS) and its row is skipped.  With index = perm_slot
 * and div = k this lays a token batch out in the plan's expert order. */
int kdb_moe_gather_rows(const void* x, const int32_t* index, int64_t div, void* out, int64_t rows, int64_t h,
                        int64_t t, void* stream);

/*
 * Grouped SwiGLU gate_up: for each group g, rows [offsets[g], offsets[g+1]) of a (bf16 [a_rows, h])
 * times packed w_gate_up[g] (bf16 [2i, h], from kdb_moe_pack_gate_up), epilogue silu(gate) * up ->
 * out bf16 [a_rows, i].  offsets / mtile_start (int32 [groups + 1], mtile_start = exclusive prefix of
 * ceil(count / KDB_MOE_TOKEN_TILE), as kdb_moe_plan / kdb_moe_ep_regroup produce) are read on the device; both NULL
 * means one dense group of a_rows rows.  Counterpart: the gate_up stage + SwiGLU epilogue warp of the
 * reference engines (okc-challenge/engines/sc_h.cu:164-187, 322-340).
 */
int kdb_moe_expert_gate_up(const void* a, int64_t a_rows, const void* w_gate_up_packed, int64_t groups, int64_t i,
                           int64_t h, const int32_t* offsets, const int32_t* mtile_start, void* out, void* stream);

/*
 * Grouped down projection: rows of a (bf16 [a_rows, i]) times w_down[g] (bf16 [h, i]) -> out bf16
 * [a_rows, h], each row scaled by row_scale[row] when row_scale is not NULL.  Grouping as above.
 * Counterpart: the down stage of the reference engines (sc_h.cu:341-381, x7_h.cu:438-590).
 */
int kdb_moe_expert_down(const void* a, int64_t a_rows, const void* w_down, int64_t groups, int64_t i, int64_t h,
                        const int32_t* offsets, const int32_t* mtile_start, const float* row_scale, void* out,
                        void* stream);

/*
 * Grouped down projection with the weighted combine merged into its epilogue, in one launch: rows_out
 * receives the scaled per-slot rows as kdb_moe_expert_down writes them (row_scale required), and each
 * tile, once its accumulator is released, counts one arrival per row on (token, 128-feature block); the
 * tile completing a block sums that block's k slot rows in slot order (+ shared_rows[t]) into y bf16
 * [t, h], bitwise as kdb_moe_combine does.  perm_slot / slot_pos from kdb_moe_plan; h % 128 == 0;
 * workspace >= kdb_moe_expert_down_combine_workspace_bytes(t, h) (arrival counters, zeroed here).
 * Counterpart of the engines' down stage with its combine (okc-challenge/engines/sc_h.cu:341-381).
 * kdb_moe_forward does not use it: measured on B200 the layer is faster with the separate combine.
 */
size_t kdb_moe_expert_down_combine_workspace_bytes(int64_t t, int64_t h);
int kdb_moe_expert_down_combine(const void* a, int64_t a_rows, const void* w_down, int64_t groups, int64_t i, int64_t h,
                                const int32_t* offsets, const int32_t* mtile_start, const float* row_scale,
                                const int32_t* perm_slot, const int32_t* slot_pos, const void* shared_rows,
                                void* rows_out, void* y, int64_t t, int64_t k, void* workspace,
                                size_t workspace_bytes, void* stream);

/*
 * Weighted combine: y[t] = sum_j (slot_w[t*k+j] or 1) * rows[slot_pos[t*k+j]] (+ shared_rows[t]),
 * summed in fp32 in slot order (deterministic), bf16 out.  slot_w NULL: rows are already scaled.
 * Counterpart: the weighted combine of the reference engines (sc_h.cu:374-381).
 */
int kdb_moe_combine(const void* rows, const int32_t* slot_pos, const float* slot_w, const void* shared_rows, void* y,
                    int64_t t, int64_t h, int64_t k, void* stream);

/* Scratch bytes of kdb_moe_ep_regroup. */
size_t kdb_moe_ep_regroup_workspace_bytes(int64_t p, int64_t er);

/*
 * Expert-parallel regroup on an expert's owner rank.  counts int32 [p, er] (device): rows received from
 * source rank s for local expert e.  to_expert_major != 0 copies rows from source-major blocks (s, e)
 * (the all-to-all receive order) to expert-major order (what the grouped GEMMs read); 0 copies back.
 * Always writes the expert-major offsets int32 [er + 1] and mtile_start int32 [er + 1]; in/out may
 * both be NULL for the tables alone.  No host synchronisation.  No counterpart in the reference, whose
 * engines simulate a single expert-parallel rank (okc_problems/muse_moe_w4a16.toml:136).
 */
int kdb_moe_ep_regroup(const int32_t* counts, int64_t p, int64_t er, int to_expert_major, const void* in, void* out,
                       int64_t h, int32_t* offsets, int32_t* mtile_start, void* workspace, size_t workspace_bytes,
                       void* stream);

/*
 * The whole layer.  x bf16 [t, h]; y bf16 [t, h]; topk_w fp32 [t, k]; topk_ids int32 [t, k] (the
 * routing outputs the reference's routing problems report at output index 2,
 * src/kdev/adapters/okc_problems/muse_prefill_layer.toml:148).  workspace: >= kdb_moe_workspace_bytes,
 * 256-byte aligned.  shared_gate_up_packed / shared_down may be NULL when shared == 0.
 * router_split / router_norms (from kdb_moe_prepare_router) select the tensor-core routing path;
 * NULL computes every logit in the fixed fp64 order.  Both give identical ids and weights.
 */
int kdb_moe_forward(const void* x, const float* router_w, const float* router_bias, const void* router_split,
                    const float* router_norms, const void* w_gate_up_packed,
                    const void* w_down, const void* shared_gate_up_packed, const void* shared_down, void* y,
                    float* topk_w, int32_t* topk_ids, int64_t t, int64_t h, int64_t e, int64_t i, int64_t k,
                    int64_t shared, int64_t shared_i, void* workspace, size_t workspace_bytes, void* stream);

/*
 * NVFP4 w4a16 MoE layer of one expert-parallel rank (the reference's muse_moe_w4a16 problem,
 * src/kdev/adapters/okc_problems/muse_moe_w4a16.toml; engines okc-challenge/engines/sc_h.cu:189-467).
 * x bf16 [t, h]; topk_ids int32 / topk_w fp32 [t, k] over e_total experts, of which ids 0..local-1 live
 * here (routes to other ids are skipped); y bf16 [t, h] = sum over local routes j of
 * y_j * topk_w * rsqrt(mean(y_j^2) + 1e-8), y_j = (bf16(silu(x.W1^T gs13) * (x.W3^T gs13)) . W2^T) gs2 pw1
 * kept in fp32, pw1 fp32 [h] the per-feature output weight of the reference engines' Params.pw1
 * (okc-challenge/engines/sc_h.cu:51, 346; NULL = 1).  Weights NVFP4 (E2M1 codes two per byte, low nibble first; E4M3 scale per
 * 16 elements; fp32 global scale per expert tensor), as 9216-byte blocks, one per (expert, weight tile,
 * 64-element k chunk), tiles and chunks in order: [part 0 codes 128 x 32 B | part 1 codes | part 0 scales
 * 128 x 4 B | part 1 scales].  w13_blocks [local][i/128][h/64]: tile f's part 0 = gate rows 128f.., part 1
 * = up rows i + 128f..; w2_blocks [local][h/256][i/64]: parts = output rows 256f.. and 256f + 128..;
 * gscales fp32 [local].  h % 256 == 0, h <= 8192, i % 128 == 0.  workspace >= kdb_moe_w4a16_workspace_bytes,
 * 256-byte aligned.
 */
size_t kdb_moe_w4a16_workspace_bytes(int64_t t, int64_t h, int64_t i, int64_t local, int64_t e_total, int64_t k);
int kdb_moe_w4a16_forward(const void* x, const int32_t* topk_ids, const float* topk_w, const void* w13_blocks,
                          const float* w13_gscale, const void* w2_blocks, const float* w2_gscale, const float* pw1,
                          void* y, int64_t t, int64_t h, int64_t i, int64_t local, int64_t e_total, int64_t k,
                          void* workspace, size_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------------------------------------- */
/* FP8-KV paged decode / verify attention                                                          */
/* ---------------------------------------------------------------------------------------------- */

/*
 * Replaces the body of kernel_fn(data) for the reference's `muse_attention_decode` problem
 * (src/kdev/adapters/okc_problems/muse_attention_decode.toml: shapes, tests, [comply] notes).
 * q bf16 [batch, q_len, q_heads, head_dim]; k_new / v_new bf16 [batch, q_len, kv_heads, head_dim];
 * k_cache / v_cache float8 e4m3 [slots, kv_heads, head_dim] (value = e4m3 * kv_scale); block_table int32
 * [batch, max_len], the cache slot of every token (page size 1); seq_lens int32 [batch], tokens per
 * sequence after the append (the new tokens are positions L - q_len .. L - 1, q_len <= L <= max_len).
 * First writes the new tokens' K/V into their slots (e4m3 of value / kv_scale, nearest-even, saturating
 * at +-448), then out bf16 [batch, q_len, q_heads, head_dim] = softmax(q K^T / sqrt(head_dim)) V per
 * query head over its KV head's keys j <= p (p the query's position), and j > p - window when window > 0
 * (a sliding layer: window 2048), 0 for the whole context.  head_dim == 128, q_heads % kv_heads == 0,
 * q_len * q_heads / kv_heads <= 64.  q, caches, k_new, v_new, out 16-byte aligned; workspace >=
 * kdb_attn_decode_workspace_bytes, 256-byte aligned.  A length or slot out of range is reported in the
 * device status word (KDB_ERR_DEVICE_BOUNDS).  Graph capturable; no host synchronisation.
 */
size_t kdb_attn_decode_workspace_bytes(int64_t batch, int64_t q_len, int64_t q_heads, int64_t kv_heads,
                                       int64_t max_len, int64_t window);
int kdb_attn_decode_fp8(const void* q, const void* k_new, const void* v_new, void* k_cache, void* v_cache,
                        const int32_t* block_table, const int32_t* seq_lens, float kv_scale, void* out,
                        int64_t batch, int64_t q_len, int64_t q_heads, int64_t kv_heads, int64_t head_dim,
                        int64_t max_len, int64_t slots, int64_t window, void* workspace, size_t workspace_bytes,
                        void* stream);

#ifdef __cplusplus
}
#endif

#endif /* KDB200_H */

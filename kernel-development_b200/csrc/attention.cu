// attention.cu — paged decode / verify attention over an FP8 E4M3 KV cache: the `muse_attention_decode` problem
// of the reference (src/kdev/adapters/okc_problems/muse_attention_decode.toml: batch 1-48, context up to 80k
// (1M in a test), q_len 1 (decode) or 8 (verify), sliding (2,048 keys) or full layers, page size 1, kv_scale,
// "kernel_fn writes the new FP8 cache entries into k_cache / v_cache").
//
// Tensors: q [B, T, Hq, 128] bf16; k_new / v_new [B, T, Hkv, 128] bf16; k_cache / v_cache [slots, Hkv, 128] e4m3
// (value = e4m3 x kv_scale); block_table [B, max_len] int32, the cache slot of every token (page = 1);
// seq_lens [B] int32, tokens after the append (the new ones are positions L - T .. L - 1).  Query row
// r = t * group + h of KV head g is query head g * group + h of token t (group = Hq / Hkv, R = T * group <= 64).
//
// Three launches:
//   attn_append_kernel   the new tokens' K/V, fp8 of value / kv_scale (round to nearest even, saturating at
//                        +-448), written into their slots;
//   attn_fwd_kernel      persistent, warp-specialised: the tiles of 128 keys of every (sequence, KV head) form
//                        one sequence, split evenly over the CTAs.  Producer warps copy a tile's K and V rows
//                        (128 B each, found through the block table) into a ring of stages with 16-byte cp.async
//                        copies, laid out with the 128-byte swizzle; one thread issues S^T = K Q^T (tcgen05
//                        kind::f8f6f4, M = 128 keys, N = 16 / 64 query rows, K = 128 dims, the fp8 cache read as
//                        it is stored); 8 or 16 softmax warps read S^T from tensor memory (thread = key), take the
//                        tile's row maxima across the 128 keys and write P^T as e4m3, and the MMA thread
//                        accumulates O^T += V^T P^T (M = 128 dims; V and P^T both MN-major, V straight from the
//                        cache rows) in tensor memory.  Queries and probabilities go in as two e4m3 terms each
//                        (x = hi + lo, the residual about 2^-8 of x), so the products carry about bf16 precision
//                        while both MMAs read the fp8 cache directly.  The running maximum is raised lazily (only
//                        when a tile's maximum exceeds it by more than 2^4), which bounds every probability by
//                        2^8 in e4m3 and rescales O^T in tensor memory rarely.  At the end of a CTA's stretch of
//                        one (sequence, KV head) the unnormalised O, row sums and maxima go to a partial slot;
//   attn_merge_kernel    per query row, the partials of the CTAs that covered its keys, merged exactly.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>

#include "gemm_sm100.cuh"
#include "host_util.h"
#include "sm100_common.cuh"

namespace kdb {

constexpr int kAttnD = 128;          // head dim
constexpr int kAttnTile = 128;       // keys per tile = TMEM lanes of S^T
constexpr int kAttnMaxCtas = 1024;   // partial slots reserved for CTAs (workspace bound)
constexpr int kAttnMaxRows = 64;     // T * group

enum : unsigned int {
  kSiteAttnProdEmpty = 0x1A1,
  kSiteAttnMmaFull = 0x1A2,
  kSiteAttnMmaQ = 0x1A3,
  kSiteAttnMmaSFree = 0x1A4,
  kSiteAttnMmaP = 0x1A5,
  kSiteAttnMmaOFree = 0x1A6,
  kSiteAttnSoftS = 0x1A7,
  kSiteAttnSoftPv = 0x1A8,
  kSiteAttnDrainMma = 0x1AA,
  kSiteAttnLen = 0x1AB,
  kSiteAttnSlot = 0x1AC,
  kSiteAttnAppend = 0x1AD,
  kSiteAttnMeta = 0x1AE,
};

struct AttnParams {
  const __nv_bfloat16* q;   // [B, T, Hq, 128]
  const uint8_t* k_cache;   // [slots, Hkv, 128] e4m3
  const uint8_t* v_cache;
  const int* block_table;   // [B, max_len]
  const int* seq_lens;      // [B]
  float score_scale;        // kv_scale / sqrt(128) * log2(e)
  int B, T, Hq, Hkv, group, R, max_len, window;
  long long slots;          // cache slots
  float* part_m;            // [slot][R]  running maximum (log2 units)
  float* part_l;            // [slot][R]  sum of probabilities
  float* part_o;            // [slot][R][128] unnormalised output (x 1 / kv_scale)
  int* meta;                // [B * Hkv][2]: first and last CTA of every (sequence, KV head)
};

// Length of sequence b, clamped into [T, max_len] (a length outside is reported: its attention is undefined).
__device__ __forceinline__ int attn_len(const AttnParams& p, int b) {
  int L = __ldg(p.seq_lens + b);
  if (L < p.T || L > p.max_len) {
    report(KDB_ERR_DEVICE_BOUNDS, kSiteAttnLen);
    L = L < p.T ? p.T : p.max_len;
  }
  return L;
}
// First key of sequence b's window union (the lowest key any of its T query rows attends).
__device__ __forceinline__ int attn_lo(const AttnParams& p, int L) {
  return p.window > 0 ? max(0, L - p.T - p.window + 1) : 0;
}
__device__ __forceinline__ int attn_tiles_of(const AttnParams& p, int L) {
  return (L - attn_lo(p, L) + kAttnTile - 1) / kAttnTile;
}

// Walks this CTA's tiles: (sequence b, KV head g, tile) in b-major, g, tile order.
struct AttnCursor {
  int b, g, tile, ntiles, L, lo;
  int remaining;   // tiles left, the current one included
  int seg;         // segment (one (b, g) stretch) index within the CTA
  bool seg_start, seg_end;

  __device__ void load_b(const AttnParams& p) {
    L = attn_len(p, b);
    lo = attn_lo(p, L);
    ntiles = (L - lo + kAttnTile - 1) / kAttnTile;
  }
  __device__ void init(const AttnParams& p, int b0, int g0, int t0, int count) {
    b = b0;
    g = g0;
    tile = t0;
    remaining = count;
    seg = 0;
    load_b(p);
    seg_start = true;
    seg_end = remaining == 1 || tile == ntiles - 1;
  }
  __device__ void next(const AttnParams& p) {
    --remaining;
    if (remaining <= 0) return;
    if (++tile == ntiles) {
      tile = 0;
      if (++g == p.Hkv) {
        g = 0;
        ++b;
        load_b(p);
      }
      ++seg;
    }
    seg_start = tile == 0;
    seg_end = remaining == 1 || tile == ntiles - 1;
  }
  // Jump to the first tile of the next segment; false when this was the CTA's last segment.
  __device__ bool next_segment(const AttnParams& p) {
    const int left_in_seg = ntiles - tile;
    if (remaining <= left_in_seg) return false;
    remaining -= left_in_seg - 1;
    tile = ntiles - 1;
    next(p);
    return true;
  }
};

// NQ: MMA N (query-row columns, 16 or 64); ROWS: query rows the softmax threads handle (R <= ROWS <= NQ);
// SPLIT: softmax warp groups, each taking ROWS / SPLIT rows of every key; STAGES: K/V ring depth; NPROD: producer
// warps (one warp's cp.async stream reaches about 1.4 TB/s of random 128-byte rows over 148 SMs; four, about 3).
template <int NQ, int ROWS, int SPLIT, int STAGES, int NPROD>
struct AttnLayout {
  static constexpr int kSoftThreads = 128 * SPLIT;
  static constexpr int kThreads = kSoftThreads + 32 * (NPROD + 1);   // + producer warps + MMA warp
  // the bound given to the compiler: the threads rounded up to whole groups of four warps, so that the registers of
  // the warps on one SM sub-partition (at most one warp in four) fit its 16K (65536 / kLaunchBound per thread)
  static constexpr int kLaunchBound = (kThreads + 127) / 128 * 128;
  static constexpr int kRpt = ROWS / SPLIT;            // query rows per softmax thread
  static constexpr int kPf = STAGES - 2;               // tiles of copies in flight
  static constexpr int kKvBytes = kAttnTile * kAttnD;  // 16 KB: 128 rows of 128 B
  static constexpr int kStageBytes = 2 * kKvBytes;     // K tile, then V tile
  static constexpr int kQBytes = NQ * kAttnD;          // one e4m3 term of Q (or of P^T: NQ rows x 128 keys)
  static constexpr int kQOffset = STAGES * kStageBytes;             // Q[buffer][hi, lo]
  static constexpr int kPOffset = kQOffset + 4 * kQBytes;           // P^T[buffer][hi, lo]
  // kMmaL: the row sums come from the tensor cores (a tile of e4m3 ones times P^T into TMEM columns beside O^T)
  // and the probabilities are computed in f16 pairs; the conversion / transcendental pipe limits many rows.
  static constexpr bool kMmaL = ROWS > 16;
  static constexpr int kOnesOffset = kPOffset + 4 * kQBytes;        // [128][128] e4m3 ones (kMmaL)
  static constexpr int kXchOffset = kOnesOffset + (kMmaL ? kKvBytes : 0);   // row maxima [2][ROWS][4]
  static constexpr int kLsumOffset = kXchOffset + 2 * ROWS * 4 * 4;   // row sums [ROWS][4]
  static constexpr int kRowmaxOffset = kLsumOffset + ROWS * 4 * 4;    // |q| maximum per row [2][ROWS]
  static constexpr int kRowtOffset = kRowmaxOffset + 2 * ROWS * 4;    // token of each row [ROWS]
  static constexpr int kBtOffset = kRowtOffset + ROWS * 4;            // block-table rings [NPROD][kPf][128]
  static constexpr int kBarOffset = kBtOffset + NPROD * kPf * kAttnTile * 4;
  // kv_full[S], kv_empty[S], s_full[2], s_free[2], p_full[2], pv_done[2], q_full[2], o_free, drain
  static constexpr int kNumBars = 2 * STAGES + 12;
  static constexpr int kMiscOffset = kBarOffset + kNumBars * 8;   // tmem slot, abort flag, scan scratch
  static constexpr int kMiscInts = 48;
  static constexpr int kSmemBytes = kMiscOffset + kMiscInts * 4 + 1024;
  static constexpr int kCols = (kMmaL ? 4 : 3) * NQ;
  static constexpr uint32_t kTmemCols = kCols <= 64 ? 64 : (kCols <= 128 ? 128 : 256);
  // TMEM columns: S^T buffers [0, NQ) and [NQ, 2 NQ); O^T [2 NQ, 3 NQ); row sums [3 NQ, 4 NQ) (kMmaL)
  static_assert(kCols <= 256, "tensor memory columns");
  static_assert(ROWS % SPLIT == 0 && ROWS <= NQ && (kRpt == 2 || kRpt == 4 || kRpt == 8 || kRpt == 16 || kRpt == 32),
                "rows per thread");
  static_assert(kThreads <= 1024 && kPf >= 1 && NPROD >= 1 && NPROD <= 8, "launch shape");
  static_assert(kSmemBytes <= 232448, "shared memory");
};

// kind::f8f6f4, e4m3 x e4m3 -> f32, M = m, N = n; A K-major (scores) or MN-major (values: V^T), B K-major.
__host__ __device__ constexpr uint32_t idesc_e4m3_f32(int m, int n, bool a_mn_major, bool b_mn_major) {
  return (1u << 4)                                   // D format: f32
         | (0u << 7)                                 // A format: e4m3
         | (0u << 10)                                // B format: e4m3
         | (a_mn_major ? (1u << 15) : 0u)            // A major
         | (b_mn_major ? (1u << 16) : 0u)            // B major
         | (static_cast<uint32_t>(n >> 3) << 17)     // N / 8
         | (static_cast<uint32_t>(m >> 4) << 24);    // M / 16
}

// Descriptor of an MN-major operand stored as rows of 128 B (one row per K index, 128 e4m3 along M) with the
// 128-byte swizzle: K groups of 8 rows 1024 B apart; M spans one 128-byte atom.
__device__ __forceinline__ uint64_t sdesc_sw128_mnmajor(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu);   // start address
  d |= static_cast<uint64_t>(8192u >> 4) << 16;              // leading byte offset: next 128-byte M atom (unused)
  d |= static_cast<uint64_t>(1024u >> 4) << 32;              // stride byte offset: next 8 K rows
  d |= static_cast<uint64_t>(1u) << 46;                       // descriptor version (sm_100)
  d |= static_cast<uint64_t>(2u) << 61;                       // layout: 128-byte swizzle
  return d;
}

__device__ __forceinline__ void mma_e4m3(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Bounded mbarrier wait whose polls suspend the thread (up to 20 us each, woken when the phase completes), so
// waiting warps leave the issue slots to the working ones; same contract as mbar_wait (abort flag, 2 s limit,
// status word on timeout).
__device__ __forceinline__ bool attn_test(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(20000u)
      : "memory");
  return ok != 0u;
}
__device__ __forceinline__ bool attn_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag, unsigned int site) {
  if (attn_test(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  while (true) {
    if (attn_test(bar, parity)) return true;
    if (*abort_flag) return false;
    if (globaltimer() - t0 > KDB_WAIT_NS) {
      report(KDB_ERR_TIMEOUT, site);
      *abort_flag = 1;
      return false;
    }
  }
}

// Programmatic dependent launch: let the next kernel of the stream start its prologue now / wait until the previous
// kernel's grid has completed and its writes are visible (a no-op when launched without the attribute).
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

__device__ __forceinline__ void soft_bar_sync(int nthreads) {
  asm volatile("bar.sync 1, %0;" ::"r"(nthreads) : "memory");
}
__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}
// Named barrier `id` over `nthreads` threads that ORs / ANDs a predicate over them.
__device__ __forceinline__ bool named_bar_or(int id, int nthreads, bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.or.pred q, %2, %3, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(static_cast<uint32_t>(v)), "r"(id), "r"(nthreads)
      : "memory");
  return r != 0u;
}
__device__ __forceinline__ bool named_bar_and(int id, int nthreads, bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.and.pred q, %2, %3, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(static_cast<uint32_t>(v)), "r"(id), "r"(nthreads)
      : "memory");
  return r != 0u;
}
// Named barrier of the softmax warps that also ORs a predicate over them.
__device__ __forceinline__ bool soft_bar_or(int nthreads, bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.or.pred q, 1, %2, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(static_cast<uint32_t>(v)), "r"(nthreads)
      : "memory");
  return r != 0u;
}
// Named barrier of the softmax warps that also ANDs a predicate over them.
__device__ __forceinline__ bool soft_bar_and(int nthreads, bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.and.pred q, 1, %2, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(static_cast<uint32_t>(v)), "r"(nthreads)
      : "memory");
  return r != 0u;
}

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float warp_max_f32(float x) {
  float r;
  asm volatile("redux.sync.max.f32 %0, %1, 0xffffffff;" : "=f"(r) : "f"(x));
  return r;
}

// 4 x 4 byte transpose across the four lanes of an aligned lane quad: lane e holds bytes x[e][0..3] and receives
// x[0..3][e] (byte k of the result from lane k).
__device__ __forceinline__ uint32_t quad_transpose(uint32_t x, int e) {
  const uint32_t p1 = __shfl_xor_sync(0xffffffffu, x, 1);
  const uint32_t y = (e & 1) ? __byte_perm(x, p1, 0x3715) : __byte_perm(x, p1, 0x6240);
  const uint32_t p2 = __shfl_xor_sync(0xffffffffu, y, 2);
  return (e & 2) ? __byte_perm(y, p2, 0x3276) : __byte_perm(y, p2, 0x5410);
}

__device__ __forceinline__ float warp_sum_f32(float v) {
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  return v;
}

// tcgen05.ld / st of N consecutive 32-bit columns of this warp's 32 lanes (shape 32x32b): thread i has lane
// (lane base + i), columns [col, col + N).
template <int N>
__device__ __forceinline__ void tmem_ld_cols(uint32_t taddr, uint32_t (&r)[N]);
template <int N>
__device__ __forceinline__ void tmem_st_cols(uint32_t taddr, const uint32_t (&r)[N]);
template <>
__device__ __forceinline__ void tmem_ld_cols<2>(uint32_t taddr, uint32_t (&r)[2]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x2.b32 {%0, %1}, [%2];" : "=r"(r[0]), "=r"(r[1]) : "r"(taddr) : "memory");
}
template <>
__device__ __forceinline__ void tmem_ld_cols<4>(uint32_t taddr, uint32_t (&r)[4]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(taddr)
               : "memory");
}
template <>
__device__ __forceinline__ void tmem_ld_cols<8>(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr)
               : "memory");
}
template <>
__device__ __forceinline__ void tmem_ld_cols<16>(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}
template <>
__device__ __forceinline__ void tmem_ld_cols<32>(uint32_t taddr, uint32_t (&r)[32]) {
  tmem_ld_32x32b_x32(taddr, r);
}
template <>
__device__ __forceinline__ void tmem_st_cols<32>(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
      "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]),
      "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),
      "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31]), "r"(r[32])
      : "memory");
}
template <>
__device__ __forceinline__ void tmem_st_cols<2>(uint32_t taddr, const uint32_t (&r)[2]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x2.b32 [%0], {%1, %2};" ::"r"(taddr), "r"(r[0]), "r"(r[1]) : "memory");
}
template <>
__device__ __forceinline__ void tmem_st_cols<4>(uint32_t taddr, const uint32_t (&r)[4]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1, %2, %3, %4};" ::"r"(taddr), "r"(r[0]), "r"(r[1]),
               "r"(r[2]), "r"(r[3])
               : "memory");
}
template <>
__device__ __forceinline__ void tmem_st_cols<8>(uint32_t taddr, const uint32_t (&r)[8]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(taddr),
               "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
               : "memory");
}
template <>
__device__ __forceinline__ void tmem_st_cols<16>(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

// 16-byte asynchronous global -> shared copy, L1 bypassed (cp.async groups).
__device__ __forceinline__ void cp_async_16(void* smem_dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem_dst)), "l"(src) : "memory");
}
// 4-byte asynchronous global -> shared copy (cp.async groups).
__device__ __forceinline__ void cp_async_4(void* smem_dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(smem_dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ uint8_t e4m3_of(float x) {
  return static_cast<uint8_t>(__nv_cvt_float_to_fp8(x, __NV_SATFINITE, __NV_E4M3));
}
__device__ __forceinline__ float f32_of_e4m3(uint8_t v) {
  const __half_raw h = __nv_cvt_fp8_to_halfraw(static_cast<__nv_fp8_storage_t>(v), __NV_E4M3);
  return __half2float(__half(h));
}

// Byte offset of element (row, col) of a [rows][128 B] tile with the 128-byte swizzle (1024-byte aligned base).
__device__ __forceinline__ int sw128_offset(int row, int col) {
  return (row >> 3) * 1024 + (row & 7) * 128 + ((((col >> 4) ^ row) & 7) << 4) + (col & 15);
}

// Block-wide inclusive scan over every thread of the CTA (blockDim.x a multiple of 32, at most 32 warps);
// *total = the sum over the block.
__device__ __forceinline__ int block_incl_scan(int v, int* warp_sums, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) warp_sums[warp] = x;
  __syncthreads();
  int before = 0, all = 0;
  for (int w = 0; w < nwarps; ++w) {
    const int s = warp_sums[w];
    if (w < warp) before += s;
    all += s;
  }
  __syncthreads();
  *total = all;
  return x + before;
}

// The CTA's stretch of the global tile sequence: [t_begin, t_end) of N tiles split evenly over min(gridDim.x, N)
// CTAs.  Returns the tile count; (b0, g0, t0) locate the first tile.  Every thread of the CTA takes part.
__device__ int attn_locate(const AttnParams& p, int* scratch, int* b0, int* g0, int* t0) {
  int* warp_sums = scratch;   // [32]
  int* found = scratch + 32;  // [3]
  const int tid = threadIdx.x;
  const bool one_chunk = p.B <= static_cast<int>(blockDim.x);   // the first pass's scan can be reused
  int total = 0, my_tiles = 0, my_incl = 0;
  for (int base = 0; base < p.B; base += blockDim.x) {
    const int b = base + tid;
    my_tiles = b < p.B ? attn_tiles_of(p, attn_len(p, b)) : 0;
    int chunk;
    my_incl = block_incl_scan(my_tiles * p.Hkv, warp_sums, &chunk);
    total += chunk;
  }
  // the first min(grid, N) CTAs take the work, so every working CTA has at least one tile and the CTAs that
  // cover one (sequence, KV head) form a gapless range (the merge reads one partial from each)
  const long long n = total, c = blockIdx.x, C = gridDim.x < n ? gridDim.x : n;
  if (c >= C) return 0;
  const int t_begin = static_cast<int>(c * n / C), t_end = static_cast<int>((c + 1) * n / C);
  if (tid == 0) found[0] = -1;
  __syncthreads();
  int running = 0;
  for (int base = 0; base < p.B; base += blockDim.x) {
    const int b = base + tid;
    int tiles = my_tiles, incl = my_incl, chunk = total;
    if (!one_chunk) {
      tiles = b < p.B ? attn_tiles_of(p, attn_len(p, b)) : 0;
      incl = block_incl_scan(tiles * p.Hkv, warp_sums, &chunk);
    }
    const int v = tiles * p.Hkv;
    const int excl = incl - v;
    if (v > 0 && running + excl <= t_begin && t_begin < running + incl) {
      const int off = t_begin - running - excl;
      found[0] = b;
      found[1] = off / tiles;
      found[2] = off % tiles;
    }
    running += chunk;
    __syncthreads();
    if (found[0] >= 0) break;
  }
  *b0 = found[0];
  *g0 = found[1];
  *t0 = found[2];
  return found[0] >= 0 ? t_end - t_begin : 0;
}

// Q rows of (b, g) as two e4m3 terms with one power-of-two scale s for the segment, chosen so the largest |q| of its
// rows lands in [128, 256): Qhi = e4m3(q s), Qlo = e4m3(q s - Qhi), into the swizzled [NQ][128 B] tiles; returns
// score_scale / s (the same in every thread).  Run by all softmax threads (one named barrier); each fences its
// writes for the tensor cores.  rowmax: this Q buffer's [ROWS] scratch.  BAR: the named barrier used; tid: the
// thread's index among the SOFT_THREADS taking part; dup > 0: both terms are written a second time dup bytes on.
template <int SOFT_THREADS, int ROWS, int BAR = 1>
__device__ float attn_prepare_q_t(const AttnParams& p, int tid, int b, int g, uint8_t* qhi, uint8_t* qlo,
                                  float* rowmax, int dup = 0) {
  const int items = p.R * 16;   // R rows x 16 pieces of 8 dims; a row's 16 pieces sit in one half-warp
  auto load = [&](int item, float (&x)[8]) {
    const int r = item >> 4, piece = item & 15;
    const int t = r / p.group, h = r - t * p.group;
    const uint4 raw = __ldg(reinterpret_cast<const uint4*>(
        p.q + ((static_cast<long long>(b) * p.T + t) * p.Hq + g * p.group + h) * kAttnD + piece * 8));
    const __nv_bfloat162* v2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = __bfloat1622float2(v2[e]);
      x[2 * e] = f.x;
      x[2 * e + 1] = f.y;
    }
  };
  // pass 1: the largest |q| of every row (the 16 lanes of a half-warp hold one row)
  for (int base = 0; base < items; base += SOFT_THREADS) {
    const int item = base + tid;
    float x[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) x[e] = 0.f;
    if (item < items) load(item, x);
    float amax = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) amax = fmaxf(amax, fabsf(x[e]));
#pragma unroll
    for (int o = 1; o < 16; o <<= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    if (item < items && (item & 15) == 0) rowmax[item >> 4] = amax;
  }
  named_bar_sync(BAR, SOFT_THREADS);
  float amax = 0.f;
  for (int r = 0; r < p.R; ++r) amax = fmaxf(amax, rowmax[r]);
  // power-of-two scale: amax * s in [128, 256); exponent clamped so s stays a finite normal float
  int e2 = amax > 0.f ? static_cast<int>((__float_as_uint(amax) >> 23) & 0xFFu) - 127 : 0;
  e2 = max(-100, min(100, e2));
  const float sc = __uint_as_float(static_cast<uint32_t>(127 + 7 - e2) << 23);
  // pass 2: the two e4m3 terms (q read again: it is in L1/L2)
  for (int item = tid; item < items; item += SOFT_THREADS) {
    float x[8];
    load(item, x);
    uint8_t hb[8], lb[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float xs = x[e] * sc;
      hb[e] = e4m3_of(xs);
      lb[e] = e4m3_of(xs - f32_of_e4m3(hb[e]));
    }
    const int off = sw128_offset(item >> 4, (item & 15) * 8);
    *reinterpret_cast<uint2*>(qhi + off) = *reinterpret_cast<const uint2*>(hb);
    *reinterpret_cast<uint2*>(qlo + off) = *reinterpret_cast<const uint2*>(lb);
    if (dup) {   // the same rows again, dup bytes further on
      *reinterpret_cast<uint2*>(qhi + dup + off) = *reinterpret_cast<const uint2*>(hb);
      *reinterpret_cast<uint2*>(qlo + dup + off) = *reinterpret_cast<const uint2*>(lb);
    }
  }
  fence_proxy_async_smem();
  return p.score_scale / sc;
}
template <int SOFT_THREADS, int ROWS>
__device__ float attn_prepare_q(const AttnParams& p, int b, int g, uint8_t* qhi, uint8_t* qlo, float* rowmax) {
  return attn_prepare_q_t<SOFT_THREADS, ROWS, 1>(p, static_cast<int>(threadIdx.x), b, g, qhi, qlo, rowmax);
}

template <int NQ, int ROWS, int SPLIT, int STAGES, int NPROD>
__global__ void __launch_bounds__(AttnLayout<NQ, ROWS, SPLIT, STAGES, NPROD>::kLaunchBound, 1)
    attn_fwd_kernel(const AttnParams p) {
  using L = AttnLayout<NQ, ROWS, SPLIT, STAGES, NPROD>;
  constexpr int RPT = L::kRpt;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* kv_full = reinterpret_cast<uint64_t*>(smem + L::kBarOffset);
  uint64_t* kv_empty = kv_full + STAGES;
  uint64_t* s_full = kv_empty + STAGES;
  uint64_t* s_free = s_full + 2;
  uint64_t* p_full = s_free + 2;
  uint64_t* pv_done = p_full + 2;
  uint64_t* q_full = pv_done + 2;
  uint64_t* o_free = q_full + 2;
  uint64_t* drain = o_free + 1;
  int* misc = reinterpret_cast<int*>(smem + L::kMiscOffset);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(misc);
  volatile int* abort_flag = misc + 1;
  int* scratch = misc + 8;   // 40 ints
  float* xch = reinterpret_cast<float*>(smem + L::kXchOffset);
  float* lsum = reinterpret_cast<float*>(smem + L::kLsumOffset);
  float* rowmax = reinterpret_cast<float*>(smem + L::kRowmaxOffset);   // [2][ROWS]
  int* rowt = reinterpret_cast<int*>(smem + L::kRowtOffset);
  int* bt_ring = reinterpret_cast<int*>(smem + L::kBtOffset);
  uint8_t* qtile = smem + L::kQOffset;   // [buffer][hi, lo][NQ][128]
  uint8_t* ptile = smem + L::kPOffset;   // [buffer][hi, lo][128 keys x NQ rows]

  const int warp = warp_id_uniform();
  const uint32_t lane = lane_id();
  const int tid = threadIdx.x;
  constexpr int kProducerWarp = L::kSoftThreads / 32;   // producer warps kProducerWarp .. + NPROD - 1
  constexpr int kMmaWarp = kProducerWarp + NPROD;

  int b0 = 0, g0 = 0, t0 = 0;
  const int count = attn_locate(p, scratch, &b0, &g0, &t0);
  if (count == 0) return;   // uniform over the CTA: no tiles

  // Q and P tiles start zero (rows R..NQ-1 stay zero); row -> token table; barriers; tensor memory
  for (int i = tid; i < 8 * L::kQBytes / 16; i += L::kThreads)
    reinterpret_cast<uint4*>(qtile)[i] = make_uint4(0u, 0u, 0u, 0u);
  if constexpr (L::kMmaL)
    for (int i = tid; i < L::kKvBytes / 16; i += L::kThreads)   // e4m3 1.0 = 0x38
      reinterpret_cast<uint4*>(smem + L::kOnesOffset)[i] = make_uint4(0x38383838u, 0x38383838u, 0x38383838u, 0x38383838u);
  if (tid < ROWS) rowt[tid] = tid / p.group;
  if (tid == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&kv_full[s], NPROD);
      mbar_init(&kv_empty[s], 1);
    }
    for (int u = 0; u < 2; ++u) {
      mbar_init(&s_full[u], 1);
      mbar_init(&s_free[u], L::kSoftThreads);
      mbar_init(&p_full[u], L::kSoftThreads);
      mbar_init(&pv_done[u], 1);
      mbar_init(&q_full[u], L::kSoftThreads);
    }
    mbar_init(o_free, L::kSoftThreads);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == kMmaWarp) {
    tmem_alloc(tmem_slot, L::kTmemCols);
    tmem_relinquish();
  }
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp >= kProducerWarp && warp < kMmaWarp) {
    // ------------------------------------------------------------------ producers: K/V row copies
    // Producer warp wp, lane l copies 16-byte chunk (l & 7) of keys 4j + (l >> 3), j = wp, wp + NPROD, .. < 32, of
    // K and V (cp.async, L1 bypassed) into the stage with the 128-byte swizzle.  Each producer warp keeps its own
    // ring of block-table entries.  Tile i's copies and the entries of tile i + kPf form one cp.async group; at
    // the start of iteration i the groups up to i - kPf have landed, so the warp signals its part of tile i - kPf
    // (after a proxy fence: the tensor cores read it) and tile i's entries are in its ring.
    constexpr int kPf = L::kPf;
    const int wp = warp - kProducerWarp;
    bt_ring += wp * kPf * kAttnTile;
    const int chunk = static_cast<int>(lane & 7), ksub = static_cast<int>(lane >> 3);
    AttnCursor cur, pf;
    cur.init(p, b0, g0, t0, count);
    pf.init(p, b0, g0, t0, count);
    auto prefetch = [&](int buf) {
      const int k0 = pf.lo + pf.tile * kAttnTile;
      const int* src = p.block_table + static_cast<long long>(pf.b) * p.max_len;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int idx = 4 * static_cast<int>(lane) + j;
        if (k0 + idx < pf.L) cp_async_4(bt_ring + buf * kAttnTile + idx, src + k0 + idx);
      }
    };
#pragma unroll 1
    for (int d = 0; d < kPf; ++d) {
      if (pf.remaining > 0) {
        prefetch(d);
        pf.next(p);
      }
    }
    cp_async_commit();
    cp_async_wait<0>();
    __syncwarp();
    // the new tokens' rows are written by the append kernel launched just before: wait for it (once) before the
    // first tile that holds one of the last T positions, so that it runs under the earlier tiles' copies
    bool appended = false;
    int issued = 0;
    for (int i = 0; cur.remaining > 0; ++i, cur.next(p)) {
      const int s = i % STAGES;
      if (i >= kPf) {
        cp_async_wait<kPf - 1>();
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&kv_full[(i - kPf) % STAGES]);
      }
      const bool ok = attn_wait(&kv_empty[s], ((i / STAGES) & 1) ^ 1u, abort_flag, kSiteAttnProdEmpty);
      if (!__all_sync(0xffffffffu, ok)) break;
      if (!appended && cur.lo + cur.tile * kAttnTile + kAttnTile > cur.L - p.T) {
        pdl_wait();
        appended = true;
      }
      const int* rt = bt_ring + (i % kPf) * kAttnTile;
      const int nvalid = cur.L - (cur.lo + cur.tile * kAttnTile);   // keys of this tile inside the sequence
      const uint8_t* kbase = p.k_cache + static_cast<long long>(cur.g) * kAttnD + chunk * 16;
      const uint8_t* vbase = p.v_cache + static_cast<long long>(cur.g) * kAttnD + chunk * 16;
      uint8_t* st = smem + s * L::kStageBytes;
#pragma unroll 8
      for (int j = wp; j < kAttnTile / 4; j += NPROD) {
        const int key = 4 * j + ksub;
        int slot = rt[key < nvalid ? key : nvalid - 1];   // keys past the sequence read its last key (masked)
        if (slot < 0 || slot >= p.slots) {
          report(KDB_ERR_DEVICE_BOUNDS, kSiteAttnSlot);
          slot = 0;
        }
        const long long off = static_cast<long long>(slot) * p.Hkv * kAttnD;
        const int dst = key * 128 + ((chunk ^ (key & 7)) << 4);
        cp_async_16(st + dst, kbase + off);
        cp_async_16(st + L::kKvBytes + dst, vbase + off);
      }
      __syncwarp();   // every lane has read tile i's entries before the ring slot is refilled
      if (pf.remaining > 0) {
        prefetch(i % kPf);
        pf.next(p);
      }
      cp_async_commit();
      issued = i + 1;
    }
    if (!appended) pdl_wait();   // this grid ends after the append grid in every case
    cp_async_wait<0>();
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0)
      for (int t = issued > kPf ? issued - kPf : 0; t < issued; ++t) mbar_arrive(&kv_full[t % STAGES]);
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t kIdQK = idesc_e4m3_f32(128, NQ, false, false);
      constexpr uint32_t kIdPV = idesc_e4m3_f32(128, NQ, true, false);
      const uint32_t o_tmem = tmem_base + 2 * NQ;
      const uint32_t l_tmem = tmem_base + 3 * NQ;
      (void)l_tmem;
      AttnCursor cur;
      cur.init(p, b0, g0, t0, count);
      bool ok = true, issued = false;
      int prev_i = -1, prev_seg = 0;
      bool prev_start = false;
      // O^T (+)= V^T P^T for tile j (after the softmax wrote P^T[j & 1]); frees the K/V stage and P buffer
      auto issue_pv = [&](int j, int seg, bool start) -> bool {
        const int uj = j & 1, sj = j % STAGES;
        if (!attn_wait(&p_full[uj], (j >> 1) & 1, abort_flag, kSiteAttnMmaP)) return false;
        if (start && seg > 0 && !attn_wait(o_free, (seg - 1) & 1, abort_flag, kSiteAttnMmaOFree)) return false;
        tc_fence_after();
        const uint32_t v_addr = smem_u32(smem + sj * L::kStageBytes + L::kKvBytes);
        const uint32_t ph_addr = smem_u32(ptile + (2 * uj) * L::kQBytes);
        const uint32_t pl_addr = ph_addr + L::kQBytes;
#pragma unroll
        for (int ks = 0; ks < kAttnTile / 32; ++ks)
          mma_e4m3(o_tmem, sdesc_sw128_mnmajor(v_addr + ks * 4096), sdesc_sw128_kmajor(ph_addr + ks * 32), kIdPV,
                   (start && ks == 0) ? 0u : 1u);
#pragma unroll
        for (int ks = 0; ks < kAttnTile / 32; ++ks)
          mma_e4m3(o_tmem, sdesc_sw128_mnmajor(v_addr + ks * 4096), sdesc_sw128_kmajor(pl_addr + ks * 32), kIdPV,
                   1u);
        if constexpr (L::kMmaL) {
          // row sums: ones[128 x keys] P^T, every TMEM lane gets the same sums
          const uint32_t ones_addr = smem_u32(smem + L::kOnesOffset);
#pragma unroll
          for (int ks = 0; ks < kAttnTile / 32; ++ks)
            mma_e4m3(l_tmem, sdesc_sw128_kmajor(ones_addr + ks * 32), sdesc_sw128_kmajor(ph_addr + ks * 32), kIdQK,
                     (start && ks == 0) ? 0u : 1u);
#pragma unroll
          for (int ks = 0; ks < kAttnTile / 32; ++ks)
            mma_e4m3(l_tmem, sdesc_sw128_kmajor(ones_addr + ks * 32), sdesc_sw128_kmajor(pl_addr + ks * 32), kIdQK,
                     1u);
        }
        mma_commit(&kv_empty[sj]);
        mma_commit(&pv_done[uj]);
        return true;
      };
      for (int i = 0; ok && cur.remaining > 0; ++i, cur.next(p)) {
        const int s = i % STAGES, u = i & 1;
        if (!attn_wait(&kv_full[s], (i / STAGES) & 1, abort_flag, kSiteAttnMmaFull)) break;
        if (cur.seg_start && !attn_wait(&q_full[cur.seg & 1], (cur.seg >> 1) & 1, abort_flag, kSiteAttnMmaQ)) break;
        if (!attn_wait(&s_free[u], ((i >> 1) & 1) ^ 1u, abort_flag, kSiteAttnMmaSFree)) break;
        tc_fence_after();
        const uint32_t k_addr = smem_u32(smem + s * L::kStageBytes);
        const uint32_t qh_addr = smem_u32(qtile + (2 * (cur.seg & 1)) * L::kQBytes);
        const uint32_t ql_addr = qh_addr + L::kQBytes;
        const uint32_t s_tmem = tmem_base + u * NQ;
#pragma unroll
        for (int ks = 0; ks < kAttnD / 32; ++ks)
          mma_e4m3(s_tmem, sdesc_sw128_kmajor(k_addr + ks * 32), sdesc_sw128_kmajor(qh_addr + ks * 32), kIdQK,
                   ks > 0 ? 1u : 0u);
#pragma unroll
        for (int ks = 0; ks < kAttnD / 32; ++ks)
          mma_e4m3(s_tmem, sdesc_sw128_kmajor(k_addr + ks * 32), sdesc_sw128_kmajor(ql_addr + ks * 32), kIdQK, 1u);
        mma_commit(&s_full[u]);
        issued = true;
        if (prev_i >= 0 && !issue_pv(prev_i, prev_seg, prev_start)) {
          ok = false;
          break;
        }
        prev_i = i;
        prev_seg = cur.seg;
        prev_start = cur.seg_start;
      }
      if (ok && prev_i >= 0 && !*abort_flag) issue_pv(prev_i, prev_seg, prev_start);
      if (issued) {
        mma_commit(drain);
        mbar_wait_drain(drain, 0, kSiteAttnDrainMma);
      }
    }
  } else {
    // ------------------------------------------------------------------ softmax / epilogue warps
    // warp (quad, rs): TMEM lanes [32 quad, +32) = keys of the tile (S^T) and dims (O^T); rows [rs RPT, +RPT).
    const int quad = warp & 3, rs = warp >> 2;
    const int key = quad * 32 + static_cast<int>(lane);
    const int r0 = rs * RPT;
    const uint32_t lane_addr = tmem_base + (static_cast<uint32_t>(quad * 32) << 16);
    constexpr float kTau = 4.f;     // raise the running maximum only past +2^4
    constexpr float kPShift = 4.f;  // probabilities scaled by 2^(8 - tau): at most 2^8 in e4m3

    AttnCursor qcur;
    qcur.init(p, b0, g0, t0, count);
    float qsc0 = attn_prepare_q<L::kSoftThreads, ROWS>(p, qcur.b, qcur.g, qtile, qtile + L::kQBytes, rowmax);
    float qsc1 = 0.f;   // score scales of the segments in Q buffers 0 and 1
    mbar_arrive(&q_full[0]);
    bool q_more = qcur.next_segment(p);
    if (q_more) {
      qsc1 = attn_prepare_q<L::kSoftThreads, ROWS>(p, qcur.b, qcur.g, qtile + 2 * L::kQBytes,
                                                   qtile + 3 * L::kQBytes, rowmax + ROWS);
      mbar_arrive(&q_full[1]);
    }

    AttnCursor cur;
    cur.init(p, b0, g0, t0, count);
    float m_used[RPT], l_lane[RPT];
#pragma unroll
    for (int j = 0; j < RPT; ++j) {
      m_used[j] = -INFINITY;
      l_lane[j] = 0.f;
    }
    bool ok = true;
    for (int i = 0; cur.remaining > 0; ++i, cur.next(p)) {
      const int u = i & 1;
      const int bg = cur.b * p.Hkv + cur.g;
      if (cur.seg_start) {
        // segment j >= 1 begins: the Q buffer of segment j - 1 is free (its score MMAs completed), so prepare
        // segment j + 1's queries there
        if (cur.seg >= 1 && q_more) {
          q_more = qcur.next_segment(p);
          if (q_more) {
            const int qb = (cur.seg + 1) & 1;
            const float sc = attn_prepare_q<L::kSoftThreads, ROWS>(
                p, qcur.b, qcur.g, qtile + 2 * qb * L::kQBytes, qtile + (2 * qb + 1) * L::kQBytes, rowmax + qb * ROWS);
            if (qb == 0) {
              qsc0 = sc;
            } else {
              qsc1 = sc;
            }
            mbar_arrive(&q_full[qb]);
          }
        }
#pragma unroll
        for (int j = 0; j < RPT; ++j) {
          m_used[j] = -INFINITY;
          l_lane[j] = 0.f;
        }
        if (tid == 0 && cur.tile == 0) p.meta[bg * 2] = blockIdx.x;
      }
      // ---- scores of this thread's key for its rows (log2 units), masked, read from S^T in chunks of CH rows.
      // Up to 8 rows per thread they are read once and kept (S^T[u] is released at once); with more rows they are
      // read again after the vote rather than kept in registers across it.
      constexpr bool kHold = RPT <= 8;
      constexpr int CH = RPT < 8 ? RPT : 8;
      const bool got = __all_sync(0xffffffffu, attn_wait(&s_full[u], (i >> 1) & 1, abort_flag, kSiteAttnSoftS));
      ok = ok && got;
      const float qcs = (cur.seg & 1) ? qsc1 : qsc0;
      const int k0 = cur.lo + cur.tile * kAttnTile;
      const int pos = k0 + key;
      const int new0 = cur.L - p.T;
      // every row sees every key of an interior tile: before the first query and inside every window
      const bool interior = k0 + kAttnTile - 1 <= new0 && (p.window == 0 || k0 > cur.L - 1 - p.window);
      auto load_x = [&](int c, float (&xv)[CH]) {
        uint32_t acc[CH];
        if (got) {
          tmem_ld_cols<CH>(lane_addr + u * NQ + r0 + c * CH, acc);
          tmem_ld_wait();
        }
#pragma unroll
        for (int e = 0; e < CH; ++e) {
          const int r = r0 + c * CH + e;
          float v = got ? __uint_as_float(acc[e]) * qcs : -INFINITY;
          if (r >= p.R) {
            v = -INFINITY;
          } else if (!interior) {
            const int qpos = new0 + rowt[r];
            if (pos > qpos || (p.window > 0 && pos <= qpos - p.window)) v = -INFINITY;
          }
          xv[e] = v;
        }
      };
      if (got) tc_fence_after();
      float xr[CH];
      if constexpr (kHold) {
        load_x(0, xr);
        tc_fence_before();
        mbar_arrive(&s_free[u]);
      }
      auto get_x = [&](int c, float (&xv)[CH]) {
        if constexpr (kHold) {
#pragma unroll
          for (int e = 0; e < CH; ++e) xv[e] = xr[e];
        } else {
          load_x(c, xv);
        }
      };
      // ---- the running maxima change only when some score exceeds its row's maximum by more than 2^tau (and on
      // a segment's first tile, where they are -inf): one CTA-wide vote; only then the tile's row maxima are
      // exchanged across the 128 keys (warp redux, then the four quads through shared memory) and O^T rescaled.
      bool over = false;
#pragma unroll
      for (int c = 0; c < RPT / CH; ++c) {
        float xv[CH];
        get_x(c, xv);
#pragma unroll
        for (int e = 0; e < CH; ++e) over = over || xv[e] > m_used[c * CH + e] + kTau;
      }
      if (soft_bar_or(L::kSoftThreads, over || !ok)) {
        float* xc = xch + (i & 1) * ROWS * 4;
#pragma unroll
        for (int c = 0; c < RPT / CH; ++c) {
          float xv[CH];
          get_x(c, xv);
#pragma unroll
          for (int e = 0; e < CH; ++e) {
            const float wm = warp_max_f32(xv[e]);
            if (static_cast<int>(lane) == c * CH + e) xc[(r0 + c * CH + e) * 4 + quad] = wm;
          }
        }
        if (!soft_bar_and(L::kSoftThreads, ok)) break;
        float f[RPT];
        bool rescale = false;   // the same in every lane of the warp (same rows, same maxima)
#pragma unroll
        for (int j = 0; j < RPT; ++j) {
          const float4 t4 = *reinterpret_cast<const float4*>(xc + (r0 + j) * 4);
          const float tmax = fmaxf(fmaxf(t4.x, t4.y), fmaxf(t4.z, t4.w));
          f[j] = 1.f;
          if (m_used[j] == -INFINITY) {
            m_used[j] = tmax;   // first keys of this row in the segment: its O^T column is still zero
          } else if (tmax > m_used[j] + kTau) {
            f[j] = fast_exp2(m_used[j] - tmax);
            m_used[j] = tmax;
            if constexpr (!L::kMmaL) l_lane[j] *= f[j];
            rescale = true;
          }
        }
        if (rescale) {
          // this warp's O^T columns (its rows, its 32 dims), PV of tile i - 1 included, times f
          const int j1 = i - 1;
          const bool pv = __all_sync(0xffffffffu, attn_wait(&pv_done[j1 & 1], (j1 >> 1) & 1, abort_flag,
                                                            kSiteAttnSoftPv));
          ok = ok && pv;
          if (pv) {
            tc_fence_after();
            uint32_t o[RPT];
            tmem_ld_cols<RPT>(lane_addr + 2 * NQ + r0, o);
            tmem_ld_wait();
#pragma unroll
            for (int j = 0; j < RPT; ++j) o[j] = __float_as_uint(__uint_as_float(o[j]) * f[j]);
            tmem_st_cols<RPT>(lane_addr + 2 * NQ + r0, o);
            if constexpr (L::kMmaL) {
              tmem_ld_cols<RPT>(lane_addr + 3 * NQ + r0, o);
              tmem_ld_wait();
#pragma unroll
              for (int j = 0; j < RPT; ++j) o[j] = __float_as_uint(__uint_as_float(o[j]) * f[j]);
              tmem_st_cols<RPT>(lane_addr + 3 * NQ + r0, o);
            }
            tmem_st_wait();
          }
        }
      }
      // ---- probabilities (x 2^(8 - tau)) as two e4m3 terms into P^T[u] ([rows][128 keys], 128-byte swizzle);
      // pairs of rows: f16x2 of p, its nearest e4m3 pair (hi), then the e4m3 pair of the exact f16 residual (lo).
      // The four lanes of a quad (keys 4m..4m+3) transpose their bytes so each stores whole 4-key words of one
      // row.  Rows >= R get zero.
      if (i >= 2) ok = attn_wait(&pv_done[u], ((i - 2) >> 1) & 1, abort_flag, kSiteAttnSoftPv) && ok;
      {
        uint8_t* ph = ptile + (2 * u) * L::kQBytes;
        uint8_t* pl = ph + L::kQBytes;
        const int e4 = static_cast<int>(lane & 3);
        const int kb = key & ~3;
#pragma unroll
        for (int c = 0; c < RPT / CH; ++c) {
          float xv[CH];
          get_x(c, xv);
          uint32_t hw[(CH + 3) / 4], lw[(CH + 3) / 4];
#pragma unroll
          for (int w = 0; w < (CH + 3) / 4; ++w) hw[w] = lw[w] = 0u;
#pragma unroll
          for (int e = 0; e < CH; e += 2) {
            const int j = c * CH + e;
            __half2 h2;
            if constexpr (L::kMmaL) {
              // exponent in f32, 2^x of the pair in one f16x2 instruction; the sums come from the tensor cores
              float a[2];
#pragma unroll
              for (int t = 0; t < 2; ++t)
                a[t] = xv[e + t] != -INFINITY ? xv[e + t] - m_used[j + t] + kPShift : -INFINITY;
              const __half2 ha = __floats2half2_rn(a[0], a[1]);
              uint32_t hv;
              asm("ex2.approx.f16x2 %0, %1;" : "=r"(hv) : "r"(*reinterpret_cast<const uint32_t*>(&ha)));
              h2 = *reinterpret_cast<const __half2*>(&hv);
            } else {
              float pv[2];
#pragma unroll
              for (int t = 0; t < 2; ++t) {
                pv[t] = xv[e + t] != -INFINITY ? fast_exp2(xv[e + t] - m_used[j + t] + kPShift) : 0.f;
                l_lane[j + t] += pv[t];
              }
              h2 = __floats2half2_rn(pv[0], pv[1]);
            }
            const __nv_fp8x2_storage_t hi = __nv_cvt_halfraw2_to_fp8x2(__half2_raw(h2), __NV_SATFINITE, __NV_E4M3);
            // hi back in f16 without a conversion: a non-negative e4m3 byte shifted into f16 bits 7..14 is its value
            // times 2^-8 (normal and subnormal alike), so the residual is h2 - 256 hi, exact in f16
            const uint32_t hb_bits = __byte_perm(static_cast<uint32_t>(hi), 0u, 0x4140) << 7;
            const __half2 res = __hfma2(*reinterpret_cast<const __half2*>(&hb_bits), __float2half2_rn(-256.f), h2);
            const __nv_fp8x2_storage_t lo = __nv_cvt_halfraw2_to_fp8x2(__half2_raw(res), __NV_SATFINITE, __NV_E4M3);
            hw[e >> 2] |= static_cast<uint32_t>(hi) << (8 * (e & 3));
            lw[e >> 2] |= static_cast<uint32_t>(lo) << (8 * (e & 3));
          }
#pragma unroll
          for (int w = 0; w < (CH + 3) / 4; ++w) {
            const uint32_t th = quad_transpose(hw[w], e4), tl = quad_transpose(lw[w], e4);
            if (CH >= 4 || e4 < CH) {   // CH = 2: bytes 2, 3 of the word are the next warp group's rows
              const int off = sw128_offset(r0 + c * CH + 4 * w + e4, kb);
              *reinterpret_cast<uint32_t*>(ph + off) = th;
              *reinterpret_cast<uint32_t*>(pl + off) = tl;
            }
          }
        }
      }
      tc_fence_before();
      if constexpr (!kHold) mbar_arrive(&s_free[u]);   // S^T[u] read for the last time
      fence_proxy_async_smem();
      mbar_arrive(&p_full[u]);

      if (cur.seg_end) {
        // ---- this segment's partial: O^T columns (thread = dim), row sums, maxima
        const bool pv = __all_sync(0xffffffffu, attn_wait(&pv_done[u], (i >> 1) & 1, abort_flag, kSiteAttnSoftPv));
        ok = ok && pv;
        const long long slot = static_cast<long long>(blockIdx.x) + bg;
        float lrow = 0.f;   // kMmaL: this lane's row sum (row r0 + lane), read from the sum columns
        if (pv) {
          tc_fence_after();
          uint32_t o[RPT];
          tmem_ld_cols<RPT>(lane_addr + 2 * NQ + r0, o);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < RPT; ++j)
            if (r0 + j < p.R) p.part_o[(slot * p.R + r0 + j) * kAttnD + key] = __uint_as_float(o[j]);
          if constexpr (L::kMmaL) {
            tmem_ld_cols<RPT>(lane_addr + 3 * NQ + r0, o);
            tmem_ld_wait();
#pragma unroll
            for (int j = 0; j < RPT; ++j)
              if (static_cast<int>(lane) == j) lrow = __uint_as_float(o[j]);
          }
        }
        tc_fence_before();
        mbar_arrive(o_free);
        if constexpr (!L::kMmaL) {
#pragma unroll
          for (int j = 0; j < RPT; ++j) {
            const int r = r0 + j;
            const float ls = warp_sum_f32(l_lane[j]);
            if (r < p.R && lane == 0) lsum[r * 4 + quad] = ls;
          }
        }
        if (!soft_bar_and(L::kSoftThreads, ok)) break;
        if (quad == 0) {
#pragma unroll
          for (int j = 0; j < RPT; ++j) {
            const int r = r0 + j;
            if (r < p.R && static_cast<int>(lane) == j) {
              if constexpr (L::kMmaL) {
                p.part_l[slot * p.R + r] = lrow;   // every TMEM lane holds the row sums
              } else {
                const float4 l4 = *reinterpret_cast<const float4*>(lsum + r * 4);
                p.part_l[slot * p.R + r] = (l4.x + l4.y) + (l4.z + l4.w);
              }
              p.part_m[slot * p.R + r] = m_used[j];
            }
          }
        }
        if (tid == 0 && cur.tile == cur.ntiles - 1) p.meta[bg * 2 + 1] = blockIdx.x;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, L::kTmemCols);
  }
}

// ---------------------------------------------------------------------------------------------
// Many query rows (verify: T x group up to 64).  S = Q K^T with the query rows in the TMEM lanes: the A operand
// holds the 64 rows twice (M = 128), so row r's scores sit in lanes r and r + 64, where warps of all four lane
// quadrants can read them.  Four softmax threads share a row, 32 keys each; they meet once per tile through
// shared memory for the row maximum, after which each computes the same running maximum, so nothing is sent
// back.  P^T (K-major, one buffer) is written as 16-byte chunks.  O^T += V^T P^T as in the decode kernel (TMEM
// lanes = dims); four correction warps own those lanes: they rescale O^T when a row's running maximum rises and
// write the partial output at a segment's end.
// ---------------------------------------------------------------------------------------------
// Warps 0..7 softmax (warp w: lane quadrant w & 3, rows 32 (w & 1) + lane, keys 32 q .. 32 q + 31 of each tile
// with q = (w >> 1 & 1) + 2 (w >> 2)); 8..11 correction (O^T lanes 32 (w & 3) + lane); 12, 13 producers; 14 MMA.
template <int STAGES, int NPROD>
struct AttnRowsLayout {
  static_assert(NPROD == 2, "warp map");
  static constexpr int kRows = 64;                    // query rows handled (R <= 64)
  static constexpr int kSoftThreads = 256;            // four threads per row, 32 keys each
  static constexpr int kCorrThreads = 128;
  static constexpr int kCorrWarp0 = 8;
  static constexpr int kProducerWarp = 12;
  static constexpr int kMmaWarp = 14;
  static constexpr int kThreads = 32 * 15;
  // the bound given to the compiler: four of the 15 warps share a sub-partition of the SM, whose 16K registers
  // allow 128 per thread (65536 / 512)
  static constexpr int kLaunchBound = 512;
  static constexpr int kPf = STAGES - 2;
  static constexpr int kKvBytes = kAttnTile * kAttnD;
  static constexpr int kStageBytes = 2 * kKvBytes;
  static constexpr int kQBytes = kRows * kAttnD;      // one copy of one e4m3 term of Q: 64 rows x 128 B
  static constexpr int kPBytes = kRows * kAttnTile;   // one e4m3 term of P^T: 64 rows x 128 keys
  static constexpr int kQOffset = STAGES * kStageBytes;          // Q hi, hi again, lo, lo again
  static constexpr int kPOffset = kQOffset + 4 * kQBytes;        // P^T hi, lo
  static constexpr int kFOffset = kPOffset + 2 * kPBytes;        // rescale factors [2][64] + flags [2]
  static constexpr int kXOffset = kFOffset + 2 * kRows * 4 + 16;         // quarter-tile maxima [2][4][64]
  static constexpr int kLOffset = kXOffset + 2 * 4 * kRows * 4;          // quarter row sums [4][64]
  static constexpr int kRowmaxOffset = kLOffset + 4 * kRows * 4;         // |q| maxima [64]
  static constexpr int kBtOffset = kRowmaxOffset + kRows * 4;             // block-table rings [NPROD][kPf][128]
  static constexpr int kBarOffset = kBtOffset + NPROD * kPf * kAttnTile * 4;
  // kv_full[S], kv_empty[S], s_full[2], s_free[2], p_full[2], pv_done[2], q_full, f_ready[2], o_free, drain
  static constexpr int kNumBars = 2 * STAGES + 13;
  static constexpr int kMiscOffset = kBarOffset + kNumBars * 8;
  static constexpr int kSmemBytes = kMiscOffset + 48 * 4 + 1024;
  static constexpr uint32_t kTmemCols = 512;          // S[2] at [0, 256), O^T at [256, 320)
  static constexpr int kOCol = 256;
  static_assert(kSmemBytes <= 232448, "shared memory");
};

// 32 probabilities p = 2^(s qcs + shift) of one row (keys outside [klo, khi) give 0 when MASK) as two e4m3 terms,
// hi = e4m3(p) and lo = e4m3(p - hi), four keys per 32-bit word; returns the sum of the p.  The exponent is taken
// in f16 pairs (shift keeps p <= 2^8); the residual is formed in f16 from hi widened by a shift of its bits.  The
// sum adds f16 pairs within groups of 8 keys (three f16 roundings at most) and the groups in f32.
template <bool MASK>
__device__ __forceinline__ float attn_row_p32(const uint32_t (&acc)[32], float qcs, float shift, int klo, int khi,
                                              uint32_t (&hw)[8], uint32_t (&lw)[8]) {
  float sum = 0.f;
  __half2 grp = __float2half2_rn(0.f);
#pragma unroll
  for (int e = 0; e < 32; e += 2) {
    float a[2];
#pragma unroll
    for (int t = 0; t < 2; ++t) {
      const float x = fmaf(__uint_as_float(acc[e + t]), qcs, shift);
      a[t] = (!MASK || (e + t >= klo && e + t < khi)) ? x : -INFINITY;
    }
    const __half2 ha = __floats2half2_rn(a[0], a[1]);
    uint32_t hv;
    asm("ex2.approx.f16x2 %0, %1;" : "=r"(hv) : "r"(*reinterpret_cast<const uint32_t*>(&ha)));
    const __half2 h2 = *reinterpret_cast<const __half2*>(&hv);
    grp = __hadd2(grp, h2);
    if ((e & 6) == 6) {   // every 8 keys: the group's f16 pair sums (at most 4 x 2^8 each) into the f32 total
      const float2 g2 = __half22float2(grp);
      sum += g2.x + g2.y;
      grp = __float2half2_rn(0.f);
    }
    const __nv_fp8x2_storage_t hi = __nv_cvt_halfraw2_to_fp8x2(__half2_raw(h2), __NV_SATFINITE, __NV_E4M3);
    const uint32_t hb_bits = __byte_perm(static_cast<uint32_t>(hi), 0u, 0x4140) << 7;
    const __half2 res = __hfma2(*reinterpret_cast<const __half2*>(&hb_bits), __float2half2_rn(-256.f), h2);
    const __nv_fp8x2_storage_t lo = __nv_cvt_halfraw2_to_fp8x2(__half2_raw(res), __NV_SATFINITE, __NV_E4M3);
    if ((e & 2) == 0) {
      hw[e >> 2] = static_cast<uint32_t>(hi);
      lw[e >> 2] = static_cast<uint32_t>(lo);
    } else {
      hw[e >> 2] |= static_cast<uint32_t>(hi) << 16;
      lw[e >> 2] |= static_cast<uint32_t>(lo) << 16;
    }
  }
  return sum;
}

template <int STAGES, int NPROD>
__global__ void __launch_bounds__(AttnRowsLayout<STAGES, NPROD>::kLaunchBound, 1) attn_rows_kernel(const AttnParams p) {
  using L = AttnRowsLayout<STAGES, NPROD>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* kv_full = reinterpret_cast<uint64_t*>(smem + L::kBarOffset);
  uint64_t* kv_empty = kv_full + STAGES;
  uint64_t* s_full = kv_empty + STAGES;
  uint64_t* s_free = s_full + 2;
  uint64_t* p_full = s_free + 2;
  uint64_t* pv_done = p_full + 2;
  uint64_t* q_full = pv_done + 2;
  uint64_t* f_ready = q_full + 1;
  uint64_t* o_free = f_ready + 2;
  uint64_t* drain = o_free + 1;
  int* misc = reinterpret_cast<int*>(smem + L::kMiscOffset);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(misc);
  volatile int* abort_flag = misc + 1;
  int* scratch = misc + 8;
  float* fbuf = reinterpret_cast<float*>(smem + L::kFOffset);                       // [2][64]
  int* fflag = reinterpret_cast<int*>(smem + L::kFOffset + 2 * L::kRows * 4);       // [2]
  float* xq = reinterpret_cast<float*>(smem + L::kXOffset);                         // [2][4][64]
  float* lq = reinterpret_cast<float*>(smem + L::kLOffset);                         // [4][64]
  float* rowmax = reinterpret_cast<float*>(smem + L::kRowmaxOffset);
  int* bt_ring = reinterpret_cast<int*>(smem + L::kBtOffset);
  uint8_t* qtile = smem + L::kQOffset;
  uint8_t* ptile = smem + L::kPOffset;

  const int warp = warp_id_uniform();
  const uint32_t lane = lane_id();
  const int tid = threadIdx.x;
  constexpr int kProducerWarp = L::kProducerWarp;
  constexpr int kMmaWarp = L::kMmaWarp;

  int b0 = 0, g0 = 0, t0 = 0;
  const int count = attn_locate(p, scratch, &b0, &g0, &t0);
  if (count == 0) return;

  for (int i = tid; i < (4 * L::kQBytes + 2 * L::kPBytes) / 16; i += L::kThreads)
    reinterpret_cast<uint4*>(qtile)[i] = make_uint4(0u, 0u, 0u, 0u);   // Q rows R..63 stay zero
  if (tid == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&kv_full[s], NPROD);
      mbar_init(&kv_empty[s], 1);
    }
    for (int u = 0; u < 2; ++u) {
      mbar_init(&s_full[u], 1);
      mbar_init(&s_free[u], L::kSoftThreads);
      mbar_init(&p_full[u], L::kSoftThreads + L::kCorrThreads);
      mbar_init(&pv_done[u], 1);
      mbar_init(&f_ready[u], L::kRows);
    }
    mbar_init(q_full, L::kSoftThreads);
    mbar_init(o_free, L::kCorrThreads);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == kMmaWarp) {
    tmem_alloc(tmem_slot, L::kTmemCols);
    tmem_relinquish();
  }
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp >= kProducerWarp && warp < kProducerWarp + NPROD) {
    // ------------------------------------------------------------------ producers (as in attn_fwd_kernel)
    constexpr int kPf = L::kPf;
    const int wp = warp - kProducerWarp;
    bt_ring += wp * kPf * kAttnTile;
    const int chunk = static_cast<int>(lane & 7), ksub = static_cast<int>(lane >> 3);
    AttnCursor cur, pf;
    cur.init(p, b0, g0, t0, count);
    pf.init(p, b0, g0, t0, count);
    auto prefetch = [&](int buf) {
      const int k0 = pf.lo + pf.tile * kAttnTile;
      const int* src = p.block_table + static_cast<long long>(pf.b) * p.max_len;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int idx = 4 * static_cast<int>(lane) + j;
        if (k0 + idx < pf.L) cp_async_4(bt_ring + buf * kAttnTile + idx, src + k0 + idx);
      }
    };
#pragma unroll 1
    for (int d = 0; d < kPf; ++d) {
      if (pf.remaining > 0) {
        prefetch(d);
        pf.next(p);
      }
    }
    cp_async_commit();
    cp_async_wait<0>();
    __syncwarp();
    // the new tokens' rows are written by the append kernel launched just before: wait for it (once) before the
    // first tile that holds one of the last T positions, so that it runs under the earlier tiles' copies
    bool appended = false;
    int issued = 0;
    for (int i = 0; cur.remaining > 0; ++i, cur.next(p)) {
      const int s = i % STAGES;
      if (i >= kPf) {
        cp_async_wait<kPf - 1>();
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&kv_full[(i - kPf) % STAGES]);
      }
      const bool ok = attn_wait(&kv_empty[s], ((i / STAGES) & 1) ^ 1u, abort_flag, kSiteAttnProdEmpty);
      if (!__all_sync(0xffffffffu, ok)) break;
      if (!appended && cur.lo + cur.tile * kAttnTile + kAttnTile > cur.L - p.T) {
        pdl_wait();
        appended = true;
      }
      const int* rt = bt_ring + (i % kPf) * kAttnTile;
      const int nvalid = cur.L - (cur.lo + cur.tile * kAttnTile);
      const uint8_t* kbase = p.k_cache + static_cast<long long>(cur.g) * kAttnD + chunk * 16;
      const uint8_t* vbase = p.v_cache + static_cast<long long>(cur.g) * kAttnD + chunk * 16;
      uint8_t* st = smem + s * L::kStageBytes;
#pragma unroll 8
      for (int j = wp; j < kAttnTile / 4; j += NPROD) {
        const int key = 4 * j + ksub;
        int slot = rt[key < nvalid ? key : nvalid - 1];
        if (slot < 0 || slot >= p.slots) {
          report(KDB_ERR_DEVICE_BOUNDS, kSiteAttnSlot);
          slot = 0;
        }
        const long long off = static_cast<long long>(slot) * p.Hkv * kAttnD;
        const int dst = key * 128 + ((chunk ^ (key & 7)) << 4);
        cp_async_16(st + dst, kbase + off);
        cp_async_16(st + L::kKvBytes + dst, vbase + off);
      }
      __syncwarp();
      if (pf.remaining > 0) {
        prefetch(i % kPf);
        pf.next(p);
      }
      cp_async_commit();
      issued = i + 1;
    }
    if (!appended) pdl_wait();   // this grid ends after the append grid in every case
    cp_async_wait<0>();
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0)
      for (int t = issued > kPf ? issued - kPf : 0; t < issued; ++t) mbar_arrive(&kv_full[t % STAGES]);
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t kIdQK = idesc_e4m3_f32(128, 128, false, false);   // S[rows (twice) x keys]
      constexpr uint32_t kIdPV = idesc_e4m3_f32(128, 64, true, false);     // O^T[dims x rows]
      const uint32_t o_tmem = tmem_base + L::kOCol;
      const uint32_t qh_addr = smem_u32(qtile);
      const uint32_t ql_addr = qh_addr + 2 * L::kQBytes;
      const uint32_t ph_addr = smem_u32(ptile);
      const uint32_t pl_addr = ph_addr + L::kPBytes;
      AttnCursor cur;
      cur.init(p, b0, g0, t0, count);
      bool ok = true, issued = false;
      int prev_i = -1, prev_seg = 0;
      bool prev_start = false;
      auto issue_pv = [&](int j, int seg, bool start) -> bool {
        const int uj = j & 1, sj = j % STAGES;
        if (!attn_wait(&p_full[uj], (j >> 1) & 1, abort_flag, kSiteAttnMmaP)) return false;
        if (start && seg > 0 && !attn_wait(o_free, (seg - 1) & 1, abort_flag, kSiteAttnMmaOFree)) return false;
        tc_fence_after();
        const uint32_t v_addr = smem_u32(smem + sj * L::kStageBytes + L::kKvBytes);
#pragma unroll
        for (int ks = 0; ks < kAttnTile / 32; ++ks)
          mma_e4m3(o_tmem, sdesc_sw128_mnmajor(v_addr + ks * 4096), sdesc_sw128_kmajor(ph_addr + ks * 32), kIdPV,
                   (start && ks == 0) ? 0u : 1u);
#pragma unroll
        for (int ks = 0; ks < kAttnTile / 32; ++ks)
          mma_e4m3(o_tmem, sdesc_sw128_mnmajor(v_addr + ks * 4096), sdesc_sw128_kmajor(pl_addr + ks * 32), kIdPV,
                   1u);
        mma_commit(&kv_empty[sj]);
        mma_commit(&pv_done[uj]);
        return true;
      };
      for (int i = 0; ok && cur.remaining > 0; ++i, cur.next(p)) {
        const int s = i % STAGES, u = i & 1;
        if (!attn_wait(&kv_full[s], (i / STAGES) & 1, abort_flag, kSiteAttnMmaFull)) break;
        if (cur.seg_start && !attn_wait(q_full, cur.seg & 1, abort_flag, kSiteAttnMmaQ)) break;
        if (!attn_wait(&s_free[u], ((i >> 1) & 1) ^ 1u, abort_flag, kSiteAttnMmaSFree)) break;
        tc_fence_after();
        const uint32_t k_addr = smem_u32(smem + s * L::kStageBytes);
        const uint32_t s_tmem = tmem_base + u * 128;
#pragma unroll
        for (int ks = 0; ks < kAttnD / 32; ++ks)
          mma_e4m3(s_tmem, sdesc_sw128_kmajor(qh_addr + ks * 32), sdesc_sw128_kmajor(k_addr + ks * 32), kIdQK,
                   ks > 0 ? 1u : 0u);
#pragma unroll
        for (int ks = 0; ks < kAttnD / 32; ++ks)
          mma_e4m3(s_tmem, sdesc_sw128_kmajor(ql_addr + ks * 32), sdesc_sw128_kmajor(k_addr + ks * 32), kIdQK, 1u);
        mma_commit(&s_full[u]);
        issued = true;
        if (prev_i >= 0 && !issue_pv(prev_i, prev_seg, prev_start)) {
          ok = false;
          break;
        }
        prev_i = i;
        prev_seg = cur.seg;
        prev_start = cur.seg_start;
      }
      if (ok && prev_i >= 0 && !*abort_flag) issue_pv(prev_i, prev_seg, prev_start);
      if (issued) {
        mma_commit(drain);
        mbar_wait_drain(drain, 0, kSiteAttnDrainMma);
      }
    }
  } else if (warp < L::kCorrWarp0) {
    // ------------------------------------------------------------------ softmax: thread = (row, quarter tile)
    const int quad = warp & 3;
    const int r = (quad & 1) * 32 + static_cast<int>(lane);      // query row
    const int qt = (quad >> 1) + 2 * (warp >> 2);               // keys 32 qt .. 32 qt + 31 of each tile
    const uint32_t s_addr = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + 32 * qt;
    const int trow = r / p.group;   // token of the row
    const bool live = r < p.R;
    constexpr float kTau = 4.f;
    constexpr float kPShift = 4.f;
    float qcs = 0.f;                        // the segment's score scale
    float m_run = -INFINITY, l_run = 0.f;   // the row's running maximum (log2) and this quarter's sum
    bool ok = true;
    AttnCursor cur;
    cur.init(p, b0, g0, t0, count);
    for (int i = 0; cur.remaining > 0; ++i, cur.next(p)) {
      const int u = i & 1;
      const int bg = cur.b * p.Hkv + cur.g;
      if (cur.seg_start) {
        // the previous segment's last S was read by these threads, so its QK MMAs no longer read Q
        qcs = attn_prepare_q_t<L::kSoftThreads, L::kRows, 2>(p, tid, cur.b, cur.g, qtile, qtile + 2 * L::kQBytes,
                                                            rowmax, L::kQBytes);
        mbar_arrive(q_full);
        m_run = -INFINITY;
        l_run = 0.f;
        if (tid == 0 && cur.tile == 0) p.meta[bg * 2] = blockIdx.x;
      }
      const bool got = __all_sync(0xffffffffu, attn_wait(&s_full[u], (i >> 1) & 1, abort_flag, kSiteAttnSoftS));
      ok = ok && got;
      const int k0 = cur.lo + cur.tile * kAttnTile + 32 * qt;   // position of this thread's first key
      const int qpos = cur.L - p.T + trow;
      // keys [klo, khi) of this thread's 32 are the row's (causal and window limits)
      int khi = qpos - k0 + 1;
      khi = khi < 0 ? 0 : (khi > 32 ? 32 : khi);
      int klo = p.window > 0 ? qpos - p.window + 1 - k0 : 0;
      klo = klo < 0 ? 0 : (klo > 32 ? 32 : klo);
      if (!live || !got) khi = 0;
      const bool full = klo == 0 && khi == 32;
      uint32_t acc[32];
      if (got) {
        tc_fence_after();
        tmem_ld_32x32b_x32(s_addr + u * 128, acc);
        tmem_ld_wait();
      }
      tc_fence_before();
      mbar_arrive(&s_free[u]);
      float qmax = -INFINITY;
      if (full) {
#pragma unroll
        for (int e = 0; e < 32; ++e) qmax = fmaxf(qmax, __uint_as_float(acc[e]));
      } else {
#pragma unroll
        for (int e = 0; e < 32; ++e)
          if (e >= klo && e < khi) qmax = fmaxf(qmax, __uint_as_float(acc[e]));
      }
      qmax = qmax == -INFINITY ? qmax : qmax * qcs;
      xq[(u * 4 + qt) * L::kRows + r] = qmax;
      if (named_bar_or(2, L::kSoftThreads, !ok)) break;
      // the four quarters' maxima: every thread of the row takes the same decision
      const float* xr = xq + u * 4 * L::kRows + r;
      const float tmax = fmaxf(fmaxf(xr[0], xr[L::kRows]), fmaxf(xr[2 * L::kRows], xr[3 * L::kRows]));
      float f = 1.f;
      bool resc = false;
      if (m_run == -INFINITY) {
        m_run = tmax;
      } else if (tmax > m_run + kTau) {
        f = fast_exp2(m_run - tmax);
        m_run = tmax;
        resc = true;
      }
      l_run *= f;
      if (qt == 0) {   // warps 0 and 1
        fbuf[u * L::kRows + r] = f;
        const bool any = named_bar_or(3, 64, resc);
        if (r == 0) fflag[u] = any ? 1 : 0;
        mbar_arrive(&f_ready[u]);
      }
      // the tensor cores have read the previous tile's P^T before this one overwrites the buffer
      if (i >= 1) ok = attn_wait(&pv_done[(i - 1) & 1], ((i - 1) >> 1) & 1, abort_flag, kSiteAttnSoftPv) && ok;
      uint32_t hw[8], lw[8];
      const float shift = kPShift - m_run;
      if (full) {
        l_run += attn_row_p32<false>(acc, qcs, shift, 0, 32, hw, lw);
      } else {
        l_run += attn_row_p32<true>(acc, qcs, shift, klo, m_run == -INFINITY ? 0 : khi, hw, lw);
      }
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int off = sw128_offset(r, 32 * qt + 16 * h);
        *reinterpret_cast<uint4*>(ptile + off) = make_uint4(hw[4 * h], hw[4 * h + 1], hw[4 * h + 2], hw[4 * h + 3]);
        *reinterpret_cast<uint4*>(ptile + L::kPBytes + off) =
            make_uint4(lw[4 * h], lw[4 * h + 1], lw[4 * h + 2], lw[4 * h + 3]);
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&p_full[u]);
      if (cur.seg_end) {
        lq[qt * L::kRows + r] = l_run;
        named_bar_sync(2, L::kSoftThreads);
        if (qt == 0 && live) {
          const long long slot = static_cast<long long>(blockIdx.x) + bg;
          p.part_m[slot * p.R + r] = m_run;
          p.part_l[slot * p.R + r] = (lq[r] + lq[L::kRows + r]) + (lq[2 * L::kRows + r] + lq[3 * L::kRows + r]);
        }
        named_bar_sync(2, L::kSoftThreads);   // lq read before a later segment end rewrites it
        if (tid == 0 && cur.tile == cur.ntiles - 1) p.meta[bg * 2 + 1] = blockIdx.x;
      }
    }
  } else {
    // ------------------------------------------------------------------ correction warps (thread = dim)
    const int quad = warp & 3;
    const int dim = quad * 32 + static_cast<int>(lane);
    const uint32_t o_addr = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + L::kOCol;
    bool ok = true;
    AttnCursor cur;
    cur.init(p, b0, g0, t0, count);
    for (int i = 0; cur.remaining > 0; ++i, cur.next(p)) {
      const int u = i & 1;
      const int bg = cur.b * p.Hkv + cur.g;
      ok = __all_sync(0xffffffffu, attn_wait(&f_ready[u], (i >> 1) & 1, abort_flag, kSiteAttnSoftPv)) && ok;
      if (ok && fflag[u] && i >= 1) {
        // O^T holds the tiles before this one once PV(i - 1) completed; rescale its columns (rows)
        const int j1 = i - 1;
        const bool pv = __all_sync(0xffffffffu, attn_wait(&pv_done[j1 & 1], (j1 >> 1) & 1, abort_flag,
                                                          kSiteAttnSoftPv));
        ok = ok && pv;
        if (pv) {
          tc_fence_after();
#pragma unroll 1
          for (int c = 0; c < 2; ++c) {
            uint32_t o[32];
            tmem_ld_32x32b_x32(o_addr + 32 * c, o);
            tmem_ld_wait();
#pragma unroll
            for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * fbuf[u * L::kRows + 32 * c + e]);
            tmem_st_cols<32>(o_addr + 32 * c, o);
          }
          tmem_st_wait();
        }
      }
      tc_fence_before();
      mbar_arrive(&p_full[u]);
      if (cur.seg_end) {
        const bool pv = __all_sync(0xffffffffu, attn_wait(&pv_done[u], (i >> 1) & 1, abort_flag, kSiteAttnSoftPv));
        ok = ok && pv;
        if (pv) {
          const long long slot = static_cast<long long>(blockIdx.x) + bg;
          tc_fence_after();
#pragma unroll 1
          for (int c = 0; c < 2; ++c) {
            uint32_t o[32];
            tmem_ld_32x32b_x32(o_addr + 32 * c, o);
            tmem_ld_wait();
#pragma unroll
            for (int e = 0; e < 32; ++e)
              if (32 * c + e < p.R) p.part_o[(slot * p.R + 32 * c + e) * kAttnD + dim] = __uint_as_float(o[e]);
          }
        }
        tc_fence_before();
        mbar_arrive(o_free);
      }
      if (!__all_sync(0xffffffffu, ok)) break;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, L::kTmemCols);
  }
}

// ---------------------------------------------------------------------------------------------
// append: one warp per new (sequence, token, KV head) row, four values per lane
// ---------------------------------------------------------------------------------------------
struct AttnAppendParams {
  const __nv_bfloat16* k_new;
  const __nv_bfloat16* v_new;
  uint8_t* k_cache;
  uint8_t* v_cache;
  const int* block_table;
  const int* seq_lens;
  float kv_scale;
  int B, T, Hkv, max_len;
  long long slots;
};

__global__ void __launch_bounds__(128) attn_append_kernel(const AttnAppendParams a) {
  pdl_launch_dependents();   // the attention kernel's prologue may overlap this kernel
  const long long row = static_cast<long long>(blockIdx.x) * 4 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= static_cast<long long>(a.B) * a.T * a.Hkv) return;
  const int g = static_cast<int>(row % a.Hkv);
  const long long bt = row / a.Hkv;
  const int t = static_cast<int>(bt % a.T), b = static_cast<int>(bt / a.T);
  int L = __ldg(a.seq_lens + b);
  L = L < a.T ? a.T : (L > a.max_len ? a.max_len : L);   // an out-of-range length is reported by attn_fwd_kernel
  const int slot = __ldg(a.block_table + static_cast<long long>(b) * a.max_len + L - a.T + t);
  if (slot < 0 || slot >= a.slots) {
    if (lane == 0) report(KDB_ERR_DEVICE_BOUNDS, kSiteAttnAppend);
    return;
  }
  const long long src = row * kAttnD + lane * 4;
  const long long dst = (static_cast<long long>(slot) * a.Hkv + g) * kAttnD + lane * 4;
#pragma unroll
  for (int w = 0; w < 2; ++w) {
    const __nv_bfloat16* x = (w == 0 ? a.k_new : a.v_new) + src;
    const uint2 raw = __ldg(reinterpret_cast<const uint2*>(x));
    const __nv_bfloat16* xv = reinterpret_cast<const __nv_bfloat16*>(&raw);
    uint32_t packed = 0;
#pragma unroll
    for (int e = 0; e < 4; ++e)
      packed |= static_cast<uint32_t>(e4m3_of(__fdiv_rn(__bfloat162float(xv[e]), a.kv_scale))) << (8 * e);
    *reinterpret_cast<uint32_t*>((w == 0 ? a.k_cache : a.v_cache) + dst) = packed;
  }
}

// ---------------------------------------------------------------------------------------------
// merge: one CTA (W warps) per (sequence, KV head, query row).  Pass 1: the largest partial maximum M; pass 2:
// warp w sums the partials of CTAs c0 + w, + W, ... weighted by 2^(m - M) (independent loads, no running
// rescale), then the W warps' sums are added through shared memory.  W = 16 when a row has many partials (long
// sequences over many CTAs); W = 4 when it has few, so that every row's CTA is resident in one wave.
// ---------------------------------------------------------------------------------------------
template <int kMergeWarps>
__global__ void __launch_bounds__(kMergeWarps * 32)
    attn_merge_kernel(const AttnParams p, int ctas, float kv_scale, __nv_bfloat16* __restrict__ out) {
  __shared__ float red[kMergeWarps], sm_l[kMergeWarps];
  __shared__ __align__(16) float sm_o[kMergeWarps][kAttnD];
  const int r = blockIdx.x % p.R;
  const int bg = blockIdx.x / p.R;
  const int g = bg % p.Hkv, b = bg / p.Hkv;
  const int t = r / p.group, h = r - t * p.group;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  pdl_wait();   // the partials come from the attention kernel launched just before
  int c0 = p.meta[bg * 2], c1 = p.meta[bg * 2 + 1];
  if (c0 < 0 || c1 >= ctas || c0 > c1) {
    if (threadIdx.x == 0) report(KDB_ERR_DEVICE_BOUNDS, kSiteAttnMeta);
    c0 = 0;
    c1 = -1;
  }
  const int n = c1 - c0 + 1;
  const long long base = static_cast<long long>(c0) + bg;   // the partial slot of CTA c0 + k is base + k
  float mx = -INFINITY;
  for (int k = threadIdx.x; k < n; k += kMergeWarps * 32) mx = fmaxf(mx, p.part_m[(base + k) * p.R + r]);
  mx = warp_max_f32(mx);
  if (lane == 0) red[warp] = mx;
  __syncthreads();
  float M = -INFINITY;
#pragma unroll
  for (int w = 0; w < kMergeWarps; ++w) M = fmaxf(M, red[w]);
  float l = 0.f;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  if (M != -INFINITY) {
#pragma unroll 4
    for (int k = warp; k < n; k += kMergeWarps) {
      const long long row = (base + k) * p.R + r;
      const float mk = p.part_m[row];
      const float lk = p.part_l[row];
      const float4 ok = *reinterpret_cast<const float4*>(p.part_o + row * kAttnD + lane * 4);
      const float w = mk != -INFINITY ? fast_exp2(mk - M) : 0.f;
      l = fmaf(w, lk, l);
      acc.x = fmaf(w, ok.x, acc.x);
      acc.y = fmaf(w, ok.y, acc.y);
      acc.z = fmaf(w, ok.z, acc.z);
      acc.w = fmaf(w, ok.w, acc.w);
    }
  }
  if (lane == 0) sm_l[warp] = l;
  *reinterpret_cast<float4*>(&sm_o[warp][lane * 4]) = acc;
  __syncthreads();
  if (warp == 0) {
    float lt = 0.f;
    float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int w = 0; w < kMergeWarps; ++w) {
      lt += sm_l[w];
      const float4 ow = *reinterpret_cast<const float4*>(&sm_o[w][lane * 4]);
      o.x += ow.x;
      o.y += ow.y;
      o.z += ow.z;
      o.w += ow.w;
    }
    const float k = lt > 0.f ? kv_scale / lt : 0.f;
    __nv_bfloat16* dst = out + ((static_cast<long long>(b) * p.T + t) * p.Hq + g * p.group + h) * kAttnD + lane * 4;
    const __nv_bfloat162 lo2 = __floats2bfloat162_rn(o.x * k, o.y * k);
    const __nv_bfloat162 hi2 = __floats2bfloat162_rn(o.z * k, o.w * k);
    uint2 pk;
    pk.x = *reinterpret_cast<const uint32_t*>(&lo2);
    pk.y = *reinterpret_cast<const uint32_t*>(&hi2);
    *reinterpret_cast<uint2*>(dst) = pk;
  }
}

// ---------------------------------------------------------------------------------------------
// host
// ---------------------------------------------------------------------------------------------
static long long attn_max_tiles(long long B, long long T, long long Hkv, long long max_len, long long window) {
  const long long span = window > 0 ? (window + T - 1 < max_len ? window + T - 1 : max_len) : max_len;
  return B * Hkv * ((span + kAttnTile - 1) / kAttnTile);
}

int attn_check(long long B, long long T, long long Hq, long long Hkv, long long D, long long max_len, long long slots,
               long long window) {
  if (B < 0 || T <= 0 || Hq <= 0 || Hkv <= 0 || max_len < 0 || slots < 0 || window < 0) return KDB_ERR_INVALID_ARG;
  if (D != kAttnD || Hq % Hkv != 0 || T * (Hq / Hkv) > kAttnMaxRows) return KDB_ERR_UNSUPPORTED;
  if (B > 0 && (max_len < T || slots <= 0)) return KDB_ERR_INVALID_ARG;
  if (B > (1ll << 24) || window > (1ll << 30) || max_len >= (1ll << 31) ||
      attn_max_tiles(B, T, Hkv, max_len, window) >= (1ll << 30) || slots * Hkv >= (1ll << 31))
    return KDB_ERR_UNSUPPORTED;
  return KDB_OK;
}

static int attn_ctas_bound(long long B, long long T, long long Hkv, long long max_len, long long window) {
  const long long n = attn_max_tiles(B, T, Hkv, max_len, window);
  return static_cast<int>(n < kAttnMaxCtas ? n : kAttnMaxCtas);
}

size_t attn_workspace_bytes(long long B, long long T, long long Hq, long long Hkv, long long max_len,
                            long long window) {
  if (attn_check(B, T, Hq, Hkv, kAttnD, max_len, 1, window) != KDB_OK || B == 0) return 0;
  const long long R = T * (Hq / Hkv);
  const long long nslots = attn_ctas_bound(B, T, Hkv, max_len, window) + B * Hkv;
  const size_t fbytes = (static_cast<size_t>(nslots) * R * (2 + kAttnD) * sizeof(float) + 255) / 256 * 256;
  return fbytes + static_cast<size_t>(B * Hkv * 2) * sizeof(int);
}

template <int NQ, int ROWS, int SPLIT, int STAGES, int NPROD>
static int attn_launch_fwd(const AttnParams& p, long long max_tiles, int* ctas_out, cudaStream_t s) {
  using L = AttnLayout<NQ, ROWS, SPLIT, STAGES, NPROD>;
  auto kern = attn_fwd_kernel<NQ, ROWS, SPLIT, STAGES, NPROD>;
  static int occ[64] = {0};
  int dev = 0;
  int rc = cuda_status(cudaGetDevice(&dev));
  if (rc) return rc;
  if (dev < 0 || dev >= 64) return KDB_ERR_UNSUPPORTED;
  if (occ[dev] == 0) {
    rc = cuda_status(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kSmemBytes));
    if (rc) return rc;
    int o = 0;
    rc = cuda_status(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&o, kern, L::kThreads, L::kSmemBytes));
    if (rc) return rc;
    occ[dev] = o > 0 ? o : 1;
  }
  // small jobs: one tile per CTA; larger ones: at least four tiles per CTA, at most one wave of resident CTAs
  const long long resident = static_cast<long long>(num_sms()) * occ[dev];
  long long c = max_tiles <= 32 ? max_tiles : (max_tiles + 3) / 4;
  if (max_tiles > 32 && c < 32) c = 32;
  if (c > resident) c = resident;
  if (c > kAttnMaxCtas) c = kAttnMaxCtas;
  if (c < 1) c = 1;
  *ctas_out = static_cast<int>(c);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned int>(c), 1, 1);
  cfg.blockDim = dim3(L::kThreads, 1, 1);
  cfg.dynamicSmemBytes = L::kSmemBytes;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;   // overlap the append kernel's tail
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cuda_status(cudaLaunchKernelEx(&cfg, kern, p));
}

template <int STAGES, int NPROD>
static int attn_launch_rows(const AttnParams& p, long long max_tiles, int* ctas_out, cudaStream_t s) {
  using L = AttnRowsLayout<STAGES, NPROD>;
  auto kern = attn_rows_kernel<STAGES, NPROD>;
  static bool done[64] = {false};
  int dev = 0;
  int rc = cuda_status(cudaGetDevice(&dev));
  if (rc) return rc;
  if (dev < 0 || dev >= 64) return KDB_ERR_UNSUPPORTED;
  if (!done[dev]) {
    rc = cuda_status(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kSmemBytes));
    if (rc) return rc;
    done[dev] = true;
  }
  // one CTA per SM (512 TMEM columns); at least four tiles per CTA once the work covers the GPU
  long long c = max_tiles <= 32 ? max_tiles : (max_tiles + 3) / 4;
  if (max_tiles > 32 && c < 32) c = 32;
  if (c > num_sms()) c = num_sms();
  if (c > kAttnMaxCtas) c = kAttnMaxCtas;
  if (c < 1) c = 1;
  *ctas_out = static_cast<int>(c);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned int>(c), 1, 1);
  cfg.blockDim = dim3(L::kThreads, 1, 1);
  cfg.dynamicSmemBytes = L::kSmemBytes;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cuda_status(cudaLaunchKernelEx(&cfg, kern, p));
}

int attn_decode_fp8(const void* q, const void* k_new, const void* v_new, void* k_cache, void* v_cache,
                    const int* block_table, const int* seq_lens, float kv_scale, void* out, long long B, long long T,
                    long long Hq, long long Hkv, long long D, long long max_len, long long slots, long long window,
                    void* workspace, size_t workspace_bytes, cudaStream_t s) {
  int rc = attn_check(B, T, Hq, Hkv, D, max_len, slots, window);
  if (rc) return rc;
  if (B == 0) return KDB_OK;
  if (!q || !k_new || !v_new || !k_cache || !v_cache || !block_table || !seq_lens || !out) return KDB_ERR_INVALID_ARG;
  if (!aligned16(q) || !aligned16(k_cache) || !aligned16(v_cache) || !aligned16(k_new) || !aligned16(v_new) ||
      !aligned16(out) || (reinterpret_cast<uintptr_t>(block_table) & 3u) || (reinterpret_cast<uintptr_t>(seq_lens) & 3u))
    return KDB_ERR_INVALID_ARG;
  if (!(kv_scale > 0.f) || !(kv_scale < INFINITY)) return KDB_ERR_INVALID_ARG;
  const size_t need = attn_workspace_bytes(B, T, Hq, Hkv, max_len, window);
  if (!workspace || workspace_bytes < need) return KDB_ERR_WORKSPACE;
  if ((reinterpret_cast<uintptr_t>(workspace) & 255u) != 0) return KDB_ERR_INVALID_ARG;

  const long long group = Hq / Hkv, R = T * group;
  const long long max_tiles = attn_max_tiles(B, T, Hkv, max_len, window);
  const long long nslots = attn_ctas_bound(B, T, Hkv, max_len, window) + B * Hkv;
  AttnParams p;
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.block_table = block_table;
  p.seq_lens = seq_lens;
  p.score_scale = kv_scale * (1.0f / sqrtf(static_cast<float>(kAttnD))) * 1.4426950408889634f;
  p.B = static_cast<int>(B);
  p.T = static_cast<int>(T);
  p.Hq = static_cast<int>(Hq);
  p.Hkv = static_cast<int>(Hkv);
  p.group = static_cast<int>(group);
  p.R = static_cast<int>(R);
  p.max_len = static_cast<int>(max_len);
  p.window = static_cast<int>(window);
  p.slots = slots;
  float* f = static_cast<float*>(workspace);
  p.part_m = f;
  p.part_l = f + nslots * R;
  p.part_o = f + 2 * nslots * R;
  const size_t fbytes = (static_cast<size_t>(nslots) * R * (2 + kAttnD) * sizeof(float) + 255) / 256 * 256;
  p.meta = reinterpret_cast<int*>(static_cast<uint8_t*>(workspace) + fbytes);

  p.k_cache = static_cast<const uint8_t*>(k_cache);
  p.v_cache = static_cast<const uint8_t*>(v_cache);

  AttnAppendParams a;
  a.k_new = static_cast<const __nv_bfloat16*>(k_new);
  a.v_new = static_cast<const __nv_bfloat16*>(v_new);
  a.k_cache = static_cast<uint8_t*>(k_cache);
  a.v_cache = static_cast<uint8_t*>(v_cache);
  a.block_table = block_table;
  a.seq_lens = seq_lens;
  a.kv_scale = kv_scale;
  a.B = p.B;
  a.T = p.T;
  a.Hkv = p.Hkv;
  a.max_len = p.max_len;
  a.slots = slots;
  const long long rows = B * T * Hkv;
  attn_append_kernel<<<static_cast<unsigned int>((rows + 3) / 4), 128, 0, s>>>(a);
  rc = cuda_status(cudaGetLastError());
  if (rc) return rc;

  int ctas = 0;
  rc = R <= 8    ? attn_launch_fwd<16, 8, 2, 6, 4>(p, max_tiles, &ctas, s)
       : R <= 16 ? attn_launch_fwd<16, 16, 2, 6, 4>(p, max_tiles, &ctas, s)
                 : attn_launch_rows<5, 2>(p, max_tiles, &ctas, s);
  if (rc) return rc;
  // partials per (sequence, KV head) on average: ctas / (B Hkv) + 1 (a CTA's range may start inside a segment)
  const bool few = ctas <= 7 * B * Hkv;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned int>(B * Hkv * R), 1, 1);
  cfg.blockDim = dim3(few ? 4 * 32 : 16 * 32, 1, 1);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  rc = cuda_status(cudaLaunchKernelEx(&cfg, few ? attn_merge_kernel<4> : attn_merge_kernel<16>,
                                      static_cast<const AttnParams>(p), ctas, kv_scale,
                                      static_cast<__nv_bfloat16*>(out)));
  if (rc) return rc;
  return cuda_status(cudaGetLastError());
}

}  // namespace kdb

// moe_gemm.cu — grouped expert GEMMs of the MoE layer.  Two kernels, chosen per launch by a bound on the
// tokens any expert can hold (the caller's; T in the layer forward):
//
// * more than 64: CTA pairs (gemm_grouped_pair_sm100.cuh), weights as the M operand (256 rows per pair),
//   all tokens of one expert (up to 512) as N, so each expert's weights stream from HBM once.
//     gate_up:  H_e = silu(X_e · Wg_eᵀ) * (X_e · Wu_eᵀ) -> bf16 intermediate.  A pair tile covers 128
//               intermediate features; each CTA stages 64 gate rows and the 64 matching up rows (two 64-row
//               boxes of the packed weights), so gate lands in TMEM lanes 0-63 and up in lanes 64-127, and
//               the two halves meet through shared memory in the epilogue.
//     down:     Y_e = H_e · Wd_eᵀ (* routing weight of the row) -> bf16.  A pair tile covers 256 output
//               features, 128 per CTA.
// * at most 64 (decode): one CTA per 256 weight rows on the swapped-operand core (gemm_swap_sm100.cuh),
//   a pure weight stream; measured faster than the pairs when tiles carry this few tokens.
//
// The tile schedule is read on the device from the routing plan (offsets[g], and mtile_start[g], the
// prefix of ceil(count / 512)), so no host synchronisation separates routing from the GEMMs and the whole
// layer is graph-capturable.  Tiles are ordered expert-major, then by weight tile, then by 512-token chunk:
// an expert with more than 512 tokens has its chunks of one weight tile in flight together.
//
// Reference counterparts: the gate_up stage + SwiGLU epilogue warp of the H200 engines
// (okc-challenge/engines/sc_h.cu:164-187, 322-340) and their down stage + weighted output
// (sc_h.cu:341-381, x7_h.cu:438-590), which stream NVFP4 weights through mma.sync.
#include "gemm_grouped_pair_sm100.cuh"
#include "gemm_sm100.cuh"
#include "gemm_swap_sm100.cuh"
#include "host_util.h"
#include "moe.h"

namespace kdb {

static_assert(kMoeTokenTile == kGpTokens, "plan tile prefix and GEMM tile size agree");

// ---------------------------------------------------------------------------------------------------
// Tiles (group g, weight tile f, token chunk j), j fastest.
struct GroupedPairSched {
  struct Params {
    const int* offsets;       // [groups + 1] token-row offsets, or null: one dense group of `rows` rows
    const int* tile_start;    // [groups + 1] exclusive prefix of ceil(count / 512), or null
    int groups, rows, f_tiles, nkb;
    int a_rows_per_group;     // weight rows of one group
    int a_f_stride;           // weight rows between consecutive weight tiles
    int a_box_stride;         // offset of a CTA's second 64-row box (gate_up: gate -> up rows)
    int a_rank_stride;        // offset of CTA 1's rows
    int f_step;               // output features per weight tile
  };
  Params p;
  int total_tt;
  __device__ explicit GroupedPairSched(const Params& pp) : p(pp) {
    total_tt = p.tile_start ? p.tile_start[p.groups] : (p.rows + kGpTokens - 1) / kGpTokens;
  }
  __device__ int num_tiles() const { return total_tt * p.f_tiles; }
  __device__ GpTile tile(int t) const {
    int g = 0, tstart = 0, tcount = total_tt, row_begin = 0, count = p.rows;
    if (p.tile_start) {
      int lo = 0, hi = p.groups - 1;
      while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (__ldg(p.tile_start + mid) * p.f_tiles <= t) lo = mid;
        else hi = mid - 1;
      }
      g = lo;
      tstart = __ldg(p.tile_start + g);
      tcount = __ldg(p.tile_start + g + 1) - tstart;
      row_begin = __ldg(p.offsets + g);
      count = __ldg(p.offsets + g + 1) - row_begin;
    }
    const int local = t - tstart * p.f_tiles;
    const int f = local / tcount;
    const int j = local - f * tcount;
    GpTile ti;
    ti.b_row = row_begin + j * kGpTokens;
    ti.n_valid = min(kGpTokens, count - j * kGpTokens);
    ti.a_row = g * p.a_rows_per_group + f * p.a_f_stride;
    ti.a_box_stride = p.a_box_stride;
    ti.a_rank_stride = p.a_rank_stride;
    ti.f0 = f * p.f_step;
    ti.nkb = p.nkb;
    return ti;
  }
};

__device__ __forceinline__ float silu_f(float g) { return __fdividef(g, 1.0f + __expf(-g)); }

// Copy-out of one transposed chunk: `rows` token rows of `width` bf16 features from shared memory
// (row-major, width * 2 bytes per row) to out[row0 + r][f0 ...] with 16-byte stores, 128 threads.
template <int kWidth>
__device__ __forceinline__ void epi_copy_out(const __nv_bfloat16* tile, int rows, __nv_bfloat16* out, long long ld,
                                             long long row0, int f0, int n_feat, bool vec_ok, int etid) {
  constexpr int kVecPerRow = kWidth / 8;
#pragma unroll
  for (int pass = 0; pass < 32 * kVecPerRow / 128; ++pass) {
    const int idx = pass * 128 + etid;
    const int r = idx / kVecPerRow, c8 = (idx % kVecPerRow) * 8;
    if (r >= rows) continue;
    const int f = f0 + c8;
    __nv_bfloat16* dst = out + (row0 + r) * ld + f;
    const __nv_bfloat16* src = tile + r * kWidth + c8;
    if (vec_ok && f + 8 <= n_feat) {
      *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(src);
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e)
        if (f + e < n_feat) dst[e] = src[e];
    }
  }
}

// gate_up: in each epilogue group, warps of lane quarters 0, 1 hold the gate rows of features 32q..32q+31 of
// this CTA's 64, quarters 2, 3 the up rows of the same features.  Per 32-token chunk the gate warps hand
// tokens 16..31 to the up warps and the up warps hand tokens 0..15 to the gate warps (fp32 through shared
// memory, row stride 17: conflict-free), each side computes silu(gate) * up for its 16 tokens into a bf16
// [32 tokens][64 features] tile, and the group stores the tile's rows with 16-byte vectors.
struct SwigluGpEpi {
  static constexpr int kXFloats = 64 * 17;
  struct Params;
  __device__ static void init_smem(uint8_t*, int) {}
  __device__ static void after_release(const Params&, const GpTile&, int, int, int, int, uint8_t*, int, int) {}
  static constexpr int kSmemBytes = 2 * kXFloats * 4 + 32 * 64 * 2;
  struct Params {
    __nv_bfloat16* out;   // [rows, ld_out] intermediate
    int ld_out;
    int n_feat;           // intermediate features (I)
    bool vec_ok;          // out 16-byte aligned and ld_out % 8 == 0
  };
  __device__ static void run(const Params& p, const GpTile& ti, int quad, int lane, int rank, int grp,
                             uint32_t taddr, int tok0, int ncols, uint8_t* smem, uint32_t&) {
    float* xg = reinterpret_cast<float*>(smem);   // gate of tokens 16..31
    float* xu = xg + kXFloats;                    // up of tokens 0..15
    __nv_bfloat16* tile = reinterpret_cast<__nv_bfloat16*>(smem + 2 * kXFloats * 4);
    const int j = (quad & 1) * 32 + lane;
    const bool up = quad >= 2;
    const int fbase = ti.f0 + rank * 64;
#pragma unroll 1
    for (int c0 = 32 * grp; c0 < ncols; c0 += 64) {
      uint32_t v[32];
      tmem_ld_32x32b_x32(taddr + c0, v);
      tmem_ld_wait();
      if (up) {
#pragma unroll
        for (int i = 0; i < 16; ++i) xu[j * 17 + i] = __uint_as_float(v[i]);
      } else {
#pragma unroll
        for (int i = 0; i < 16; ++i) xg[j * 17 + i] = __uint_as_float(v[16 + i]);
      }
      epi_bar_sync(grp);
      if (up) {
#pragma unroll
        for (int i = 0; i < 16; ++i)
          tile[(16 + i) * 64 + j] = __float2bfloat16_rn(silu_f(xg[j * 17 + i]) * __uint_as_float(v[16 + i]));
      } else {
#pragma unroll
        for (int i = 0; i < 16; ++i)
          tile[i * 64 + j] = __float2bfloat16_rn(silu_f(__uint_as_float(v[i])) * xu[j * 17 + i]);
      }
      epi_bar_sync(grp);
      epi_copy_out<64>(tile, min(32, ncols - c0), p.out, p.ld_out, ti.b_row + tok0 + c0, fbase, p.n_feat, p.vec_ok,
                       quad * 32 + lane);
    }
  }
};

// down: lane row r of this CTA = output feature f0 + 128 * rank + r; each token row scaled by its routing
// weight (1 when row_scale is null).  Per 32-token chunk a group writes a bf16 [32 tokens][128 features]
// tile (double-buffered) and stores its rows with 16-byte vectors.
struct ScaleGpEpi {
  static constexpr int kTileElems = 32 * 128;
  struct Params;
  __device__ static void init_smem(uint8_t*, int) {}
  __device__ static void after_release(const Params&, const GpTile&, int, int, int, int, uint8_t*, int, int) {}
  static constexpr int kSmemBytes = 2 * kTileElems * 2;
  struct Params {
    __nv_bfloat16* out;       // [rows, ld_out]
    const float* row_scale;   // [rows] or null
    int ld_out;
    int n_total;              // valid output features
    bool vec_ok;              // out 16-byte aligned and ld_out % 8 == 0
  };
  __device__ static void run(const Params& p, const GpTile& ti, int quad, int lane, int rank, int grp,
                             uint32_t taddr, int tok0, int ncols, uint8_t* smem, uint32_t& seq) {
    const int r = quad * 32 + lane;
    const int fbase = ti.f0 + rank * 128;
    const int row_base = ti.b_row + tok0;
#pragma unroll 1
    for (int c0 = 32 * grp; c0 < ncols; c0 += 64, ++seq) {
      __nv_bfloat16* tile = reinterpret_cast<__nv_bfloat16*>(smem) + (seq & 1u) * kTileElems;
      const int n = min(32, ncols - c0);
      const float my_scale = (p.row_scale && lane < n) ? __ldg(p.row_scale + row_base + c0 + lane) : 1.0f;
      uint32_t v[32];
      tmem_ld_32x32b_x32(taddr + c0, v);
      tmem_ld_wait();
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const float sc = __shfl_sync(0xffffffffu, my_scale, i);
        tile[i * 128 + r] = __float2bfloat16_rn(__uint_as_float(v[i]) * sc);
      }
      epi_bar_sync(grp);
      epi_copy_out<128>(tile, n, p.out, p.ld_out, row_base + c0, fbase, p.n_total, p.vec_ok, r);
    }
  }
};

// down with the weighted combine fused in.  As ScaleGpEpi, each 32-token chunk's scaled bf16 rows go to the
// per-slot buffer `out`.  Once the accumulator slot is handed back to the MMA (after_release), every row of
// the slot counts one arrival on (its token, this CTA's 128-feature block), and the tile whose arrival
// completes a token's block (k arrivals: one per routed expert) merges that block:
// y[t][block] = bf16( sum over j of out[slot_pos[t*k + j]][block] (+ yshared[t][block]) ), fp32 in slot
// order then the shared row, exactly as moe_combine_kernel, so the result does not depend on which tile
// arrives last.  Running the arrivals and merges after the release overlaps their memory latency (the
// merge reads other tiles' rows, mostly from HBM) with the next tile's MMAs.  Ordering (the release /
// acquire pattern of a split-K semaphore): the group meets at a barrier after its slot-row stores, its first
// warp fences (release) and makes the arrivals; a warp that completed a block fences again (acquire) before
// the barrier that hands the list to the group, and merge reads bypass L1.  The arrival counters
// ([T, H / 128] int32) are zeroed before the launch.
struct ScaleCombineGpEpi {
  static constexpr int kTileElems = 32 * 128;
  static constexpr int kListInts = 132;   // [0] count, then the tokens to merge (<= 128 rows per group and slot)
  static constexpr int kSmemBytes = kTileElems * 2 + kListInts * 4;
  static_assert(kSmemBytes % 16 == 0, "the second epilogue group's tile must stay 16-byte aligned");
  struct Params {
    __nv_bfloat16* out;           // [rows, ld_out] per-slot rows (scaled)
    const float* row_scale;       // [rows]
    int ld_out;                   // = H, a multiple of 128
    const int* perm_slot;         // [rows]: slot t*k + j held by each permuted row
    const int* slot_pos;          // [T*k]: permuted row of each slot (< 0: none)
    int* arrivals;                // [T, ld_out / 128], zero at launch
    const __nv_bfloat16* yshared; // [T, ld_out] or null
    __nv_bfloat16* y;             // [T, ld_out]
    int k;
  };
  __device__ static int* list_of(uint8_t* smem) { return reinterpret_cast<int*>(smem + kTileElems * 2); }
  __device__ static void init_smem(uint8_t* smem, int etid) {
    if (etid == 0) list_of(smem)[0] = 0;
  }

  __device__ static void run(const Params& p, const GpTile& ti, int quad, int lane, int rank, int grp,
                             uint32_t taddr, int tok0, int ncols, uint8_t* smem, uint32_t&) {
    const int r = quad * 32 + lane;
    const int fbase = ti.f0 + rank * 128;
    if (fbase >= p.ld_out) return;   // CTA 1 of a last pair tile past H (H % 256 == 128): no features
    const int row_base = ti.b_row + tok0;
    __nv_bfloat16* tile = reinterpret_cast<__nv_bfloat16*>(smem);
#pragma unroll 1
    for (int c0 = 32 * grp; c0 < ncols; c0 += 64) {
      const int n = min(32, ncols - c0);
      const float my_scale = lane < n ? __ldg(p.row_scale + row_base + c0 + lane) : 1.0f;
      uint32_t v[32];
      tmem_ld_32x32b_x32(taddr + c0, v);
      tmem_ld_wait();
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const float sc = __shfl_sync(0xffffffffu, my_scale, i);
        tile[i * 128 + r] = __float2bfloat16_rn(__uint_as_float(v[i]) * sc);
      }
      epi_bar_sync(grp);
      epi_copy_out<128>(tile, n, p.out, p.ld_out, row_base + c0, fbase, p.ld_out, true, r);
      epi_bar_sync(grp);   // the tile buffer is free again
    }
  }

  // After the accumulator slot is released: count this group's rows of the slot, merge the blocks they
  // complete, then clear the list.
  __device__ static void after_release(const Params& p, const GpTile& ti, int quad, int lane, int rank, int grp,
                                       uint8_t* smem, int tok0, int ncols) {
    const int etid = quad * 32 + lane;
    const int fbase = ti.f0 + rank * 128;
    if (fbase >= p.ld_out) return;
    const int nfb = p.ld_out >> 7;
    const int fb = fbase >> 7;
    int* list = list_of(smem);
    // Arrivals by the group's first warp only (the split-K semaphore pattern): the group barrier orders
    // every thread's slot-row stores before that warp's fence, which then releases them (cumulatively)
    // ahead of its relaxed atomics, one fence per group and slot instead of one per thread.
    epi_bar_sync(grp);
    if (etid < 32) {
      asm volatile("fence.acq_rel.gpu;" ::: "memory");
      // the group's rows: chunks c0 = 32 * grp + 64 * i (i < 4); lane l takes row l of each chunk
      int tok[4], old[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int c = 32 * grp + 64 * i + etid;
        tok[i] = c < ncols ? __ldg(p.perm_slot + ti.b_row + tok0 + c) / p.k : -1;
      }
#pragma unroll
      for (int i = 0; i < 4; ++i)
        old[i] = tok[i] >= 0 ? atomicAdd(p.arrivals + static_cast<long long>(tok[i]) * nfb + fb, 1) : -1;
      bool any_last = false;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        if (old[i] == p.k - 1) {
          any_last = true;
          list[1 + atomicAdd(list, 1)] = tok[i];
        }
      }
      // acquire: the other tiles' rows of the completed blocks are visible to the group after the barrier
      if (__any_sync(0xffffffffu, any_last)) asm volatile("fence.acq_rel.gpu;" ::: "memory");
    }
    epi_bar_sync(grp);
    const int nm = list[0];
    const int c8 = (etid & 15) * 8;
#pragma unroll 1
    for (int m = etid >> 4; m < nm; m += 8) {
      const int tok = list[1 + m];
      const int* sp = p.slot_pos + static_cast<long long>(tok) * p.k;
      float acc[8];
#pragma unroll
      for (int q = 0; q < 8; ++q) acc[q] = 0.f;
#pragma unroll 1
      for (int j0 = 0; j0 < p.k; j0 += 8) {
        const int nj = min(8, p.k - j0);
        int pos[8];
        uint4 u[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) pos[j] = j < nj ? __ldg(sp + j0 + j) : -1;
#pragma unroll
        for (int j = 0; j < 8; ++j)   // all loads of the group in flight before any add
          u[j] = pos[j] >= 0 ? __ldcg(reinterpret_cast<const uint4*>(p.out + static_cast<long long>(pos[j]) * p.ld_out +
                                                                     fbase + c8))
                             : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          if (pos[j] < 0) continue;
          const __nv_bfloat162* b = reinterpret_cast<const __nv_bfloat162*>(&u[j]);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const float2 f = __bfloat1622float2(b[q]);
            acc[2 * q] += f.x;
            acc[2 * q + 1] += f.y;
          }
        }
      }
      if (p.yshared) {
        const uint4 u = __ldcg(reinterpret_cast<const uint4*>(p.yshared + static_cast<long long>(tok) * p.ld_out +
                                                              fbase + c8));
        const __nv_bfloat162* b = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float2 f = __bfloat1622float2(b[q]);
          acc[2 * q] += f.x;
          acc[2 * q + 1] += f.y;
        }
      }
      uint4 o;
      o.x = pack_bf16x2(acc[0], acc[1]);
      o.y = pack_bf16x2(acc[2], acc[3]);
      o.z = pack_bf16x2(acc[4], acc[5]);
      o.w = pack_bf16x2(acc[6], acc[7]);
      *reinterpret_cast<uint4*>(p.y + static_cast<long long>(tok) * p.ld_out + fbase + c8) = o;
    }
    epi_bar_sync(grp);   // every thread has read the list
    if (etid == 0) list[0] = 0;
  }
};

// ---------------------------------------------------------------------------------------------------
// Weight-streaming path (every group holds <= 64 tokens, as in decode): one CTA per tile of 256 weight rows
// (two 128-row parts) x the group's tokens on the single-CTA swapped-operand core (gemm_swap_sm100.cuh).
// Measured faster than the pair kernel when the tiles carry so few tokens that the kernel only streams
// weights.  Tiles (group g, weight tile f); a group's tile prefix counts 1 per non-empty group here.
struct StreamSched {
  struct Params {
    const int* offsets;       // [groups + 1] token-row offsets, or null: one dense group of `rows` rows
    const int* tile_start;    // [groups + 1] exclusive prefix of ceil(count / 512) (0 or 1 per group), or null
    int groups, rows, f_tiles, nkb;
    int a_rows_per_group;     // weight rows of one group
    int a_tile_rows;          // weight rows one tile spans (two 128-row parts)
    int a_part_stride;        // offset of part 1
    int f_step;               // output features per weight tile
  };
  Params p;
  int total_groups;
  __device__ explicit StreamSched(const Params& pp) : p(pp) {
    total_groups = p.tile_start ? p.tile_start[p.groups] : (p.rows > 0 ? 1 : 0);
  }
  __device__ int num_tiles() const { return total_groups * p.f_tiles; }
  __device__ SwapTile tile(int t) const {
    int g = 0, row_begin = 0, count = p.rows, gstart = 0;
    if (p.tile_start) {
      int lo = 0, hi = p.groups - 1;
      while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (__ldg(p.tile_start + mid) * p.f_tiles <= t) lo = mid;
        else hi = mid - 1;
      }
      g = lo;
      gstart = __ldg(p.tile_start + g);
      row_begin = __ldg(p.offsets + g);
      count = __ldg(p.offsets + g + 1) - row_begin;
    }
    const int f = t - gstart * p.f_tiles;
    SwapTile ti;
    ti.row0 = row_begin;
    ti.n_valid = min(64, count);
    ti.b_row = row_begin;
    ti.a_row = g * p.a_rows_per_group + f * p.a_tile_rows;
    ti.a_part_stride = p.a_part_stride;
    ti.f0 = f * p.f_step;
    ti.kb0 = 0;
    ti.nkb = p.nkb;
    ti.split = 0;
    return ti;
  }
};

// gate_up: accumulator part 0 = gate rows f0..f0+127, part 1 = the up rows of the same features.
struct SwigluStreamEpi {
  struct Params {
    __nv_bfloat16* out;   // [rows, ld_out] intermediate
    int ld_out;
  };
  template <int NB>
  __device__ static void run(const Params& p, const SwapTile& ti, int r, uint32_t taddr) {
    __nv_bfloat16* col = p.out + ti.f0 + r;
#pragma unroll 1
    for (int c0 = 0; c0 < ti.n_valid; c0 += 32) {
      uint32_t g[32], u[32];
      tmem_ld_32x32b_x32(taddr + c0, g);
      tmem_ld_32x32b_x32(taddr + NB + c0, u);
      tmem_ld_wait();
      const int n = min(32, ti.n_valid - c0);
      __nv_bfloat16* dst = col + static_cast<long long>(ti.row0 + c0) * p.ld_out;
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if (i < n)
          dst[static_cast<long long>(i) * p.ld_out] =
              __float2bfloat16_rn(silu_f(__uint_as_float(g[i])) * __uint_as_float(u[i]));
    }
  }
};

// down: accumulator parts 0 and 1 = output features f0..f0+127 and f0+128..f0+255, each token row scaled
// by its routing weight (1 when row_scale is null).
struct ScaleStreamEpi {
  struct Params {
    __nv_bfloat16* out;       // [rows, ld_out]
    const float* row_scale;   // [rows] or null
    int ld_out;
    int n_total;              // valid output features
  };
  template <int NB>
  __device__ static void run(const Params& p, const SwapTile& ti, int r, uint32_t taddr) {
#pragma unroll 1
    for (int a = 0; a < 2; ++a) {
      const int feat = ti.f0 + a * 128 + r;
      const bool ok = feat < p.n_total;
      __nv_bfloat16* col = p.out + feat;
#pragma unroll 1
      for (int c0 = 0; c0 < ti.n_valid; c0 += 32) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(taddr + a * NB + c0, v);
        tmem_ld_wait();
        const int n = min(32, ti.n_valid - c0);
        if (!ok) continue;
        __nv_bfloat16* dst = col + static_cast<long long>(ti.row0 + c0) * p.ld_out;
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          if (i < n) {
            const float sc = p.row_scale ? __ldg(p.row_scale + ti.row0 + c0 + i) : 1.0f;
            dst[static_cast<long long>(i) * p.ld_out] = __float2bfloat16_rn(__uint_as_float(v[i]) * sc);
          }
        }
      }
    }
  }
};

template <class Kern>
static int ensure_smem_attr(Kern kern, int bytes, bool* done) {
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return KDB_ERR_NO_DEVICE;
  if (!done[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e != cudaSuccess) return cuda_status(e);
    done[dev] = true;
  }
  return KDB_OK;
}

template <class Epi, int ABOXES>
static int launch_grouped_pair(const void* tokens, int a_rows, const void* weights, uint64_t weight_rows, int K,
                               const GroupedPairSched::Params& sp, const typename Epi::Params& ep, cudaStream_t s) {
  constexpr int kStages = 4;   // 48 KB per stage: 128 weight rows + two 128-row token groups
  using L = GpLayout<ABOXES, kStages, 2 * Epi::kSmemBytes>;
  auto kern = gemm_grouped_pair_kernel<GroupedPairSched, Epi, ABOXES, kStages>;
  static bool done[64] = {false};
  int rc = ensure_smem_attr(kern, L::kSmemBytes, done);
  if (rc) return rc;
  CUtensorMap ta;
  TokenMaps tb;
  rc = make_tmap_bf16_2d(&ta, weights, K, weight_rows, K, kBK, L::kABoxRows);
  if (rc) return rc;
  rc = make_token_maps(&tb, tokens, a_rows, K);
  if (rc) return rc;
  int pairs = num_sms() / 2;
  if (!sp.tile_start) {
    const int tiles = ((a_rows + kGpTokens - 1) / kGpTokens) * sp.f_tiles;
    pairs = tiles < pairs ? tiles : pairs;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * pairs, 1, 1);
  cfg.blockDim = dim3(kGpThreads, 1, 1);
  cfg.dynamicSmemBytes = L::kSmemBytes;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cuda_status(cudaLaunchKernelEx(&cfg, kern, ta, tb, sp, ep));
}

template <class Epi>
static int launch_stream(const void* tokens, int a_rows, const void* weights, uint64_t weight_rows, int K,
                         const StreamSched::Params& sp, const typename Epi::Params& ep, cudaStream_t s) {
  constexpr int MA = 2, NB = 64, STAGES = 5;
  using L = SwapLayout<MA, NB, STAGES>;
  auto kern = gemm_swap_kernel<StreamSched, Epi, MA, NB, STAGES>;
  static bool done[64] = {false};
  int rc = ensure_smem_attr(kern, L::kSmemBytes, done);
  if (rc) return rc;
  CUtensorMap ta;
  TokenMaps tb;
  rc = make_tmap_bf16_2d(&ta, weights, K, weight_rows, K, kBK, 128);
  if (rc) return rc;
  rc = make_token_maps(&tb, tokens, a_rows, K);
  if (rc) return rc;
  int grid = num_sms();
  if (!sp.tile_start) grid = sp.f_tiles < grid ? sp.f_tiles : grid;
  kern<<<grid, kGemmThreads, L::kSmemBytes, s>>>(ta, tb, sp, ep);
  return cuda_status(cudaGetLastError());
}

int moe_gemm_gate_up(const void* a, int a_rows, const void* w_packed, int groups, int I, int H, const int* offsets,
                     const int* mtile_start, void* out, cudaStream_t s, int max_group_tokens) {
  if (a_rows <= 0) return KDB_OK;
  const int bound = max_group_tokens > 0 && max_group_tokens < a_rows ? max_group_tokens : a_rows;
  if (bound <= 64) {
    StreamSched::Params sp;
    sp.offsets = offsets;
    sp.tile_start = mtile_start;
    sp.groups = groups;
    sp.rows = a_rows;
    sp.f_tiles = I / 128;      // 128 intermediate features (one packed block) per tile
    sp.nkb = (H + kBK - 1) / kBK;
    sp.a_rows_per_group = 2 * I;
    sp.a_tile_rows = 256;
    sp.a_part_stride = 128;
    sp.f_step = 128;
    SwigluStreamEpi::Params ep;
    ep.out = static_cast<__nv_bfloat16*>(out);
    ep.ld_out = I;
    return launch_stream<SwigluStreamEpi>(a, a_rows, w_packed, static_cast<uint64_t>(groups) * 2 * I, H, sp, ep, s);
  }
  GroupedPairSched::Params sp;
  sp.offsets = offsets;
  sp.tile_start = mtile_start;
  sp.groups = groups;
  sp.rows = a_rows;
  sp.f_tiles = I / 128;        // one packed block (128 gate + 128 up rows) per pair tile
  sp.nkb = (H + kBK - 1) / kBK;
  sp.a_rows_per_group = 2 * I;
  sp.a_f_stride = 256;
  sp.a_box_stride = 128;       // gate row r -> its up row r + 128 within the packed block
  sp.a_rank_stride = 64;       // CTA 1 takes features 64..127 of the block
  sp.f_step = 128;
  SwigluGpEpi::Params ep;
  ep.out = static_cast<__nv_bfloat16*>(out);
  ep.ld_out = I;
  ep.n_feat = I;
  ep.vec_ok = aligned16(out) && I % 8 == 0;
  return launch_grouped_pair<SwigluGpEpi, 2>(a, a_rows, w_packed, static_cast<uint64_t>(groups) * 2 * I, H, sp, ep,
                                             s);
}

int moe_gemm_down(const void* a, int a_rows, const void* w_down, int groups, int I, int H, const int* offsets,
                  const int* mtile_start, const float* row_scale, void* out, cudaStream_t s, int max_group_tokens) {
  if (a_rows <= 0) return KDB_OK;
  const int bound = max_group_tokens > 0 && max_group_tokens < a_rows ? max_group_tokens : a_rows;
  if (bound <= 64) {
    StreamSched::Params sp;
    sp.offsets = offsets;
    sp.tile_start = mtile_start;
    sp.groups = groups;
    sp.rows = a_rows;
    sp.f_tiles = (H + 255) / 256;   // 256 output features (two 128-row parts) per tile
    sp.nkb = (I + kBK - 1) / kBK;
    sp.a_rows_per_group = H;
    sp.a_tile_rows = 256;
    sp.a_part_stride = 128;
    sp.f_step = 256;
    ScaleStreamEpi::Params ep;
    ep.out = static_cast<__nv_bfloat16*>(out);
    ep.row_scale = row_scale;
    ep.ld_out = H;
    ep.n_total = H;
    return launch_stream<ScaleStreamEpi>(a, a_rows, w_down, static_cast<uint64_t>(groups) * H, I, sp, ep, s);
  }
  GroupedPairSched::Params sp;
  sp.offsets = offsets;
  sp.tile_start = mtile_start;
  sp.groups = groups;
  sp.rows = a_rows;
  sp.f_tiles = (H + 255) / 256;   // 256 output features per pair tile
  sp.nkb = (I + kBK - 1) / kBK;
  sp.a_rows_per_group = H;
  sp.a_f_stride = 256;
  sp.a_box_stride = 0;
  sp.a_rank_stride = 128;
  sp.f_step = 256;
  ScaleGpEpi::Params ep;
  ep.out = static_cast<__nv_bfloat16*>(out);
  ep.row_scale = row_scale;
  ep.ld_out = H;
  ep.n_total = H;
  ep.vec_ok = aligned16(out) && H % 8 == 0;
  return launch_grouped_pair<ScaleGpEpi, 1>(a, a_rows, w_down, static_cast<uint64_t>(groups) * H, I, sp, ep, s);
}

int moe_gemm_down_combine(const void* a, int a_rows, const void* w_down, int groups, int I, int H,
                          const int* offsets, const int* mtile_start, const float* row_scale, const int* perm_slot,
                          const int* slot_pos, int* arrivals, const void* yshared, void* rows_out, void* y, int T,
                          int k, cudaStream_t s) {
  if (T <= 0 || a_rows <= 0) return KDB_OK;
  if (H % 128 != 0 || !aligned16(rows_out) || !aligned16(y) || (yshared && !aligned16(yshared)))
    return KDB_ERR_UNSUPPORTED;
  int rc = cuda_status(cudaMemsetAsync(arrivals, 0, sizeof(int) * static_cast<size_t>(T) * (H / 128), s));
  if (rc) return rc;
  GroupedPairSched::Params sp;
  sp.offsets = offsets;
  sp.tile_start = mtile_start;
  sp.groups = groups;
  sp.rows = a_rows;
  sp.f_tiles = (H + 255) / 256;   // 256 output features per pair tile
  sp.nkb = (I + kBK - 1) / kBK;
  sp.a_rows_per_group = H;
  sp.a_f_stride = 256;
  sp.a_box_stride = 0;
  sp.a_rank_stride = 128;
  sp.f_step = 256;
  ScaleCombineGpEpi::Params ep;
  ep.out = static_cast<__nv_bfloat16*>(rows_out);
  ep.row_scale = row_scale;
  ep.ld_out = H;
  ep.perm_slot = perm_slot;
  ep.slot_pos = slot_pos;
  ep.arrivals = arrivals;
  ep.yshared = static_cast<const __nv_bfloat16*>(yshared);
  ep.y = static_cast<__nv_bfloat16*>(y);
  ep.k = k;
  (void)T;
  return launch_grouped_pair<ScaleCombineGpEpi, 1>(a, a_rows, w_down, static_cast<uint64_t>(groups) * H, I, sp, ep,
                                                   s);
}

}  // namespace kdb

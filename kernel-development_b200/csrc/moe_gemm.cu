// moe_gemm.cu — grouped expert GEMMs of the MoE layer on the persistent tcgen05 core with swapped
// operands (gemm_swap_sm100.cuh: weights as M, each expert's tokens as N rounded up to 16).
//
//   gate_up:  H_e = silu(X_e · Wg_eᵀ) * (X_e · Wu_eᵀ) -> bf16 intermediate; one tile = 128 gate rows and
//             the matching 128 up rows of the packed weights against <= 128 token rows
//   down:     Y_e = H_e · Wd_eᵀ (* routing weight of the row) -> bf16; one tile = 256 output features
//             against <= 128 token rows
//
// The tile schedule is read on the device from the routing plan (offsets[g], mtile_start[g]), so no
// host synchronisation separates routing from the GEMMs and the whole layer is graph-capturable.
// Tiles are ordered expert-major, then by weight tile, with token tiles fastest: the tiles in flight
// at once share an expert's weight tiles in L2.
//
// Reference counterparts: the gate_up stage + SwiGLU epilogue warp of the H200 engines
// (okc-challenge/engines/sc_h.cu:164-187, 322-340) and their down stage + weighted output
// (sc_h.cu:341-381, x7_h.cu:438-590), which stream NVFP4 weights through mma.sync.
#include "gemm_sm100.cuh"
#include "gemm_swap_sm100.cuh"
#include "host_util.h"
#include "moe.h"

namespace kdb {

// ---------------------------------------------------------------------------------------------------
// Swapped-operand grouped schedule: tiles (group g, weight tile f, token tile tt), tt fastest.
struct SwapSched {
  struct Params {
    const int* offsets;       // [groups + 1] token-row offsets, or null: one dense group of `rows` rows
    const int* mtile_start;   // [groups + 1] exclusive prefix of ceil(count / 128), or null
    int groups, rows, f_tiles, nkb;
    int a_rows_per_group;     // weight rows of one group
    int a_tile_rows;          // weight rows one tile spans (two 128-row parts)
    int f_step;               // feature index advance per weight tile
  };
  Params p;
  int total_mt;
  __device__ explicit SwapSched(const Params& pp) : p(pp) {
    total_mt = p.mtile_start ? p.mtile_start[p.groups] : (p.rows + 127) / 128;
  }
  __device__ int num_tiles() const { return total_mt * p.f_tiles; }
  __device__ SwapTile tile(int t) const {
    int g = 0, mstart = 0, mcount = total_mt, row_begin = 0, count = p.rows;
    if (p.mtile_start) {
      int lo = 0, hi = p.groups - 1;
      while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (__ldg(p.mtile_start + mid) * p.f_tiles <= t) lo = mid;
        else hi = mid - 1;
      }
      g = lo;
      mstart = __ldg(p.mtile_start + g);
      mcount = __ldg(p.mtile_start + g + 1) - mstart;
      row_begin = __ldg(p.offsets + g);
      count = __ldg(p.offsets + g + 1) - row_begin;
    }
    const int local = t - mstart * p.f_tiles;
    const int f = local / mcount;
    const int tt = local - f * mcount;
    SwapTile ti;
    ti.row0 = row_begin + tt * 128;
    ti.n_valid = min(128, count - tt * 128);
    ti.b_row = ti.row0;
    ti.a_row = g * p.a_rows_per_group + f * p.a_tile_rows;
    ti.a_part_stride = 128;
    ti.f0 = f * p.f_step;
    ti.kb0 = 0;
    ti.nkb = p.nkb;
    ti.split = 0;
    return ti;
  }
};

__device__ __forceinline__ float silu_swap(float g) { return g / (1.0f + __expf(-g)); }

// gate_up: accumulator part 0 = gate rows f0..f0+127, part 1 = the up rows of the same features.
struct SwigluSwapEpi {
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
              __float2bfloat16_rn(silu_swap(__uint_as_float(g[i])) * __uint_as_float(u[i]));
    }
  }
};

// down: accumulator parts 0 and 1 = output features f0..f0+127 and f0+128..f0+255, each token row
// scaled by its routing weight (1 when row_scale is null).
struct ScaleSwapEpi {
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

constexpr int kSwapMA = 2, kSwapNB = 128, kSwapStages = 4;

template <class Epi>
static int launch_swap(const void* tokens, int a_rows, const void* weights, uint64_t weight_rows, int K,
                       const SwapSched::Params& sp, const typename Epi::Params& ep, cudaStream_t s) {
  using L = SwapLayout<kSwapMA, kSwapNB, kSwapStages>;
  auto kern = gemm_swap_kernel<SwapSched, Epi, kSwapMA, kSwapNB, kSwapStages>;
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
  if (!sp.mtile_start) {
    const int tiles = ((a_rows + 127) / 128) * sp.f_tiles;
    grid = tiles < grid ? tiles : grid;
  }
  kern<<<grid, kGemmThreads, L::kSmemBytes, s>>>(ta, tb, sp, ep);
  return cuda_status(cudaGetLastError());
}

int moe_gemm_gate_up(const void* a, int a_rows, const void* w_packed, int groups, int I, int H, const int* offsets,
                     const int* mtile_start, void* out, cudaStream_t s) {
  if (a_rows <= 0) return KDB_OK;
  SwapSched::Params sp;
  sp.offsets = offsets;
  sp.mtile_start = mtile_start;
  sp.groups = groups;
  sp.rows = a_rows;
  sp.f_tiles = I / 128;               // 128 intermediate features (256 packed weight rows) per tile
  sp.nkb = (H + kBK - 1) / kBK;
  sp.a_rows_per_group = 2 * I;
  sp.a_tile_rows = 256;
  sp.f_step = 128;
  SwigluSwapEpi::Params ep;
  ep.out = static_cast<__nv_bfloat16*>(out);
  ep.ld_out = I;
  return launch_swap<SwigluSwapEpi>(a, a_rows, w_packed, static_cast<uint64_t>(groups) * 2 * I, H, sp, ep, s);
}

int moe_gemm_down(const void* a, int a_rows, const void* w_down, int groups, int I, int H, const int* offsets,
                  const int* mtile_start, const float* row_scale, void* out, cudaStream_t s) {
  if (a_rows <= 0) return KDB_OK;
  SwapSched::Params sp;
  sp.offsets = offsets;
  sp.mtile_start = mtile_start;
  sp.groups = groups;
  sp.rows = a_rows;
  sp.f_tiles = (H + 255) / 256;       // 256 output features per tile
  sp.nkb = (I + kBK - 1) / kBK;
  sp.a_rows_per_group = H;
  sp.a_tile_rows = 256;
  sp.f_step = 256;
  ScaleSwapEpi::Params ep;
  ep.out = static_cast<__nv_bfloat16*>(out);
  ep.row_scale = row_scale;
  ep.ld_out = H;
  ep.n_total = H;
  return launch_swap<ScaleSwapEpi>(a, a_rows, w_down, static_cast<uint64_t>(groups) * H, I, sp, ep, s);
}

}  // namespace kdb

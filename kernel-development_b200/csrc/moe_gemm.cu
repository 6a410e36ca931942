// moe_gemm.cu — grouped expert GEMMs of the MoE layer on the persistent tcgen05 core.
//
//   gate_up:  H_e = X_perm[rows of e] · Wgu_e(packed)ᵀ, epilogue silu(gate) * up -> bf16 intermediate
//   down:     Y_e = H[rows of e] · Wd_eᵀ,  epilogue * routing weight of the row -> bf16 per-slot rows
//
// The tile schedule is read on the device from the routing plan (offsets[g], mtile_start[g]), so no
// host synchronisation separates routing from the GEMMs and the whole layer is graph-capturable.
// Tiles are ordered group-major, then by N-tile, with M-tiles fastest: the tiles in flight at once
// share an expert's weight tiles in L2.
//
// Reference counterparts: the gate_up stage + SwiGLU epilogue warp of the H200 engines
// (okc-challenge/engines/sc_h.cu:164-187, 322-340) and their down stage + weighted output
// (sc_h.cu:341-381, x7_h.cu:438-590), which stream NVFP4 weights through mma.sync.
#include "gemm_sm100.cuh"
#include "host_util.h"
#include "moe.h"

namespace kdb {

struct GroupTile {
  int a_row, b_row, nkb, a_kwrap;
  int row0, valid, n0;
};

template <int BM, int BN>
struct GroupSched {
  struct Params {
    const int* offsets;       // [groups + 1] row offsets, or null: one dense group of `rows` rows
    const int* mtile_start;   // [groups + 1] exclusive prefix of ceil(count / BM), or null
    int groups, rows, n_tiles, nkb;
    int b_rows_per_group;     // B row of (group g, n-tile nb) = g * b_rows_per_group + nb * BN
  };
  Params p;
  int total_mt;
  __device__ explicit GroupSched(const Params& pp) : p(pp) {
    total_mt = p.mtile_start ? p.mtile_start[p.groups] : (p.rows + BM - 1) / BM;
  }
  __device__ int num_tiles() const { return total_mt * p.n_tiles; }
  __device__ GroupTile tile(int t) const {
    GroupTile ti;
    int g = 0, mstart = 0, mcount = total_mt, row_begin = 0, count = p.rows;
    if (p.mtile_start) {
      // largest g with mtile_start[g] * n_tiles <= t (empty groups share their successor's start)
      int lo = 0, hi = p.groups - 1;
      while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (__ldg(p.mtile_start + mid) * p.n_tiles <= t) lo = mid;
        else hi = mid - 1;
      }
      g = lo;
      mstart = __ldg(p.mtile_start + g);
      mcount = __ldg(p.mtile_start + g + 1) - mstart;
      row_begin = __ldg(p.offsets + g);
      count = __ldg(p.offsets + g + 1) - row_begin;
    }
    const int local = t - mstart * p.n_tiles;
    const int nb = local / mcount;
    const int mt = local - nb * mcount;
    ti.row0 = row_begin + mt * BM;
    ti.valid = min(BM, count - mt * BM);
    ti.n0 = nb * BN;
    ti.a_row = ti.row0;
    ti.b_row = g * p.b_rows_per_group + nb * BN;
    ti.nkb = p.nkb;
    ti.a_kwrap = 0;
    return ti;
  }
};

__device__ __forceinline__ float silu_f(float g) { return g / (1.0f + __expf(-g)); }

// BN = 256 tile of the packed gate_up weights: TMEM columns [0, 128) hold gate rows j0..j0+127 and
// [128, 256) the up rows of the same j, so each thread computes silu(g) * u for 128 outputs.
struct SwigluEpi {
  struct Params {
    __nv_bfloat16* out;   // [rows, ld_out]
    int ld_out;
  };
  __device__ static void run(const Params& p, const GroupTile& ti, int r, uint32_t taddr) {
    const bool ok = r < ti.valid;
    __nv_bfloat16* orow = p.out + static_cast<long long>(ti.row0 + r) * p.ld_out + ti.n0 / 2;
#pragma unroll 1
    for (int c = 0; c < 4; ++c) {
      uint32_t g[32], u[32];
      tmem_ld_32x32b_x32(taddr + c * 32, g);
      tmem_ld_32x32b_x32(taddr + 128 + c * 32, u);
      tmem_ld_wait();
      if (!ok) continue;
      uint4* dst = reinterpret_cast<uint4*>(orow + c * 32);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float h[8];
#pragma unroll
        for (int z = 0; z < 8; ++z) h[z] = silu_f(__uint_as_float(g[q * 8 + z])) * __uint_as_float(u[q * 8 + z]);
        uint4 o;
        o.x = pack_bf16x2(h[0], h[1]);
        o.y = pack_bf16x2(h[2], h[3]);
        o.z = pack_bf16x2(h[4], h[5]);
        o.w = pack_bf16x2(h[6], h[7]);
        dst[q] = o;
      }
    }
  }
};

// Down projection: each output row is scaled by its routing weight (1 when row_scale is null).
template <int BN>
struct ScaleEpi {
  struct Params {
    __nv_bfloat16* out;       // [rows, ld_out]
    const float* row_scale;   // [rows] or null
    int ld_out;
    int n_total;              // valid output columns
  };
  __device__ static void run(const Params& p, const GroupTile& ti, int r, uint32_t taddr) {
    const bool ok = r < ti.valid;
    const int row = ti.row0 + r;
    const float sc = (ok && p.row_scale) ? __ldg(p.row_scale + row) : 1.0f;
    __nv_bfloat16* orow = p.out + static_cast<long long>(row) * p.ld_out;
#pragma unroll 1
    for (int c = 0; c < BN / 32; ++c) {
      uint32_t v[32];
      tmem_ld_32x32b_x32(taddr + c * 32, v);
      tmem_ld_wait();
      const int col0 = ti.n0 + c * 32;
      if (!ok || col0 >= p.n_total) continue;
      if (col0 + 32 <= p.n_total) {
        uint4* dst = reinterpret_cast<uint4*>(orow + col0);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint4 o;
          o.x = pack_bf16x2(__uint_as_float(v[q * 8 + 0]) * sc, __uint_as_float(v[q * 8 + 1]) * sc);
          o.y = pack_bf16x2(__uint_as_float(v[q * 8 + 2]) * sc, __uint_as_float(v[q * 8 + 3]) * sc);
          o.z = pack_bf16x2(__uint_as_float(v[q * 8 + 4]) * sc, __uint_as_float(v[q * 8 + 5]) * sc);
          o.w = pack_bf16x2(__uint_as_float(v[q * 8 + 6]) * sc, __uint_as_float(v[q * 8 + 7]) * sc);
          dst[q] = o;
        }
      } else {
        for (int j = 0; j < 32 && col0 + j < p.n_total; ++j)
          orow[col0 + j] = __float2bfloat16_rn(__uint_as_float(v[j]) * sc);
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

constexpr int kGroupBM = 128, kGroupBN = 256, kGroupStages = 4;

int moe_gemm_gate_up(const void* a, int a_rows, const void* w_packed, int groups, int I, int H, const int* offsets,
                     const int* mtile_start, void* out, cudaStream_t s) {
  using L = GemmLayout<kGroupBM, kGroupBN, kGroupStages>;
  using Sched = GroupSched<kGroupBM, kGroupBN>;
  auto kern = gemm_tn_kernel<Sched, SwigluEpi, kGroupBM, kGroupBN, kGroupStages>;
  static bool done[64] = {false};
  int rc = ensure_smem_attr(kern, L::kSmemBytes, done);
  if (rc) return rc;
  if (a_rows <= 0) return KDB_OK;
  CUtensorMap ta, tb;
  rc = make_tmap_bf16_2d(&ta, a, H, a_rows, H, kBK, kGroupBM);
  if (rc) return rc;
  rc = make_tmap_bf16_2d(&tb, w_packed, H, static_cast<uint64_t>(groups) * 2 * I, H, kBK, kGroupBN);
  if (rc) return rc;
  Sched::Params sp;
  sp.offsets = offsets;
  sp.mtile_start = mtile_start;
  sp.groups = groups;
  sp.rows = a_rows;
  sp.n_tiles = (2 * I) / kGroupBN;
  sp.nkb = (H + kBK - 1) / kBK;
  sp.b_rows_per_group = 2 * I;
  SwigluEpi::Params ep;
  ep.out = static_cast<__nv_bfloat16*>(out);
  ep.ld_out = I;
  int grid = num_sms();
  if (!mtile_start) {
    const int tiles = ((a_rows + kGroupBM - 1) / kGroupBM) * sp.n_tiles;
    grid = tiles < grid ? tiles : grid;
  }
  kern<<<grid, kGemmThreads, L::kSmemBytes, s>>>(ta, tb, sp, ep);
  return cuda_status(cudaGetLastError());
}

int moe_gemm_down(const void* a, int a_rows, const void* w_down, int groups, int I, int H, const int* offsets,
                  const int* mtile_start, const float* row_scale, void* out, cudaStream_t s) {
  using L = GemmLayout<kGroupBM, kGroupBN, kGroupStages>;
  using Sched = GroupSched<kGroupBM, kGroupBN>;
  using Epi = ScaleEpi<kGroupBN>;
  auto kern = gemm_tn_kernel<Sched, Epi, kGroupBM, kGroupBN, kGroupStages>;
  static bool done[64] = {false};
  int rc = ensure_smem_attr(kern, L::kSmemBytes, done);
  if (rc) return rc;
  if (a_rows <= 0) return KDB_OK;
  CUtensorMap ta, tb;
  rc = make_tmap_bf16_2d(&ta, a, I, a_rows, I, kBK, kGroupBM);
  if (rc) return rc;
  rc = make_tmap_bf16_2d(&tb, w_down, I, static_cast<uint64_t>(groups) * H, I, kBK, kGroupBN);
  if (rc) return rc;
  Sched::Params sp;
  sp.offsets = offsets;
  sp.mtile_start = mtile_start;
  sp.groups = groups;
  sp.rows = a_rows;
  sp.n_tiles = (H + kGroupBN - 1) / kGroupBN;
  sp.nkb = (I + kBK - 1) / kBK;
  sp.b_rows_per_group = H;
  Epi::Params ep;
  ep.out = static_cast<__nv_bfloat16*>(out);
  ep.row_scale = row_scale;
  ep.ld_out = H;
  ep.n_total = H;
  int grid = num_sms();
  if (!mtile_start) {
    const int tiles = ((a_rows + kGroupBM - 1) / kGroupBM) * sp.n_tiles;
    grid = tiles < grid ? tiles : grid;
  }
  kern<<<grid, kGemmThreads, L::kSmemBytes, s>>>(ta, tb, sp, ep);
  return cuda_status(cudaGetLastError());
}

}  // namespace kdb

// proj.cu — the bf16 dense projection Y[M, N] = X[M, K] · W[N, K]ᵀ (fp32 accumulate, bf16 out).
//
// Replaces the computation behind the `muse_bf16_proj` problem's kernel_fn(data, state)
// (kdev: src/kdev/adapters/okc.py:534-537, config src/kdev/adapters/okc_problems/muse_bf16_proj.toml).
// One persistent tcgen05 kernel (gemm_sm100.cuh); the tile width BN is picked per shape so that
// small-M, weight-streaming shapes still put a tile on every SM.
#include "gemm_pair_sm100.cuh"
#include "gemm_sm100.cuh"
#include "gemm_swap_sm100.cuh"
#include "host_util.h"
#include "moe.h"
#include "proj.h"

namespace kdb {

struct ProjTile {
  int a_row, b_row, nkb, a_kwrap;
  int m0, n0;
};

template <int BM, int BN>
struct ProjSched {
  struct Params {
    int M, N, K;
    int num_m, num_n, group_m;
    int kwrap;   // 0, or k slices after which A's k coordinate wraps (K spans several copies of A's K)
  };
  Params p;
  __device__ explicit ProjSched(const Params& pp) : p(pp) {}
  __device__ int num_tiles() const { return p.num_m * p.num_n; }
  // Grouped raster: group_m consecutive M-blocks sweep the N-blocks together, so the tiles in
  // flight at once share both their X rows and their W rows in L2.
  __device__ ProjTile tile(int t) const {
    const int width = p.group_m * p.num_n;
    const int g = t / width;
    const int first_m = g * p.group_m;
    const int gsz = min(p.num_m - first_m, p.group_m);
    const int r = t - g * width;
    const int mb = first_m + r % gsz;
    const int nb = r / gsz;
    ProjTile ti;
    ti.m0 = mb * BM;
    ti.n0 = nb * BN;
    ti.a_row = ti.m0;
    ti.b_row = ti.n0;
    ti.nkb = (p.K + kBK - 1) / kBK;
    ti.a_kwrap = p.kwrap;
    return ti;
  }
};

template <int BN>
struct ProjEpi {
  struct Params {
    __nv_bfloat16* y;
    long long ldy;
    int M, N;
    int vec_ok;   // y 16-byte aligned and ldy % 8 == 0
  };
  __device__ static void run(const Params& p, const ProjTile& ti, int r, uint32_t taddr) {
    const int row = ti.m0 + r;
    const bool row_ok = row < p.M;
    __nv_bfloat16* yrow = p.y + static_cast<long long>(row) * p.ldy;
#pragma unroll 1
    for (int c = 0; c < BN / 32; ++c) {
      uint32_t v[32];
      tmem_ld_32x32b_x32(taddr + c * 32, v);
      tmem_ld_wait();
      if (!row_ok) continue;
      const int col0 = ti.n0 + c * 32;
      if (col0 >= p.N) continue;
      if (p.vec_ok && col0 + 32 <= p.N) {
        uint4* dst = reinterpret_cast<uint4*>(yrow + col0);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint4 o;
          o.x = pack_bf16x2(__uint_as_float(v[q * 8 + 0]), __uint_as_float(v[q * 8 + 1]));
          o.y = pack_bf16x2(__uint_as_float(v[q * 8 + 2]), __uint_as_float(v[q * 8 + 3]));
          o.z = pack_bf16x2(__uint_as_float(v[q * 8 + 4]), __uint_as_float(v[q * 8 + 5]));
          o.w = pack_bf16x2(__uint_as_float(v[q * 8 + 6]), __uint_as_float(v[q * 8 + 7]));
          dst[q] = o;
        }
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (col0 + j < p.N) yrow[col0 + j] = __float2bfloat16_rn(__uint_as_float(v[j]));
      }
    }
  }
};

template <int BN, int STAGES>
static int launch_proj_cfg(const void* x, const void* w, void* y, int M, int N, int K, long long ldy,
                           cudaStream_t stream) {
  constexpr int BM = 128;
  using L = GemmLayout<BM, BN, STAGES>;
  using Sched = ProjSched<BM, BN>;
  using Epi = ProjEpi<BN>;
  auto kern = gemm_tn_kernel<Sched, Epi, BM, BN, STAGES>;

  static bool attr_done[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_done[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kSmemBytes);
    if (e != cudaSuccess) return cuda_status(e);
    attr_done[dev] = true;
  }

  CUtensorMap ta, tb;
  int rc = make_tmap_bf16_2d(&ta, x, K, M, K, kBK, BM);
  if (rc) return rc;
  rc = make_tmap_bf16_2d(&tb, w, K, N, K, kBK, BN);
  if (rc) return rc;

  typename Sched::Params sp;
  sp.M = M;
  sp.N = N;
  sp.K = K;
  sp.num_m = (M + BM - 1) / BM;
  sp.num_n = (N + BN - 1) / BN;
  sp.kwrap = 0;
  // M-blocks per raster group: as many as keep the group's X rows (group_m x 128 x K bf16) within
  // 64 MiB of L2, so W is streamed from DRAM once per group and the whole of X when it fits.
  {
    const long long per_block = static_cast<long long>(BM) * K * 2;
    long long g = (64ll << 20) / (per_block > 0 ? per_block : 1);
    if (g < 1) g = 1;
    if (g > sp.num_m) g = sp.num_m;
    sp.group_m = static_cast<int>(g);
  }
  typename Epi::Params ep;
  ep.y = static_cast<__nv_bfloat16*>(y);
  ep.ldy = ldy;
  ep.M = M;
  ep.N = N;
  ep.vec_ok = aligned16(y) && (ldy % 8 == 0);

  const int tiles = sp.num_m * sp.num_n;
  const int grid = tiles < num_sms() ? tiles : num_sms();
  kern<<<grid, kGemmThreads, L::kSmemBytes, stream>>>(ta, tb, sp, ep);
  return cuda_status(cudaGetLastError());
}

// CTA-pair variant: 256 x BN tiles on 2-CTA clusters (gemm_pair_sm100.cuh).
template <int BN, int STAGES>
static int launch_proj_pair(const void* x, const void* w, void* y, int M, int N, int K, long long ldy,
                            cudaStream_t stream) {
  constexpr int BM = 256;
  using L = PairLayout<BN, STAGES>;
  using Sched = ProjSched<BM, BN>;
  using Epi = ProjEpi<BN>;
  auto kern = gemm_tn_pair_kernel<Sched, Epi, BN, STAGES>;
  static bool attr_done[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_done[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kSmemBytes);
    if (e != cudaSuccess) return cuda_status(e);
    attr_done[dev] = true;
  }
  CUtensorMap ta, tb;
  int rc = make_tmap_bf16_2d(&ta, x, K, M, K, kBK, 128);
  if (rc) return rc;
  rc = make_tmap_bf16_2d(&tb, w, K, N, K, kBK, BN / 2);
  if (rc) return rc;
  typename Sched::Params sp;
  sp.M = M;
  sp.N = N;
  sp.K = K;
  sp.num_m = (M + BM - 1) / BM;
  sp.num_n = (N + BN - 1) / BN;
  sp.kwrap = 0;
  {
    const long long per_block = static_cast<long long>(BM) * K * 2;
    long long g = (64ll << 20) / (per_block > 0 ? per_block : 1);
    if (g < 1) g = 1;
    if (g > sp.num_m) g = sp.num_m;
    sp.group_m = static_cast<int>(g);
  }
  typename Epi::Params ep;
  ep.y = static_cast<__nv_bfloat16*>(y);
  ep.ldy = ldy;
  ep.M = M;
  ep.N = N;
  ep.vec_ok = aligned16(y) && (ldy % 8 == 0);
  const int tiles = sp.num_m * sp.num_n;
  const int max_pairs = num_sms() / 2;
  const int pairs = tiles < max_pairs ? tiles : max_pairs;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * pairs, 1, 1);
  cfg.blockDim = dim3(kGemmThreads, 1, 1);
  cfg.dynamicSmemBytes = L::kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cuda_status(cudaLaunchKernelEx(&cfg, kern, ta, tb, sp, ep));
}

// ---------------------------------------------------------------------------------------------------
// Small M (weight streaming): W as the 128-row M operand, X's rows as N (rounded up to 16), K split
// over `splits` slices so every SM streams a share of W.  With splits > 1 the epilogue writes fp32
// partials [splits, M, N] into the caller's workspace and proj_reduce_kernel sums them in slice order
// (deterministic) into bf16 Y.
struct ProjSwapSched {
  struct Params {
    int M, N, f_tiles, t_tiles, splits, nkb_total, nkb_per, nb;   // nb: token rows per tile
    int b_kwrap;                                                  // 0, or the token k chunks (wrap)
    int a_tile_rows;                                              // weight rows per tile: 128 or 256 (2 parts)
  };
  Params p;
  __device__ explicit ProjSwapSched(const Params& pp) : p(pp) {}
  __device__ int num_tiles() const { return p.f_tiles * p.t_tiles * p.splits; }
  // order: feature tile, then split, then token tile (fastest)
  __device__ SwapTile tile(int t) const {
    const int tt = t % p.t_tiles;
    const int rest = t / p.t_tiles;
    const int sp = rest % p.splits;
    const int f = rest / p.splits;
    SwapTile ti;
    ti.a_row = f * p.a_tile_rows;
    ti.a_part_stride = 128;
    ti.b_row = tt * p.nb;
    ti.row0 = ti.b_row;
    ti.n_valid = min(p.nb, p.M - ti.row0);
    ti.kb0 = sp * p.nkb_per;
    ti.nkb = min(p.nkb_per, p.nkb_total - ti.kb0);
    ti.f0 = f * p.a_tile_rows;
    ti.split = sp;
    ti.b_kwrap = p.b_kwrap;
    return ti;
  }
};

struct ProjSwapEpi {
  struct Params {
    __nv_bfloat16* y;   // used when partial and y32 are null
    float* y32;         // fp32 output instead of y (when partial is null), or null
    float* partial;     // [splits, M, N] fp32, or null
    long long ldy;
    int M, N;
    int parts;          // 128-row weight parts per tile (accumulators NB columns apart)
  };
  template <int NB>
  __device__ static void run(const Params& p, const SwapTile& ti, int r, uint32_t taddr) {
#pragma unroll 1
    for (int a = 0; a < p.parts; ++a) run_part<NB>(p, ti, ti.f0 + a * 128 + r, taddr + a * NB);
  }
  template <int NB>
  __device__ static void run_part(const Params& p, const SwapTile& ti, int feat, uint32_t taddr) {
    const bool ok = feat < p.N;
#pragma unroll 1
    for (int c0 = 0; c0 < ti.n_valid; c0 += 32) {
      uint32_t v[32];
      tmem_ld_32x32b_x32(taddr + c0, v);
      tmem_ld_wait();
      const int n = min(32, ti.n_valid - c0);
      if (!ok) continue;
      if (p.partial) {
        float* dst = p.partial + (static_cast<long long>(ti.split) * p.M + ti.row0 + c0) * p.N + feat;
#pragma unroll
        for (int i = 0; i < 32; ++i)
          if (i < n) dst[static_cast<long long>(i) * p.N] = __uint_as_float(v[i]);
      } else if (p.y32) {
        float* dst = p.y32 + static_cast<long long>(ti.row0 + c0) * p.ldy + feat;
#pragma unroll
        for (int i = 0; i < 32; ++i)
          if (i < n) dst[static_cast<long long>(i) * p.ldy] = __uint_as_float(v[i]);
      } else {
        __nv_bfloat16* dst = p.y + static_cast<long long>(ti.row0 + c0) * p.ldy + feat;
#pragma unroll
        for (int i = 0; i < 32; ++i)
          if (i < n) dst[static_cast<long long>(i) * p.ldy] = __float2bfloat16_rn(__uint_as_float(v[i]));
      }
    }
  }
};

// y[m, n] = bf16(sum_s partial[s, m, n]) (or the fp32 sum into y32), s ascending.
__global__ void __launch_bounds__(256)
    proj_reduce_kernel(const float* __restrict__ partial, __nv_bfloat16* __restrict__ y, float* __restrict__ y32,
                       long long ldy, int M, int N, int splits) {
  const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  const long long total = static_cast<long long>(M) * N;
  if (idx >= total) return;
  const long long m = idx / N, n = idx % N;
  float acc = 0.f;
  for (int s = 0; s < splits; ++s) acc += partial[static_cast<long long>(s) * total + idx];
  if (y32) y32[m * ldy + n] = acc;
  else y[m * ldy + n] = __float2bfloat16_rn(acc);
}

// The same with four consecutive columns per thread (N % 4 == 0, ldy % 4 == 0, y 8-byte aligned): 16-byte
// partial loads, the slices' loads issued together, summed in slice order as above.
__global__ void __launch_bounds__(256)
    proj_reduce4_kernel(const float4* __restrict__ partial, __nv_bfloat16* __restrict__ y, float* __restrict__ y32,
                        long long ldy, int M, int N, int splits) {
  const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  const long long n4 = N / 4, total4 = static_cast<long long>(M) * n4;
  if (idx >= total4) return;
  const long long m = idx / n4, n = (idx % n4) * 4;
  float4 acc = partial[idx];
  for (int s0 = 1; s0 < splits; s0 += 4) {
    float4 v[4];
#pragma unroll
    for (int j = 0; j < 4; ++j)
      if (s0 + j < splits) v[j] = partial[static_cast<long long>(s0 + j) * total4 + idx];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (s0 + j < splits) {
        acc.x += v[j].x;
        acc.y += v[j].y;
        acc.z += v[j].z;
        acc.w += v[j].w;
      }
    }
  }
  if (y32) {
    y32[m * ldy + n] = acc.x;
    y32[m * ldy + n + 1] = acc.y;
    y32[m * ldy + n + 2] = acc.z;
    y32[m * ldy + n + 3] = acc.w;
  } else {
    uint2 packed;
    packed.x = pack_bf16x2(acc.x, acc.y);
    packed.y = pack_bf16x2(acc.z, acc.w);
    *reinterpret_cast<uint2*>(y + m * ldy + n) = packed;
  }
}

// Small-M plan: weight rows per tile (128, or 256 as two parts when M > 32) and the K split.  Cost model
// (bytes staged or moved, over the wave efficiency of the persistent grid): the weights once, the token
// rows once per weight tile (so 256-row tiles halve that term), and the fp32 partials written and read
// back when K is split.
struct SmallMPlan {
  int parts, splits;
};

static SmallMPlan small_m_plan(long long M, long long N, long long K, long long sms) {
  const long long nkb = (K + 63) / 64;
  const long long m_pad = M <= 32 ? 32 : 128;
  const long long max_s = M <= 32 ? 32 : 16;
  SmallMPlan best{1, 1};
  double best_cost = 1e30;
  for (int parts = 1; parts <= (M > 32 ? 2 : 1); ++parts) {
    const long long rows = 128 * parts;
    const long long f_tiles = (N + rows - 1) / rows;
    const double w_bytes = 2.0 * N * K, x_bytes = 2.0 * f_tiles * m_pad * K;
    for (long long s = 1; s <= max_s && s <= nkb; ++s) {
      const long long per = (nkb + s - 1) / s;
      const long long used = (nkb + per - 1) / per;   // slices actually non-empty
      if (used != s) continue;
      const long long tiles = f_tiles * ((M + 127) / 128) * s;
      const long long rounds = (tiles + sms - 1) / sms;
      const double wave = static_cast<double>(tiles) / static_cast<double>(rounds * sms);
      const double partial = s > 1 ? 2.0 * 4.0 * s * M * N : 0.0;
      const double cost = (w_bytes + x_bytes + partial) / wave;
      if (cost < best_cost * (1.0 - 1e-9)) {
        best_cost = cost;
        best = SmallMPlan{parts, static_cast<int>(s)};
      }
    }
  }
  return best;
}

int proj_small_m_splits(long long M, long long N, long long K, long long sms) {
  return small_m_plan(M, N, K, sms).splits;
}

size_t proj_workspace_bytes(long long M, long long N, long long K) {
  if (M <= 0 || N <= 0 || K <= 0 || M > 128) return 0;
  const int s = proj_small_m_splits(M, N, K, num_sms());
  return s > 1 ? static_cast<size_t>(s) * M * N * sizeof(float) : 0;
}

// y32 (fp32 output) replaces y when not null.  kx: the token operand's width when the weights are
// [W_hi | W_mid] (K = 2 kx, token k chunks wrap at kx); 0 otherwise.
template <int MA, int NB, int STAGES, int KC>
static int launch_proj_small_m(const void* x, const void* w, void* y, int M, int N, int K, long long ldy,
                               void* workspace, size_t ws_bytes, cudaStream_t stream, float* y32 = nullptr,
                               int kx = 0) {
  using L = SwapLayout<MA, NB, STAGES, KC>;
  auto kern = gemm_swap_kernel<ProjSwapSched, ProjSwapEpi, MA, NB, STAGES, KC>;
  static bool attr_done[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_done[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kSmemBytes);
    if (e != cudaSuccess) return cuda_status(e);
    attr_done[dev] = true;
  }
  int splits = proj_small_m_splits(M, N, K, num_sms());
  const size_t need = splits > 1 ? static_cast<size_t>(splits) * M * N * sizeof(float) : 0;
  if (splits > 1 && (!workspace || ws_bytes < need)) splits = 1;   // no workspace: one K slice
  CUtensorMap ta;
  TokenMaps tb;
  int rc = make_tmap_bf16_2d(&ta, w, K, N, K, kBK, 128);
  if (rc) return rc;
  rc = make_token_maps(&tb, x, M, kx > 0 ? kx : K);
  if (rc) return rc;
  ProjSwapSched::Params sp;
  sp.b_kwrap = kx > 0 ? kx / kBK : 0;
  sp.M = M;
  sp.N = N;
  sp.a_tile_rows = 128 * MA;
  sp.f_tiles = (N + sp.a_tile_rows - 1) / sp.a_tile_rows;
  sp.t_tiles = (M + NB - 1) / NB;
  sp.nb = NB;
  sp.splits = splits;
  sp.nkb_total = (K + kBK - 1) / kBK;
  sp.nkb_per = (sp.nkb_total + splits - 1) / splits;
  ProjSwapEpi::Params ep;
  ep.y = static_cast<__nv_bfloat16*>(y);
  ep.y32 = y32;
  ep.partial = splits > 1 ? static_cast<float*>(workspace) : nullptr;
  ep.ldy = ldy;
  ep.M = M;
  ep.N = N;
  ep.parts = MA;
  const int tiles = sp.f_tiles * sp.t_tiles * splits;
  const int grid = tiles < num_sms() ? tiles : num_sms();
  kern<<<grid, kGemmThreads, L::kSmemBytes, stream>>>(ta, tb, sp, ep);
  rc = cuda_status(cudaGetLastError());
  if (rc || splits == 1) return rc;
  const long long total = static_cast<long long>(M) * N;
  const bool vec4 = N % 4 == 0 && ldy % 4 == 0 && (y32 ? aligned16(y32) : (reinterpret_cast<uintptr_t>(y) & 7) == 0);
  if (vec4)
    proj_reduce4_kernel<<<static_cast<unsigned int>((total / 4 + 255) / 256), 256, 0, stream>>>(
        static_cast<const float4*>(workspace), static_cast<__nv_bfloat16*>(y), y32, ldy, M, N, splits);
  else
    proj_reduce_kernel<<<static_cast<unsigned int>((total + 255) / 256), 256, 0, stream>>>(
        static_cast<const float*>(workspace), static_cast<__nv_bfloat16*>(y), y32, ldy, M, N, splits);
  return cuda_status(cudaGetLastError());
}

// Output tile shape.  A persistent grid runs ceil(tiles / workers) rounds of tiles, so the tile
// count's remainder idles SMs in the last round (896 tiles of 128 x 256 on 148 SMs: 6.05 rounds, 7
// paid).  Candidates are scored by wave efficiency x column efficiency x the shape's intrinsic
// efficiency, measured on B200 with the L2 flushed: 256-row tiles on CTA pairs (half the B bytes per
// FLOP staged per SM) 1.00 at width 256 and 0.89 at 224; 128-row single-CTA tiles 0.85 / 0.81 / 0.78 at
// 256 / 224 / 192.  With fewer 128 x 256 tiles than SMs (weight-streaming shapes) the widest
// single-CTA width that still gives every SM a tile.
void pick_tile(long long M, long long N, long long sms, int* bn, int* pair) {
  const long long mb = (M + 127) / 128;
  *pair = 0;
  if (mb * ((N + 255) / 256) < sms) {
    *bn = (mb * ((N + 127) / 128) >= sms) ? 128 : 64;
    return;
  }
  struct Cand { int bn, pair; double eff; };
  static const Cand cands[5] = {{256, 1, 1.0}, {224, 1, 0.89}, {256, 0, 0.85}, {224, 0, 0.81}, {192, 0, 0.78}};
  double best = -1.0;
  for (const Cand& c : cands) {
    const long long rows = c.pair ? 256 : 128;
    const long long workers = c.pair ? sms / 2 : sms;
    const long long nb = (N + c.bn - 1) / c.bn;
    const long long tiles = ((M + rows - 1) / rows) * nb;
    const long long rounds = (tiles + workers - 1) / workers;
    const double wave = static_cast<double>(tiles) / static_cast<double>(rounds * workers);
    const double cols = static_cast<double>(N) / static_cast<double>(nb * c.bn);
    const double score = wave * cols * c.eff;
    if (score > best + 1e-9) {
      best = score;
      *bn = c.bn;
      *pair = c.pair;
    }
  }
}

int proj_bf16(const void* x, const void* w, void* y, long long M, long long N, long long K, long long ldy,
              int force_bn, int cta_pair, cudaStream_t stream, void* workspace, size_t ws_bytes) {
  if (M < 0 || N < 0 || K < 0) return KDB_ERR_INVALID_ARG;
  if (M == 0 || N == 0) return KDB_OK;
  if (!y || ldy < N) return KDB_ERR_INVALID_ARG;
  if (M > (1ll << 30) || N > (1ll << 30) || K > (1ll << 30)) return KDB_ERR_UNSUPPORTED;
  if (K == 0) {   // empty reduction: Y = 0 (X and W are empty and may be null)
    return cuda_status(cudaMemset2DAsync(y, static_cast<size_t>(ldy) * 2, 0, static_cast<size_t>(N) * 2,
                                         static_cast<size_t>(M), stream));
  }
  if (!x || !w) return KDB_ERR_INVALID_ARG;
  // TMA: 16-byte aligned base and row stride.
  if (K % 8 != 0 || !aligned16(x) || !aligned16(w)) return KDB_ERR_INVALID_ARG;

  int bn = force_bn;
  if (bn == 0 && cta_pair == 0) {
    // weight streaming: swapped operands with a K split; the narrower token block of M <= 32 leaves
    // room for 11 pipeline stages (more weight bytes in flight per SM)
    // two 64-wide k chunks per stage: 256 contiguous bytes of every weight row per request (7% faster
    // than one chunk at 16 x 7168 x 7168)
    if (M <= 32) return launch_proj_small_m<1, 32, 5, 2>(x, w, y, (int)M, (int)N, (int)K, ldy, workspace, ws_bytes, stream);
    if (M <= 128) {
      if (small_m_plan(M, N, K, num_sms()).parts == 2)
        return launch_proj_small_m<2, 128, 4, 1>(x, w, y, (int)M, (int)N, (int)K, ldy, workspace, ws_bytes, stream);
      return launch_proj_small_m<1, 128, 6, 1>(x, w, y, (int)M, (int)N, (int)K, ldy, workspace, ws_bytes, stream);
    }
    pick_tile(M, N, num_sms(), &bn, &cta_pair);
  }
  if (cta_pair > 0) {
    if (bn == 0) bn = 256;
    switch (bn) {
      case 256: return launch_proj_pair<256, 6>(x, w, y, (int)M, (int)N, (int)K, ldy, stream);
      case 224: return launch_proj_pair<224, 7>(x, w, y, (int)M, (int)N, (int)K, ldy, stream);
      case 192: return launch_proj_pair<192, 7>(x, w, y, (int)M, (int)N, (int)K, ldy, stream);
      default: return KDB_ERR_INVALID_ARG;
    }
  }
  switch (bn) {
    case 256: return launch_proj_cfg<256, 4>(x, w, y, (int)M, (int)N, (int)K, ldy, stream);
    case 224: return launch_proj_cfg<224, 5>(x, w, y, (int)M, (int)N, (int)K, ldy, stream);
    case 192: return launch_proj_cfg<192, 5>(x, w, y, (int)M, (int)N, (int)K, ldy, stream);
    case 128: return launch_proj_cfg<128, 6>(x, w, y, (int)M, (int)N, (int)K, ldy, stream);
    case 64: return launch_proj_cfg<64, 8>(x, w, y, (int)M, (int)N, (int)K, ldy, stream);
    default: return KDB_ERR_INVALID_ARG;
  }
}

// ---------------------------------------------------------------------------------------------------
// Projection with fp32 weights and fp32 output: the reference's router layer, whose precision rule is
// "fp32 weights and output (BF16 hi+lo pair with FP32 accumulation allowed)"
// (src/kdev/adapters/okc_problems/muse_bf16_proj.toml:371).  proj_split_f32 stores, once,
// w_split[n] = [bf16(W[n]) | bf16(W[n] - bf16(W[n]))] (n x 2k, lossless to 2^-16 of each weight: the
// probe-row rule's 0.1% holds), and Y = X · W_hiᵀ + X · W_midᵀ is one bf16 GEMM over K = 2k whose token
// operand repeats along K: the small-M swapped path wraps the token k chunk at k, the tiled path
// (router_approx) wraps A's k coordinate.
int proj_split_f32(const float* w, void* w_split, long long N, long long K, cudaStream_t stream) {
  if (N < 0 || K < 0) return KDB_ERR_INVALID_ARG;
  if (N == 0 || K == 0) return KDB_OK;
  if (!w || !w_split) return KDB_ERR_INVALID_ARG;
  if (N > (1ll << 24) || K > (1ll << 30) || N * K > (1ll << 40)) return KDB_ERR_UNSUPPORTED;
  return router_prepare(w, w_split, nullptr, static_cast<int>(N), static_cast<int>(K), stream);
}

size_t proj_f32w_workspace_bytes(long long M, long long N, long long K) {
  if (M <= 0 || N <= 0 || K <= 0 || M > 128) return 0;
  const int s = proj_small_m_splits(M, N, 2 * K, num_sms());
  return s > 1 ? static_cast<size_t>(s) * M * N * sizeof(float) : 0;
}

int proj_f32w(const void* x, const void* w_split, float* y, long long M, long long N, long long K, void* workspace,
              size_t ws_bytes, cudaStream_t stream) {
  if (M < 0 || N < 0 || K < 0) return KDB_ERR_INVALID_ARG;
  if (M == 0 || N == 0) return KDB_OK;
  if (!y) return KDB_ERR_INVALID_ARG;
  if (M > (1ll << 30) || N > (1ll << 30) || K > (1ll << 29) || M * N > (1ll << 31) / 4) return KDB_ERR_UNSUPPORTED;
  if (K == 0) return cuda_status(cudaMemsetAsync(y, 0, static_cast<size_t>(M) * N * sizeof(float), stream));
  if (!x || !w_split) return KDB_ERR_INVALID_ARG;
  if (K % kBK != 0) return KDB_ERR_UNSUPPORTED;   // the token operand wraps on whole 64-wide k chunks
  if (!aligned16(x) || !aligned16(w_split)) return KDB_ERR_INVALID_ARG;
  const int m = static_cast<int>(M), n = static_cast<int>(N), k2 = static_cast<int>(2 * K);
  if (M <= 32)
    return launch_proj_small_m<1, 32, 5, 2>(x, w_split, nullptr, m, n, k2, n, workspace, ws_bytes, stream, y, (int)K);
  if (M <= 128)
    return small_m_plan(M, N, 2 * K, num_sms()).parts == 2
               ? launch_proj_small_m<2, 128, 4, 1>(x, w_split, nullptr, m, n, k2, n, workspace, ws_bytes, stream, y, (int)K)
               : launch_proj_small_m<1, 128, 6, 1>(x, w_split, nullptr, m, n, k2, n, workspace, ws_bytes, stream, y, (int)K);
  return router_approx(x, w_split, y, m, static_cast<int>(K), n, stream);
}

}  // namespace kdb

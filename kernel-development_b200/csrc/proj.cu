// proj.cu — the bf16 dense projection Y[M, N] = X[M, K] · W[N, K]ᵀ (fp32 accumulate, bf16 out).
//
// Replaces the computation behind the `muse_bf16_proj` problem's kernel_fn(data, state)
// (kdev: src/kdev/adapters/okc.py:534-537, config src/kdev/adapters/okc_problems/muse_bf16_proj.toml).
// One persistent tcgen05 kernel (gemm_sm100.cuh); the tile width BN is picked per shape so that
// small-M, weight-streaming shapes still put a tile on every SM.
#include "gemm_pair_sm100.cuh"
#include "gemm_sm100.cuh"
#include "gemm_splitk_sm100.cuh"
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
// Small M (weight streaming, M <= 128): W as the MMA's M operand, X's rows as N, K split over the S CTAs
// of a thread-block cluster that reduce their partials through distributed shared memory inside the
// same launch (gemm_splitk_sm100.cuh).
//
// Plan: MA weight parts per output tile (1 or 2: 128 or 256 features) and the split S (cluster size,
// 1..8).  Each candidate is costed as the bytes one CTA streams (its slice of the tile's weight rows and
// of the token rows) times the number of rounds the grid needs, where a round holds as many clusters of S
// as the device can keep resident (queried once per device and configuration); the cost of staging and
// reading the partials is small against the weight stream and is ignored.
struct SmallMPlan {
  int parts, splits;
};

template <int MA, int NB, int STAGES, int KC>
static int splitk_capacity(int s) {
  // CTAs of this kernel, in clusters of s, resident at once on the current device (cached per device)
  using L = SplitKLayout<MA, NB, STAGES, KC>;
  static int cache[64][9] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64 || s < 1 || s > 8) return num_sms();
  if (cache[dev][s] > 0) return cache[dev][s];
  auto kern = gemm_splitk_kernel<MA, NB, STAGES, KC>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kSmemBytes) != cudaSuccess)
    return num_sms();
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(s * 64, 1, 1);
  cfg.blockDim = dim3(kGemmThreads, 1, 1);
  cfg.dynamicSmemBytes = L::kSmemBytes;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = s;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int clusters = 0;
  if (cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg) != cudaSuccess || clusters <= 0) {
    cudaGetLastError();
    clusters = num_sms() / s;
  }
  cache[dev][s] = clusters * s;
  return cache[dev][s];
}

template <int MA, int NB, int STAGES, int KC>
static void splitk_consider(long long M, long long N, long long K, SmallMPlan* best, double* best_cost) {
  const long long nkb = (K + 63) / 64;
  const long long f_tiles = (N + 128 * MA - 1) / (128 * MA);
  const long long t_tiles = (M + NB - 1) / NB;
  for (int s = 1; s <= 8 && s <= nkb; ++s) {
    const long long per = (nkb + s - 1) / s;
    if ((nkb + per - 1) / per != s) continue;   // every slice non-empty
    const long long ctas = f_tiles * t_tiles * s;
    const long long cap = splitk_capacity<MA, NB, STAGES, KC>(s);
    const long long rounds = (ctas + cap - 1) / cap;
    const double cta_bytes = 2.0 * per * 64 * (128.0 * MA + NB);
    const double cost = static_cast<double>(rounds) * cta_bytes * (1.0 + 0.02 * s);
    if (cost < *best_cost * (1.0 - 1e-9)) {
      *best_cost = cost;
      *best = SmallMPlan{MA, s};
    }
  }
}

static SmallMPlan small_m_plan(long long M, long long N, long long K) {
  SmallMPlan best{1, 1};
  double cost = 1e300;
  if (M <= 32) {
    splitk_consider<1, 32, 5, 2>(M, N, K, &best, &cost);
  } else {
    splitk_consider<1, 128, 6, 1>(M, N, K, &best, &cost);
    splitk_consider<2, 128, 4, 1>(M, N, K, &best, &cost);
  }
  return best;
}

size_t proj_workspace_bytes(long long, long long, long long) { return 0; }

// y32 (fp32 output) replaces y when not null.  kx: the token operand's width when the weights are
// [W_hi | W_mid] (K = 2 kx, token k chunks wrap at kx); 0 otherwise.
template <int MA, int NB, int STAGES, int KC>
static int launch_splitk(const void* x, const void* w, void* y, int M, int N, int K, long long ldy, int splits,
                         cudaStream_t stream, float* y32 = nullptr, int kx = 0) {
  using L = SplitKLayout<MA, NB, STAGES, KC>;
  auto kern = gemm_splitk_kernel<MA, NB, STAGES, KC>;
  static bool attr_done[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_done[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kSmemBytes);
    if (e != cudaSuccess) return cuda_status(e);
    attr_done[dev] = true;
  }
  CUtensorMap ta;
  TokenMaps tb;
  int rc = make_tmap_bf16_2d(&ta, w, K, N, K, kBK, 128);
  if (rc) return rc;
  rc = make_token_maps(&tb, x, M, kx > 0 ? kx : K);
  if (rc) return rc;
  SplitKParams p;
  p.M = M;
  p.N = N;
  p.K = K;
  p.f_tiles = (N + L::kFeat - 1) / L::kFeat;
  p.t_tiles = (M + NB - 1) / NB;
  p.nkb_total = (K + kBK - 1) / kBK;
  p.nkb_per = (p.nkb_total + splits - 1) / splits;
  p.splits = splits;
  p.b_kwrap = kx > 0 ? kx / kBK : 0;
  p.y = static_cast<__nv_bfloat16*>(y);
  p.y32 = y32;
  p.ldy = ldy;
  p.vec_ok = ldy % 4 == 0 && (y32 ? aligned16(y32) : (reinterpret_cast<uintptr_t>(y) & 7) == 0);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.f_tiles * p.t_tiles * splits, 1, 1);
  cfg.blockDim = dim3(kGemmThreads, 1, 1);
  cfg.dynamicSmemBytes = L::kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = splits;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cuda_status(cudaLaunchKernelEx(&cfg, kern, ta, tb, p));
}

// Small-M dispatch (M <= 128) for bf16 or fp32 (y32) output; kx as in launch_splitk.
static int proj_small_m(const void* x, const void* w, void* y, long long M, long long N, long long K, long long ldy,
                        cudaStream_t stream, float* y32 = nullptr, int kx = 0) {
  const SmallMPlan pl = small_m_plan(M, N, K);
  const int m = static_cast<int>(M), n = static_cast<int>(N), k = static_cast<int>(K);
  if (M <= 32) return launch_splitk<1, 32, 5, 2>(x, w, y, m, n, k, ldy, pl.splits, stream, y32, kx);
  if (pl.parts == 2) return launch_splitk<2, 128, 4, 1>(x, w, y, m, n, k, ldy, pl.splits, stream, y32, kx);
  return launch_splitk<1, 128, 6, 1>(x, w, y, m, n, k, ldy, pl.splits, stream, y32, kx);
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
    // weight streaming: swapped operands, K split over a cluster reduced in shared memory (one launch);
    // M <= 32 stages two 64-wide k chunks per stage: 256 contiguous bytes of every weight row per request
    (void)workspace;
    (void)ws_bytes;
    if (M <= 128) return proj_small_m(x, w, y, M, N, K, ldy, stream);
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

size_t proj_f32w_workspace_bytes(long long, long long, long long) { return 0; }

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
  (void)workspace;
  (void)ws_bytes;
  const int m = static_cast<int>(M), n = static_cast<int>(N);
  if (M <= 128) return proj_small_m(x, w_split, nullptr, M, N, 2 * K, N, stream, y, static_cast<int>(K));
  return router_approx(x, w_split, y, m, static_cast<int>(K), n, stream);
}

}  // namespace kdb

// moe_w4a16.cu — the NVFP4 w4a16 MoE layer of one expert-parallel rank: the reference's
// `muse_moe_w4a16` problem (src/kdev/adapters/okc_problems/muse_moe_w4a16.toml) that its H200 engines
// compute (okc-challenge/engines/sc_h.cu:189-467, x3_h.cu, x7_h.cu).
//
//   plan       the routing plan over all e_total experts (moe_plan); the local experts are ids
//              0..local-1, so their rows are the plan's first offsets[local] rows
//   tile prefix  ceil(count / 64) per local expert (w4_prefix_kernel)
//   gather     local token rows, converted to f16 (exact for activations inside f16's range)
//   gate_up    h = bf16(silu(x.W1^T * gs13) * (x.W3^T * gs13)), stored as f16 (gemm_fp4w_sm100.cuh)
//   down       y = (h.W2^T) * gs2 * pw1, kept in fp32 (pw1: the per-feature output weight, sc_h.cu:51, 346)
//   combine    out[t] = sum over t's local routes j (in route order) of y * tw[t, j] * rsqrt(mean(y^2) + 1e-8)
//
// Weights arrive already tiled by prepare() (a lossless reordering of NVFP4): for each expert, weight tile f
// (gate_up: the gate rows of 128 features and their up rows; down: 256 output features as two 128-row
// parts) and 64-element k chunk, one 9 KB block [part 0 codes | part 1 codes | part 0 scales | part 1
// scales], the chunks of a tile consecutive: blocks [local][f_tiles][K / 64][9216 B].
#include "gemm_fp4w_sm100.cuh"
#include "host_util.h"
#include "moe.h"

#include <algorithm>

namespace kdb {

constexpr int kW4Tokens = 64;   // tokens per tile (kFp4NB)

// Tiles (local expert g, weight tile f, 64-token tile tt), tt fastest.
struct Fp4Sched {
  struct Params {
    const int* offsets;      // [groups + 1] token-row offsets of the local experts
    const int* tile_start;   // [groups + 1] exclusive prefix of ceil(count / 64)
    int groups, f_tiles, nkb;
    int f_step;              // output features per weight tile (gate_up 128, down 256)
  };
  Params p;
  int total;
  __device__ explicit Fp4Sched(const Params& pp) : p(pp) { total = p.tile_start[p.groups]; }
  __device__ int num_tiles() const { return total * p.f_tiles; }
  __device__ Fp4Tile tile(int t) const {
    int lo = 0, hi = p.groups - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (__ldg(p.tile_start + mid) * p.f_tiles <= t) lo = mid;
      else hi = mid - 1;
    }
    const int g = lo;
    const int tstart = __ldg(p.tile_start + g), tcount = __ldg(p.tile_start + g + 1) - tstart;
    const int row_begin = __ldg(p.offsets + g), count = __ldg(p.offsets + g + 1) - row_begin;
    const int local = t - tstart * p.f_tiles;
    const int f = local / tcount, tt = local - f * tcount;
    Fp4Tile ti;
    ti.group = g;
    ti.f = f;
    ti.b_row = row_begin + tt * kW4Tokens;
    ti.n_valid = min(kW4Tokens, count - tt * kW4Tokens);
    ti.f0 = f * p.f_step;
    return ti;
  }
};

__device__ __forceinline__ float silu_w4(float g) { return __fdividef(g, 1.0f + __expf(-g)); }

// gate_up: accumulator lane r = gate feature f0 + r (part 0) and its up row (part 1); columns = the tile's
// tokens.  h is rounded to bf16 (the layer's intermediate precision) and stored as the f16 of that value
// (the down GEMM's token operand); for each token the warp's 32 lanes store 32 consecutive features.
struct SwigluFp4Epi {
  struct Params {
    __half* out;            // [rows, ld_out]
    const float* gscale;    // [local]: gs13 per expert
    int ld_out;
  };
  __device__ static void run(const Params& p, const Fp4Tile& ti, int r, uint32_t taddr) {
    const float gs = __ldg(p.gscale + ti.group);
    __half* col = p.out + ti.f0 + r;
#pragma unroll 1
    for (int c0 = 0; c0 < ti.n_valid; c0 += 32) {
      uint32_t g[32], u[32];
      tmem_ld_32x32b_x32(taddr + c0, g);
      tmem_ld_32x32b_x32(taddr + kFp4NB + c0, u);
      tmem_ld_wait();
      const int n = min(32, ti.n_valid - c0);
      __half* dst = col + static_cast<long long>(ti.b_row + c0) * p.ld_out;
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        if (i < n) {
          const float h = silu_w4(__uint_as_float(g[i]) * gs) * (__uint_as_float(u[i]) * gs);
          dst[static_cast<long long>(i) * p.ld_out] = __float2half_rn(__bfloat162float(__float2bfloat16_rn(h)));
        }
      }
    }
  }
};

// down: accumulator lane r of part a = output feature f0 + 128 a + r; columns = the tile's tokens; times gs2
// of the expert and pw1 of the feature, kept in fp32 (the engines' y, sc_h.cu:346; x3_h.cu:529-530).
struct ScaleFp4Epi {
  struct Params {
    float* out;             // [rows, ld_out]
    const float* gscale;    // [local]: gs2 per expert
    const float* pw1;       // [ld_out] per-feature output weight, or null (1)
    int ld_out;
  };
  __device__ static void run(const Params& p, const Fp4Tile& ti, int r, uint32_t taddr) {
    const float gs = __ldg(p.gscale + ti.group);
#pragma unroll 1
    for (int a = 0; a < 2; ++a) {
      const int feat = ti.f0 + a * 128 + r;
      const float mul = p.pw1 ? gs * __ldg(p.pw1 + feat) : gs;
      float* col = p.out + feat;
#pragma unroll 1
      for (int c0 = 0; c0 < ti.n_valid; c0 += 32) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(taddr + a * kFp4NB + c0, v);
        tmem_ld_wait();
        const int n = min(32, ti.n_valid - c0);
        float* dst = col + static_cast<long long>(ti.b_row + c0) * p.ld_out;
#pragma unroll
        for (int i = 0; i < 32; ++i)
          if (i < n) dst[static_cast<long long>(i) * p.ld_out] = __uint_as_float(v[i]) * mul;
      }
    }
  }
};

// tile_start[g] = sum_{g' < g} ceil(count_g' / 64) for the first L experts of the plan (L <= 1024).
__global__ void __launch_bounds__(32) w4_prefix_kernel(const int* __restrict__ offsets, int L, int* __restrict__ tile_start) {
  if (threadIdx.x != 0) return;
  int run = 0;
  for (int g = 0; g < L; ++g) {
    tile_start[g] = run;
    run += (offsets[g + 1] - offsets[g] + kW4Tokens - 1) / kW4Tokens;
  }
  tile_start[L] = run;
}

// out[r] = f16(x[perm_token[r]]) for the local rows r < offsets[L] (one warp per row, 16-byte vectors).
__global__ void __launch_bounds__(256)
    w4_gather_f16_kernel(const __nv_bfloat16* __restrict__ x, const int* __restrict__ perm_token,
                         const int* __restrict__ local_rows, __half* __restrict__ out, int R, int H, int T) {
  const int rows = min(R, __ldg(local_rows));
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  const int nwarps = (gridDim.x * blockDim.x) >> 5;
  for (int r = warp; r < rows; r += nwarps) {
    const int tok = __ldg(perm_token + r);
    if (tok < 0 || tok >= T) {
      if (lane == 0) report(KDB_ERR_DEVICE_BOUNDS, 0x121);
      continue;
    }
    const uint4* src = reinterpret_cast<const uint4*>(x + static_cast<long long>(tok) * H);
    uint4* dst = reinterpret_cast<uint4*>(out + static_cast<long long>(r) * H);
    for (int v = lane; v < H / 8; v += 32) {
      const uint4 u = __ldg(src + v);
      const __nv_bfloat162* b = reinterpret_cast<const __nv_bfloat162*>(&u);
      uint4 o;
      __half2* h = reinterpret_cast<__half2*>(&o);
#pragma unroll
      for (int q = 0; q < 4; ++q) h[q] = __float22half2_rn(__bfloat1622float2(b[q]));
      dst[v] = o;
    }
  }
}

// One CTA per token: the post-expert RMS normalisation and the weighted sum over the token's local routes
// in route order (deterministic).  H <= 256 * kW4CombineMax.
constexpr int kW4CombineMax = 32;

__global__ void __launch_bounds__(256)
    w4_combine_kernel(const float* __restrict__ rows, const int* __restrict__ ids, const float* __restrict__ tw,
                      const int* __restrict__ slot_pos, int local, __nv_bfloat16* __restrict__ out, int H, int k) {
  __shared__ float red[8];
  const int t = blockIdx.x, tid = threadIdx.x;
  const int per = (H + 255) / 256;
  float acc[kW4CombineMax];
#pragma unroll
  for (int i = 0; i < kW4CombineMax; ++i) acc[i] = 0.f;
  for (int j = 0; j < k; ++j) {
    const int e = __ldg(ids + static_cast<long long>(t) * k + j);
    if (e < 0 || e >= local) continue;   // a route to another rank's expert
    const int r = __ldg(slot_pos + static_cast<long long>(t) * k + j);
    const float* y = rows + static_cast<long long>(r) * H;
    float v[kW4CombineMax];
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < kW4CombineMax; ++i) {
      const int h = tid + 256 * i;
      v[i] = (i < per && h < H) ? y[h] : 0.f;
      ss = fmaf(v[i], v[i], ss);
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
    if ((tid & 31) == 0) red[tid >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) tot += red[w];
    __syncthreads();
    const float wj = __ldg(tw + static_cast<long long>(t) * k + j);
    const float rr = rsqrtf(tot / static_cast<float>(H) + 1e-8f);
#pragma unroll
    for (int i = 0; i < kW4CombineMax; ++i) acc[i] = fmaf(v[i] * wj, rr, acc[i]);   // y * tw * rsqrt, as x3_h.cu:654
  }
#pragma unroll
  for (int i = 0; i < kW4CombineMax; ++i) {
    const int h = tid + 256 * i;
    if (i < per && h < H) out[static_cast<long long>(t) * H + h] = __float2bfloat16_rn(acc[i]);
  }
}

// ---------------------------------------------------------------------------------------------------
struct W4Carve {
  size_t chunk_counts, chunk_base, mtile, perm_token, perm_w, counts, offsets, perm_slot, slot_pos, tile_start,
      xf16, hbuf, yrows, total;
};

static W4Carve w4_carve(long long T, long long H, long long I, long long L, long long E, long long k) {
  auto up = [](size_t v) { return (v + 255) / 256 * 256; };
  const size_t C = static_cast<size_t>((T + 255) / 256), R = static_cast<size_t>(T * k);
  W4Carve c;
  size_t o = 0;
  c.chunk_counts = o;  o += up(sizeof(int) * C * E);
  c.chunk_base = o;    o += up(sizeof(int) * C * E);
  c.mtile = o;         o += up(sizeof(int) * (E + 1));
  c.perm_token = o;    o += up(sizeof(int) * R);
  c.perm_w = o;        o += up(sizeof(float) * R);
  c.counts = o;        o += up(sizeof(int) * E);
  c.offsets = o;       o += up(sizeof(int) * (E + 1));
  c.perm_slot = o;     o += up(sizeof(int) * R);
  c.slot_pos = o;      o += up(sizeof(int) * R);
  c.tile_start = o;    o += up(sizeof(int) * (L + 1));
  c.xf16 = o;          o += up(2 * R * H);
  c.hbuf = o;          o += up(2 * R * I);
  c.yrows = o;         o += up(4 * R * H);   // fp32 y rows
  c.total = o;
  return c;
}

static int w4_check(long long T, long long H, long long I, long long L, long long E, long long k) {
  if (T < 0 || H <= 0 || I <= 0 || L <= 0 || E <= 0 || k <= 0) return KDB_ERR_INVALID_ARG;
  if (L > E || E > 1024 || k > E) return KDB_ERR_INVALID_ARG;
  if (H % 256 != 0 || I % 128 != 0) return KDB_ERR_UNSUPPORTED;
  if (H > 256 * kW4CombineMax || T * k > (1ll << 24) || T * k * H > (1ll << 34)) return KDB_ERR_UNSUPPORTED;
  return KDB_OK;
}

size_t moe_w4a16_workspace_bytes(long long T, long long H, long long I, long long L, long long E, long long k) {
  if (w4_check(T, H, I, L, E, k)) return 0;
  return w4_carve(T, H, I, L, E, k).total;
}

template <class Epi>
static int launch_fp4w(const void* tokens, int rows, int K, const uint8_t* blocks, const Fp4Sched::Params& sp,
                       const typename Epi::Params& ep, cudaStream_t s) {
  constexpr int RS = 6, CS = 4;   // 6 raw stages of 2 chunks (108 KB of NVFP4 + their 96 KB of tokens), 4 TMEM stages
  using L = Fp4Layout<RS, CS>;
  auto kern = gemm_fp4w_kernel<Fp4Sched, Epi, RS, CS>;
  static bool done[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return KDB_ERR_NO_DEVICE;
  if (!done[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kSmemBytes);
    if (e != cudaSuccess) return cuda_status(e);
    done[dev] = true;
  }
  TokenMaps tb;
  int rc = make_token_maps(&tb, tokens, rows, K);
  if (rc) return rc;
  kern<<<num_sms(), kFp4Threads, L::kSmemBytes, s>>>(tb, blocks, sp, ep);
  return cuda_status(cudaGetLastError());
}

int moe_w4a16_forward(const void* x, const int* ids, const float* tw, const void* w13_blocks, const float* w13_gscale,
                      const void* w2_blocks, const float* w2_gscale, const float* pw1,
                      void* y, long long T, long long H, long long I, long long L, long long E, long long k,
                      void* workspace, size_t workspace_bytes, cudaStream_t s) {
  int rc = w4_check(T, H, I, L, E, k);
  if (rc) return rc;
  if (T == 0) return KDB_OK;
  if (!x || !ids || !tw || !w13_blocks || !w13_gscale || !w2_blocks || !w2_gscale || !y) return KDB_ERR_INVALID_ARG;
  if (!aligned16(x) || !aligned16(w13_blocks) || !aligned16(w2_blocks) || !aligned16(y)) return KDB_ERR_INVALID_ARG;
  const W4Carve c = w4_carve(T, H, I, L, E, k);
  if (!workspace || workspace_bytes < c.total) return KDB_ERR_WORKSPACE;
  if ((reinterpret_cast<uintptr_t>(workspace) & 255) != 0) return KDB_ERR_INVALID_ARG;
  char* ws = static_cast<char*>(workspace);
  auto Ip = [&](size_t off) { return reinterpret_cast<int*>(ws + off); };
  const int Ti = static_cast<int>(T), Hi = static_cast<int>(H), Ii = static_cast<int>(I), Li = static_cast<int>(L);
  const int Ei = static_cast<int>(E), ki = static_cast<int>(k), R = Ti * ki;

  rc = moe_plan(ids, tw, Ti, Ei, ki, Ip(c.chunk_counts), Ip(c.chunk_base), Ip(c.counts), Ip(c.offsets), Ip(c.mtile),
                Ip(c.perm_slot), Ip(c.slot_pos), Ip(c.perm_token), reinterpret_cast<float*>(ws + c.perm_w), s);
  if (rc) return rc;
  w4_prefix_kernel<<<1, 32, 0, s>>>(Ip(c.offsets), Li, Ip(c.tile_start));
  rc = cuda_status(cudaGetLastError());
  if (rc) return rc;
  {
    const int blocks = std::min(R, 4 * num_sms() * 8) / 8 + 1;
    w4_gather_f16_kernel<<<blocks, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(x), Ip(c.perm_token),
                                                Ip(c.offsets) + Li, reinterpret_cast<__half*>(ws + c.xf16), R, Hi, Ti);
    rc = cuda_status(cudaGetLastError());
    if (rc) return rc;
  }
  {
    Fp4Sched::Params sp;
    sp.offsets = Ip(c.offsets);
    sp.tile_start = Ip(c.tile_start);
    sp.groups = Li;
    sp.f_tiles = Ii / 128;
    sp.nkb = Hi / kBK;
    sp.f_step = 128;
    SwigluFp4Epi::Params ep;
    ep.out = reinterpret_cast<__half*>(ws + c.hbuf);
    ep.gscale = w13_gscale;
    ep.ld_out = Ii;
    rc = launch_fp4w<SwigluFp4Epi>(ws + c.xf16, R, Hi, static_cast<const uint8_t*>(w13_blocks), sp, ep, s);
    if (rc) return rc;
  }
  {
    Fp4Sched::Params sp;
    sp.offsets = Ip(c.offsets);
    sp.tile_start = Ip(c.tile_start);
    sp.groups = Li;
    sp.f_tiles = Hi / 256;
    sp.nkb = Ii / kBK;
    sp.f_step = 256;
    ScaleFp4Epi::Params ep;
    ep.out = reinterpret_cast<float*>(ws + c.yrows);
    ep.gscale = w2_gscale;
    ep.pw1 = pw1;
    ep.ld_out = Hi;
    rc = launch_fp4w<ScaleFp4Epi>(ws + c.hbuf, R, Ii, static_cast<const uint8_t*>(w2_blocks), sp, ep, s);
    if (rc) return rc;
  }
  w4_combine_kernel<<<Ti, 256, 0, s>>>(reinterpret_cast<const float*>(ws + c.yrows), ids, tw, Ip(c.slot_pos),
                                       Li, static_cast<__nv_bfloat16*>(y), Hi, ki);
  return cuda_status(cudaGetLastError());
}

}  // namespace kdb

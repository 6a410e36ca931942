// moe_router_fast.cu — bit-exact top-k routing at tensor-core speed.
//
// The routing decision must equal the one taken on the fixed-order fp64 logits (moe_route.cu), but
// computing every logit that way costs T*E*H fp64 FMAs (15 G for the 8192-token, 256-expert, 7168-wide
// prefill layer).  Instead:
//
//  1. approx = x · [W_hi | W_mid]ᵀ on the tensor cores (one tcgen05 GEMM, K = 2H with A's k coordinate
//     wrapping at H), where W_hi = bf16(W) and W_mid = bf16(W - W_hi) are prepared once.
//  2. Error bound: |approx - dot| <= delta_t for every expert of token t, with
//       delta_t = (2^-16 + 1.01 * 17 * 2^-23 * ceil(2H / 16) + 2^-20) * ||x_t||_2 * max_e ||W_e||_2 * 1.01
//                 + 2^-20 * (1 + max |bias|).
//     2^-16 bounds the dropped W - W_hi - W_mid (two bf16 roundings of 8 significant bits); each of the
//     ceil(2H/16) MMA steps adds 16 exact bf16 x bf16 products to the fp32 accumulator, and the bound
//     allows 17 units of 2^-23 of the running magnitude per step (every addend truncated by a full unit
//     when aligned, plus the result) — a worst case far above the usual one-rounding behaviour; the
//     magnitude of every partial sum is at most sum_h |x_h| |W_eh| (1 + 2^-7) <= ||x_t|| ||W_e|| (1.01).
//     The 2^-20 terms cover the fp32 rounding of the dot product and of the bias addition.
//  3. Candidates: every expert whose approx logit is >= (k-th largest approx) - 2 delta_t.  Any expert
//     outside that set has an exact logit strictly below the exact logits of the k experts with the
//     largest approx values, so the exact top-k lies inside the set.  Tokens with more than kCandMax
//     (64) candidates take every expert; the prefill configuration averages 15.6 and peaks near 30.
//  4. The candidates' logits are recomputed in the fixed fp64 order (bit-identical to the full router
//     and the oracle) and the top-k and renormalised weights are taken from them exactly as moe_topk_kernel
//     does, so ids and weights are bit-identical to the full path.
#include "gemm_sm100.cuh"
#include "host_util.h"
#include "moe.h"

namespace kdb {

constexpr int kCandMax = 64;

// One warp per expert row: wcat[e] = [bf16(w) | bf16(w - bf16(w))], norms[e] >= ||w_e||_2.
__global__ void __launch_bounds__(256)
    router_split_kernel(const float* __restrict__ w, __nv_bfloat16* __restrict__ wcat, float* __restrict__ norms,
                        int E, int H) {
  const int e = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (e >= E) return;
  double ss = 0.0;
  for (int h = lane; h < H; h += 32) {
    const float v = w[static_cast<long long>(e) * H + h];
    const __nv_bfloat16 hi = __float2bfloat16_rn(v);
    const float r = v - __bfloat162float(hi);   // exact: hi holds v's leading bits
    wcat[static_cast<long long>(e) * 2 * H + h] = hi;
    wcat[static_cast<long long>(e) * 2 * H + H + h] = __float2bfloat16_rn(r);
    ss = fma(static_cast<double>(v), static_cast<double>(v), ss);
  }
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
  if (lane == 0 && norms) norms[e] = __double2float_ru(sqrt(ss) * (1.0 + 1e-12));
}

// fp32 output tile of the approx-logit GEMM: out[row, col] = accumulator (row < M, col < N).
template <int BN>
struct F32Epi {
  struct Params {
    float* out;
    int ld, M, N;
  };
  __device__ static void run(const Params& p, const ProjTile& ti, int r, uint32_t taddr) {
    const int row = ti.m0 + r;
    float* orow = p.out + static_cast<long long>(row) * p.ld;
#pragma unroll 1
    for (int c = 0; c < BN / 32; ++c) {
      uint32_t v[32];
      tmem_ld_32x32b_x32(taddr + c * 32, v);
      tmem_ld_wait();
      if (row >= p.M) continue;
      const int col0 = ti.n0 + c * 32;
      for (int j = 0; j < 32 && col0 + j < p.N; ++j) orow[col0 + j] = __uint_as_float(v[j]);
    }
  }
};

// One warp per token: the error bound, the k-th largest approx logit, and the candidate list.
template <int PER_LANE>
__global__ void __launch_bounds__(256)
    router_candidates_kernel(const float* __restrict__ approx, const __nv_bfloat16* __restrict__ x,
                             const float* __restrict__ bias, const float* __restrict__ norms, float gamma, int T,
                             int H, int E, int k, int* __restrict__ cand, int* __restrict__ ncand) {
  const int t = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (t >= T) return;
  // ||x_t||_2 (fp64 sum of squares of bf16 values, rounded up)
  double ss = 0.0;
  const uint4* xr = reinterpret_cast<const uint4*>(x + static_cast<long long>(t) * H);
  for (int v = lane; v < H / 8; v += 32) {
    const uint4 u = __ldg(xr + v);
    const __nv_bfloat162* b = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float2 f = __bfloat1622float2(b[q]);
      ss = fma(static_cast<double>(f.x), static_cast<double>(f.x), ss);
      ss = fma(static_cast<double>(f.y), static_cast<double>(f.y), ss);
    }
  }
  float wmax = 0.f, bmax = 0.f;
  for (int e = lane; e < E; e += 32) {
    wmax = fmaxf(wmax, norms[e]);
    if (bias) bmax = fmaxf(bmax, fabsf(bias[e]));
  }
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) {
    ss += __shfl_xor_sync(0xffffffffu, ss, off);
    wmax = fmaxf(wmax, __shfl_xor_sync(0xffffffffu, wmax, off));
    bmax = fmaxf(bmax, __shfl_xor_sync(0xffffffffu, bmax, off));
  }
  const double xn = sqrt(ss) * (1.0 + 1e-12);
  const float delta = static_cast<float>(static_cast<double>(gamma) * xn * static_cast<double>(wmax) * 1.01 +
                                         9.5367431640625e-07 * (1.0 + static_cast<double>(bmax)));
  float v[PER_LANE];
#pragma unroll
  for (int i = 0; i < PER_LANE; ++i) {
    const int e = i * 32 + lane;
    v[i] = (e < E) ? approx[static_cast<long long>(t) * E + e] + (bias ? bias[e] : 0.f) : -INFINITY;
  }
  // k-th largest approx value: k rounds of warp max (removing one occurrence per round)
  unsigned int taken = 0;
  float vk = -INFINITY;
  for (int j = 0; j < k; ++j) {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < PER_LANE; ++i) {
      const int e = i * 32 + lane;
      if (e < E && !(taken & (1u << i)) && (bi == 0x7fffffff || v[i] > bv)) {
        bv = v[i];
        bi = e;
      }
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
      if (oi != 0x7fffffff && (bi == 0x7fffffff || ov > bv || (ov == bv && oi < bi))) {
        bv = ov;
        bi = oi;
      }
    }
    if (bi != 0x7fffffff && (bi & 31) == lane) taken |= 1u << (bi >> 5);
    vk = bv;
  }
  const float thr = vk - 2.0f * delta;
  // candidates in ascending expert order
  int count = 0;
  int* out = cand + static_cast<long long>(t) * kCandMax;
#pragma unroll
  for (int i = 0; i < PER_LANE; ++i) {
    const int e = i * 32 + lane;
    const bool pick = e < E && !(v[i] < thr);   // NaN approx values are kept as candidates
    const unsigned int m = __ballot_sync(0xffffffffu, pick);
    const int pos = count + __popc(m & ((1u << lane) - 1u));
    if (pick && pos < kCandMax) out[pos] = e;
    count += __popc(m);
  }
  if (lane == 0) ncand[t] = count <= kCandMax ? count : -1;
}

// Fixed-order fp64 logit of expert rows we[0..NC) for token row xt, all NC accumulated together so
// their loads and fma chains overlap; lane l takes h = 256*b + 8*l + j (the fixed order).
template <int NC>
__device__ __forceinline__ void exact_logits(const __nv_bfloat16* __restrict__ xt, const float* const (&we)[NC],
                                             int H, int lane, double (&acc)[NC]) {
#pragma unroll
  for (int q = 0; q < NC; ++q) acc[q] = 0.0;
  for (int base = 0; base < H; base += 256) {
    const int h = base + 8 * lane;
    if (h < H) {   // H % 8 == 0: a lane's 8 elements are all inside or all outside
      const uint4 u = __ldg(reinterpret_cast<const uint4*>(xt + h));
      const __nv_bfloat162* b = reinterpret_cast<const __nv_bfloat162*>(&u);
      double xv[8];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 f = __bfloat1622float2(b[q]);
        xv[2 * q] = f.x;
        xv[2 * q + 1] = f.y;
      }
      float4 w0[NC], w1[NC];
#pragma unroll
      for (int q = 0; q < NC; ++q) {
        w0[q] = __ldg(reinterpret_cast<const float4*>(we[q] + h));
        w1[q] = __ldg(reinterpret_cast<const float4*>(we[q] + h + 4));
      }
#pragma unroll
      for (int q = 0; q < NC; ++q) {
        acc[q] = fma(xv[0], static_cast<double>(w0[q].x), acc[q]);
        acc[q] = fma(xv[1], static_cast<double>(w0[q].y), acc[q]);
        acc[q] = fma(xv[2], static_cast<double>(w0[q].z), acc[q]);
        acc[q] = fma(xv[3], static_cast<double>(w0[q].w), acc[q]);
        acc[q] = fma(xv[4], static_cast<double>(w1[q].x), acc[q]);
        acc[q] = fma(xv[5], static_cast<double>(w1[q].y), acc[q]);
        acc[q] = fma(xv[6], static_cast<double>(w1[q].z), acc[q]);
        acc[q] = fma(xv[7], static_cast<double>(w1[q].w), acc[q]);
      }
    }
  }
#pragma unroll
  for (int q = 0; q < NC; ++q) {
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) acc[q] = acc[q] + __shfl_xor_sync(0xffffffffu, acc[q], off);
  }
}

constexpr int kExactWarps = 4;
constexpr int kExactGroup = 4;   // candidates one warp accumulates together

// NC candidates c0, c0 + kExactWarps, ... of one token: fixed-order logits into vals/ids.
template <int NC>
__device__ __forceinline__ void exact_pass(const __nv_bfloat16* __restrict__ xt, const float* __restrict__ wr,
                                           const float* __restrict__ bias, const int* __restrict__ ct, bool all,
                                           int c0, int H, int lane, float* vals, int* ids) {
  const float* we[NC];
  int es[NC];
#pragma unroll
  for (int q = 0; q < NC; ++q) {
    const int c = c0 + q * kExactWarps;
    es[q] = all ? c : ct[c];
    we[q] = wr + static_cast<long long>(es[q]) * H;
  }
  double acc[NC];
  exact_logits<NC>(xt, we, H, lane, acc);
  if (lane == 0) {
#pragma unroll
    for (int q = 0; q < NC; ++q) {
      float l = __double2float_rn(acc[q]);
      if (bias) l = __fadd_rn(l, bias[es[q]]);
      vals[c0 + q * kExactWarps] = l;
      ids[c0 + q * kExactWarps] = es[q];
    }
  }
}

// One CTA per token: its warps compute the fixed-order fp64 logits of the token's candidates (all
// experts when ncand < 0), then warp 0 takes the top-k and weights exactly as moe_topk_kernel does.
__global__ void __launch_bounds__(kExactWarps * 32)
    router_exact_topk_kernel(const __nv_bfloat16* __restrict__ x, const float* __restrict__ wr,
                             const float* __restrict__ bias, const int* __restrict__ cand,
                             const int* __restrict__ ncand, int T, int H, int E, int k,
                             float* __restrict__ topk_w, int* __restrict__ topk_ids) {
  extern __shared__ float sm[];
  const int t = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int slots = E > kCandMax ? E : kCandMax;
  float* vals = sm;
  int* ids = reinterpret_cast<int*>(sm + slots);
  int n = ncand[t];
  const bool all = n < 0;
  if (all) n = E;
  const __nv_bfloat16* xt = x + static_cast<long long>(t) * H;
  const int* ct = cand + static_cast<long long>(t) * kCandMax;
  // warp w takes candidates w, w + W, w + 2W, ... (W warps), up to kExactGroup of them per pass
  for (int c0 = warp; c0 < n; c0 += kExactWarps * kExactGroup) {
    const int left = (n - c0 + kExactWarps - 1) / kExactWarps;   // this warp's remaining candidates
    const int nc = left < kExactGroup ? left : kExactGroup;
    if (nc >= 4) exact_pass<4>(xt, wr, bias, ct, all, c0, H, lane, vals, ids);
    else if (nc == 3) exact_pass<3>(xt, wr, bias, ct, all, c0, H, lane, vals, ids);
    else if (nc == 2) exact_pass<2>(xt, wr, bias, ct, all, c0, H, lane, vals, ids);
    else exact_pass<1>(xt, wr, bias, ct, all, c0, H, lane, vals, ids);
  }
  __syncthreads();
  if (warp != 0) return;
  // top-k over (vals, ids)[0, n): value desc, expert asc
  float vmax = 0.f, my_val = 0.f;
  int my_id = -1;
  for (int j = 0; j < k; ++j) {
    float bv = -INFINITY;
    int bi = 0x7fffffff, bc = -1;
    for (int c = lane; c < n; c += 32) {
      const int e = ids[c];
      if (e < 0) continue;   // taken
      const float vv = vals[c];
      if (bi == 0x7fffffff || vv > bv || (vv == bv && e < bi)) {
        bv = vv;
        bi = e;
        bc = c;
      }
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
      const int oc = __shfl_xor_sync(0xffffffffu, bc, off);
      if (oi != 0x7fffffff && (bi == 0x7fffffff || ov > bv || (ov == bv && oi < bi))) {
        bv = ov;
        bi = oi;
        bc = oc;
      }
    }
    __syncwarp();
    if (lane == 0 && bc >= 0) ids[bc] = -1;
    __syncwarp();
    if (j == 0) vmax = bv;
    if (lane == j) {
      my_val = bv;
      my_id = bi;
    }
  }
  const float p = (lane < k) ? __expf(my_val - vmax) : 0.f;
  float s = p;
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
  if (lane < k) {
    topk_ids[static_cast<long long>(t) * k + lane] = my_id;
    topk_w[static_cast<long long>(t) * k + lane] = p / s;
  }
}

// ------------------------------------------------------------------------------------------------
size_t router_fast_scratch_bytes(long long T, long long E) {
  auto up = [](size_t v) { return (v + 255) / 256 * 256; };
  return up(sizeof(float) * T * E) + up(sizeof(int) * T * kCandMax) + up(sizeof(int) * T);
}

int router_prepare(const float* wr, void* wcat, float* norms, int E, int H, cudaStream_t s) {
  if (E <= 0) return KDB_OK;
  router_split_kernel<<<(E * 32 + 255) / 256, 256, 0, s>>>(wr, static_cast<__nv_bfloat16*>(wcat), norms, E, H);
  return cuda_status(cudaGetLastError());
}

static float router_gamma(int H) {
  const double steps = (2.0 * H + 15) / 16;
  return static_cast<float>(1.52587890625e-05 + 1.01 * 17.0 * 1.1920928955078125e-07 * steps +
                            9.5367431640625e-07);
}

template <int BN>
static int launch_router_gemm(const void* x, const void* wcat, float* approx, int T, int H, int E, cudaStream_t s) {
  constexpr int BM = 128, STAGES = (BN == 128) ? 6 : 8;
  using L = GemmLayout<BM, BN, STAGES>;
  using Sched = ProjSched<BM, BN>;
  using Epi = F32Epi<BN>;
  auto kern = gemm_tn_kernel<Sched, Epi, BM, BN, STAGES>;
  static bool done[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return KDB_ERR_NO_DEVICE;
  if (!done[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kSmemBytes);
    if (e != cudaSuccess) return cuda_status(e);
    done[dev] = true;
  }
  CUtensorMap ta, tb;
  int rc = make_tmap_bf16_2d(&ta, x, H, T, H, kBK, BM);
  if (rc) return rc;
  rc = make_tmap_bf16_2d(&tb, wcat, 2 * H, E, 2 * H, kBK, BN);
  if (rc) return rc;
  typename Sched::Params sp;
  sp.M = T;
  sp.N = E;
  sp.K = 2 * H;
  sp.num_m = (T + BM - 1) / BM;
  sp.num_n = (E + BN - 1) / BN;
  sp.group_m = sp.num_m;
  sp.kwrap = H / kBK;
  typename Epi::Params ep;
  ep.out = approx;
  ep.ld = E;
  ep.M = T;
  ep.N = E;
  const int tiles = sp.num_m * sp.num_n;
  const int grid = tiles < num_sms() ? tiles : num_sms();
  kern<<<grid, kGemmThreads, L::kSmemBytes, s>>>(ta, tb, sp, ep);
  return cuda_status(cudaGetLastError());
}

int router_approx(const void* x, const void* wcat, float* approx, int T, int H, int E, cudaStream_t s) {
  if (T <= 0) return KDB_OK;
  if (H % kBK != 0) return KDB_ERR_UNSUPPORTED;
  return E <= 64 ? launch_router_gemm<64>(x, wcat, approx, T, H, E, s)
                 : launch_router_gemm<128>(x, wcat, approx, T, H, E, s);
}

int moe_route_fast(const void* x, const float* wr, const float* bias, const void* wcat, const float* norms,
                   float* topk_w, int* topk_ids, int T, int H, int E, int k, void* scratch, cudaStream_t s) {
  if (T <= 0) return KDB_OK;
  auto up = [](size_t v) { return (v + 255) / 256 * 256; };
  char* ws = static_cast<char*>(scratch);
  float* approx = reinterpret_cast<float*>(ws);
  int* cand = reinterpret_cast<int*>(ws + up(sizeof(float) * T * E));
  int* ncand = reinterpret_cast<int*>(ws + up(sizeof(float) * T * E) + up(sizeof(int) * T * kCandMax));
  int rc = router_approx(x, wcat, approx, T, H, E, s);
  if (rc) return rc;
  const int blocks = (T * 32 + 255) / 256;
  const float gamma = router_gamma(H);
  const auto* xb = static_cast<const __nv_bfloat16*>(x);
  const int per_lane = (E + 31) / 32;
  if (per_lane <= 2) router_candidates_kernel<2><<<blocks, 256, 0, s>>>(approx, xb, bias, norms, gamma, T, H, E, k, cand, ncand);
  else if (per_lane <= 4) router_candidates_kernel<4><<<blocks, 256, 0, s>>>(approx, xb, bias, norms, gamma, T, H, E, k, cand, ncand);
  else if (per_lane <= 8) router_candidates_kernel<8><<<blocks, 256, 0, s>>>(approx, xb, bias, norms, gamma, T, H, E, k, cand, ncand);
  else router_candidates_kernel<32><<<blocks, 256, 0, s>>>(approx, xb, bias, norms, gamma, T, H, E, k, cand, ncand);
  rc = cuda_status(cudaGetLastError());
  if (rc) return rc;
  const int slots = E > kCandMax ? E : kCandMax;
  const size_t smem = static_cast<size_t>(2) * slots * sizeof(float);   // <= 8 KB (E <= 1024)
  router_exact_topk_kernel<<<T, kExactWarps * 32, smem, s>>>(xb, wr, bias, cand, ncand, T, H, E, k, topk_w, topk_ids);
  return cuda_status(cudaGetLastError());
}

}  // namespace kdb

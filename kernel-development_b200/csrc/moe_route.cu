// moe_route.cu — MoE routing on the GPU: router logits, top-k with renormalised weights, and the
// stable (expert, token) permutation plan the grouped GEMMs consume.
//
// Reference structure: the `up_moe` plan stage (okc-challenge/engines/x3_h.cu:346-385) builds
// per-expert token masks, counts them with popc and scans them with __shfl_up_sync into per-expert
// base rows, on the device, with no host sync.  Here the same plan is produced for any T and E by
// three small kernels (count per chunk, scan, scatter); positions are stable: grouped by expert,
// tokens ascending within an expert, so the result is deterministic and matches the CPU oracle
// exactly.
//
// Router logits use a fixed fp64 summation order so they are bit-identical to the oracle: h is cut
// into blocks of 256; lane l of a warp accumulates, block by block, h = 256*b + 8*l + j for
// j = 0..7 with fma; then the 32 partials are combined by an xor butterfly with offsets 16, 8, 4,
// 2, 1; the fp64 sum is rounded once to fp32, then the optional fp32 bias is added.
#include "moe.h"
#include "host_util.h"
#include "sm100_common.cuh"

namespace kdb {

constexpr int kRouteTokTile = 16;   // tokens per CTA
constexpr int kRouteExpPerWarp = 2; // experts per warp
constexpr int kRouteWarps = 8;      // -> 16 experts per CTA
constexpr int kRouteHChunk = 256;   // hidden elements staged per pass: one block of the fixed order

__global__ void __launch_bounds__(kRouteWarps * 32)
    moe_router_logits_kernel(const __nv_bfloat16* __restrict__ x, const float* __restrict__ wr,
                             const float* __restrict__ bias, float* __restrict__ logits, int T, int H, int E) {
  __shared__ double xs[kRouteTokTile][kRouteHChunk];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t0 = blockIdx.x * kRouteTokTile;
  const int e0 = blockIdx.y * (kRouteWarps * kRouteExpPerWarp) + warp * kRouteExpPerWarp;
  double acc[kRouteExpPerWarp][kRouteTokTile];
#pragma unroll
  for (int q = 0; q < kRouteExpPerWarp; ++q)
#pragma unroll
    for (int t = 0; t < kRouteTokTile; ++t) acc[q][t] = 0.0;

  for (int h0 = 0; h0 < H; h0 += kRouteHChunk) {
    __syncthreads();
    for (int idx = threadIdx.x; idx < kRouteTokTile * kRouteHChunk; idx += blockDim.x) {
      const int t = idx / kRouteHChunk, hh = idx % kRouteHChunk;
      const int tok = t0 + t, h = h0 + hh;
      xs[t][hh] = (tok < T && h < H) ? static_cast<double>(__bfloat162float(x[static_cast<long long>(tok) * H + h])) : 0.0;
    }
    __syncthreads();
    // this lane's 8 consecutive elements of the 256-block (kRouteHChunk == 256)
#pragma unroll 1
    for (int j = 0; j < 8; ++j) {
      const int hh = 8 * lane + j;
      if (h0 + hh >= H) break;
      double wv[kRouteExpPerWarp];
#pragma unroll
      for (int q = 0; q < kRouteExpPerWarp; ++q) {
        const int e = e0 + q;
        wv[q] = (e < E) ? static_cast<double>(wr[static_cast<long long>(e) * H + h0 + hh]) : 0.0;
      }
#pragma unroll
      for (int t = 0; t < kRouteTokTile; ++t) {
        const double xv = xs[t][hh];
#pragma unroll
        for (int q = 0; q < kRouteExpPerWarp; ++q) acc[q][t] = fma(xv, wv[q], acc[q][t]);
      }
    }
  }
  // Butterfly: every lane ends with the same sum.
#pragma unroll
  for (int q = 0; q < kRouteExpPerWarp; ++q)
#pragma unroll
    for (int t = 0; t < kRouteTokTile; ++t) {
      double v = acc[q][t];
#pragma unroll
      for (int off = 16; off >= 1; off >>= 1) v = v + __shfl_xor_sync(0xffffffffu, v, off);
      acc[q][t] = v;
    }
  // Lane (q * 16 + t) writes logit (t, e0 + q).
#pragma unroll
  for (int q = 0; q < kRouteExpPerWarp; ++q)
#pragma unroll
    for (int t = 0; t < kRouteTokTile; ++t) {
      if (lane == q * kRouteTokTile + t) {
        const int tok = t0 + t, e = e0 + q;
        if (tok < T && e < E) {
          float l = __double2float_rn(acc[q][t]);
          if (bias) l = __fadd_rn(l, bias[e]);
          logits[static_cast<long long>(tok) * E + e] = l;
        }
      }
    }
}

// One warp per token: top-k of the token's E logits (descending; equal values: lower index first)
// and the renormalised softmax weights w_j = exp(l_j - l_max) / sum_i exp(l_i - l_max).
template <int PER_LANE>
__global__ void __launch_bounds__(256)
    moe_topk_kernel(const float* __restrict__ logits, float* __restrict__ topk_w, int* __restrict__ topk_ids,
                    int T, int E, int k) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= T) return;
  const float* row = logits + static_cast<long long>(warp) * E;
  float v[PER_LANE];
#pragma unroll
  for (int i = 0; i < PER_LANE; ++i) {
    const int e = i * 32 + lane;
    v[i] = (e < E) ? row[e] : -INFINITY;
  }
  unsigned int taken = 0;   // bit i: v[i] already selected
  float vmax = 0.f, my_val = 0.f;
  int my_id = -1;
  for (int j = 0; j < k; ++j) {
    // lane-local best among untaken (value desc, index asc)
    float bv = -INFINITY;
    int bi = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < PER_LANE; ++i) {
      const int e = i * 32 + lane;
      if (e < E && !(taken & (1u << i))) {
        if (v[i] > bv || (v[i] == bv && e < bi) || bi == 0x7fffffff) {
          bv = v[i];
          bi = e;
        }
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
    if ((bi & 31) == lane && bi != 0x7fffffff) taken |= 1u << (bi >> 5);
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
    topk_ids[static_cast<long long>(warp) * k + lane] = my_id;
    topk_w[static_cast<long long>(warp) * k + lane] = p / s;
  }
}

// ------------------------------------------------------------------------------------------------
// Permutation plan.  Chunks of kPlanChunk tokens.
// ------------------------------------------------------------------------------------------------
constexpr int kPlanChunk = 256;

// chunk_counts[c, e] = number of slots of chunk c routed to expert e.
__global__ void __launch_bounds__(kPlanChunk)
    moe_plan_count_kernel(const int* __restrict__ ids, int T, int E, int k, int* __restrict__ chunk_counts) {
  extern __shared__ int hist[];
  for (int e = threadIdx.x; e < E; e += blockDim.x) hist[e] = 0;
  __syncthreads();
  const int t = blockIdx.x * kPlanChunk + threadIdx.x;
  if (t < T) {
    for (int j = 0; j < k; ++j) {
      const int e = ids[static_cast<long long>(t) * k + j];
      if (e >= 0 && e < E) atomicAdd(&hist[e], 1);
      else report(KDB_ERR_DEVICE_BOUNDS, 0x201);
    }
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) chunk_counts[static_cast<long long>(blockIdx.x) * E + e] = hist[e];
}

// One CTA: counts[e], offsets[e] (exclusive, offsets[E] = T*k), chunk_base[c, e] (first row of
// chunk c's slots for expert e) and mtile_start[e] (exclusive prefix of ceil(counts / kMoeTokenTile)).
__global__ void __launch_bounds__(1024)
    moe_plan_scan_kernel(const int* __restrict__ chunk_counts, int C, int E, int* __restrict__ chunk_base,
                         int* __restrict__ counts, int* __restrict__ offsets, int* __restrict__ mtile_start) {
  __shared__ int s_warp[2][32];
  const int e = threadIdx.x;
  int total = 0;
  if (e < E) {
    for (int c = 0; c < C; ++c) total += chunk_counts[static_cast<long long>(c) * E + e];
  }
  const int mt = (total + kMoeTokenTile - 1) / kMoeTokenTile;
  // block-wide exclusive scans of total and mt (E <= 1024)
  const int lane = e & 31, w = e >> 5;
  int a = total, b = mt;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const int ya = __shfl_up_sync(0xffffffffu, a, off), yb = __shfl_up_sync(0xffffffffu, b, off);
    if (lane >= off) {
      a += ya;
      b += yb;
    }
  }
  if (lane == 31) {
    s_warp[0][w] = a;
    s_warp[1][w] = b;
  }
  __syncthreads();
  if (w == 0) {
    int pa = (lane < (int)(blockDim.x >> 5)) ? s_warp[0][lane] : 0;
    int pb = (lane < (int)(blockDim.x >> 5)) ? s_warp[1][lane] : 0;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int ya = __shfl_up_sync(0xffffffffu, pa, off), yb = __shfl_up_sync(0xffffffffu, pb, off);
      if (lane >= off) {
        pa += ya;
        pb += yb;
      }
    }
    s_warp[0][lane] = pa;
    s_warp[1][lane] = pb;
  }
  __syncthreads();
  const int incl_a = a + (w > 0 ? s_warp[0][w - 1] : 0);
  const int incl_b = b + (w > 0 ? s_warp[1][w - 1] : 0);
  if (e < E) {
    const int off0 = incl_a - total;
    counts[e] = total;
    offsets[e] = off0;
    mtile_start[e] = incl_b - mt;
    int run = off0;
    for (int c = 0; c < C; ++c) {
      chunk_base[static_cast<long long>(c) * E + e] = run;
      run += chunk_counts[static_cast<long long>(c) * E + e];
    }
    if (e == E - 1) {
      offsets[E] = incl_a;
      mtile_start[E] = incl_b;
    }
  }
}

// One CTA per chunk.  The chunk's expert ids and routing weights are staged in shared memory by all 256
// threads (coalesced loads, pieces of kScatterPiece slots); warp 0 then walks the slots in (token, j) order
// and hands out rows in that order within each expert, so the serial walk reads only shared memory.
// Writes perm_slot, slot_pos, perm_token and perm_w.
constexpr int kScatterPiece = 2048;

__global__ void __launch_bounds__(256)
    moe_plan_scatter_kernel(const int* __restrict__ ids, const float* __restrict__ topk_w, int T, int E, int k,
                            const int* __restrict__ chunk_base, int* __restrict__ perm_slot,
                            int* __restrict__ slot_pos, int* __restrict__ perm_token, float* __restrict__ perm_w) {
  extern __shared__ int cursor[];
  __shared__ int s_id[kScatterPiece];
  __shared__ float s_w[kScatterPiece];
  const int c = blockIdx.x;
  for (int e = threadIdx.x; e < E; e += blockDim.x) cursor[e] = chunk_base[static_cast<long long>(c) * E + e];
  const long long s0 = static_cast<long long>(c) * kPlanChunk * k;
  const long long s1 = min(static_cast<long long>(T) * k, s0 + static_cast<long long>(kPlanChunk) * k);
  for (long long p0 = s0; p0 < s1; p0 += kScatterPiece) {
    const int n = static_cast<int>(min(static_cast<long long>(kScatterPiece), s1 - p0));
    __syncthreads();   // cursors written; the previous piece consumed
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
      s_id[i] = ids[p0 + i];
      s_w[i] = topk_w[p0 + i];
    }
    __syncthreads();
    if (threadIdx.x >= 32) continue;
    const int lane = threadIdx.x;
    for (int base = 0; base < n; base += 32) {
      const int i = base + lane;
      const long long s = p0 + i;
      const bool valid = i < n;
      int e = valid ? s_id[i] : -1;
      if (valid && (e < 0 || e >= E)) e = -1;   // counted as a bounds error by the count kernel
      const unsigned int peers = __match_any_sync(0xffffffffu, e);
      const int rank = __popc(peers & ((1u << lane) - 1u));
      const int cur = (e >= 0) ? cursor[e] : 0;
      __syncwarp();
      if (e >= 0) {
        const int pos = cur + rank;
        perm_slot[pos] = static_cast<int>(s);
        slot_pos[s] = pos;
        perm_token[pos] = static_cast<int>(s / k);
        perm_w[pos] = s_w[i];
        const int leader = 31 - __clz(peers);   // highest lane of the group advances the cursor
        if (lane == leader) cursor[e] = cur + __popc(peers);
      } else if (valid) {
        slot_pos[s] = -1;
      }
      __syncwarp();
    }
  }
}

// x_perm[p, :] = x[perm_token[p] / div, :]  (16-byte vectors; H % 8 == 0)
__global__ void __launch_bounds__(256)
    moe_gather_rows_kernel(const __nv_bfloat16* __restrict__ x, const int* __restrict__ perm_token,
                           __nv_bfloat16* __restrict__ x_perm, int R, int H, int T, int div) {
  const int vec_per_row = H / 8;
  const int warps_per_cta = blockDim.x / 32;
  const int row = blockIdx.x * warps_per_cta + (threadIdx.x >> 5);
  if (row >= R) return;
  const int t = perm_token[row] / div;
  if (t < 0 || t >= T) {
    if ((threadIdx.x & 31) == 0) report(KDB_ERR_DEVICE_BOUNDS, 0x202);
    return;
  }
  const uint4* src = reinterpret_cast<const uint4*>(x + static_cast<long long>(t) * H);
  uint4* dst = reinterpret_cast<uint4*>(x_perm + static_cast<long long>(row) * H);
  for (int v = threadIdx.x & 31; v < vec_per_row; v += 32) dst[v] = __ldg(src + v);
}

// y[t, :] = sum_j [w[t*k + j] *] yperm[slot_pos[t*k + j], :] + yshared[t, :]   (fp32 sum in slot order, bf16 out)
__global__ void __launch_bounds__(256)
    moe_combine_kernel(const __nv_bfloat16* __restrict__ yperm, const int* __restrict__ slot_pos,
                       const float* __restrict__ slot_w, const __nv_bfloat16* __restrict__ yshared,
                       __nv_bfloat16* __restrict__ y, int T, int H, int k) {
  const int vec_per_row = H / 8;
  const long long gid = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  const long long t = gid / vec_per_row;
  const int v = static_cast<int>(gid % vec_per_row);
  if (t >= T) return;
  float acc[8];
#pragma unroll
  for (int q = 0; q < 8; ++q) acc[q] = 0.f;
  for (int j = 0; j < k; ++j) {
    const int p = slot_pos[t * k + j];
    if (p < 0) continue;
    const uint4 u = __ldg(reinterpret_cast<const uint4*>(yperm + static_cast<long long>(p) * H) + v);
    const __nv_bfloat162* b = reinterpret_cast<const __nv_bfloat162*>(&u);
    if (slot_w) {   // rows not yet scaled by their routing weight (expert-parallel path)
      const float wj = slot_w[t * k + j];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 f = __bfloat1622float2(b[q]);
        acc[2 * q] = fmaf(wj, f.x, acc[2 * q]);
        acc[2 * q + 1] = fmaf(wj, f.y, acc[2 * q + 1]);
      }
    } else {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 f = __bfloat1622float2(b[q]);
        acc[2 * q] += f.x;
        acc[2 * q + 1] += f.y;
      }
    }
  }
  if (yshared) {
    const uint4 u = __ldg(reinterpret_cast<const uint4*>(yshared + t * H) + v);
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
  reinterpret_cast<uint4*>(y + t * H)[v] = o;
}

// packed[e, nb*256 + half*128 + r, :] = w[e, half*I + nb*128 + r, :]
__global__ void __launch_bounds__(256)
    moe_pack_gate_up_kernel(const __nv_bfloat16* __restrict__ w, __nv_bfloat16* __restrict__ packed, int E, int I,
                            int H) {
  const long long rows = static_cast<long long>(E) * 2 * I;
  const int vec_per_row = H / 8;
  const long long prow = static_cast<long long>(blockIdx.x) * (blockDim.x / 32) + (threadIdx.x >> 5);
  if (prow >= rows) return;
  const long long e = prow / (2 * I);
  const int r = static_cast<int>(prow % (2 * I));
  const int nb = r / 256, half = (r % 256) / 128, rr = r % 128;
  const long long srow = e * 2 * I + static_cast<long long>(half) * I + nb * 128 + rr;
  const uint4* src = reinterpret_cast<const uint4*>(w + srow * H);
  uint4* dst = reinterpret_cast<uint4*>(packed + prow * H);
  for (int v = threadIdx.x & 31; v < vec_per_row; v += 32) dst[v] = src[v];
}

// ------------------------------------------------------------------------------------------------
// Host launchers
// ------------------------------------------------------------------------------------------------
int moe_route(const void* x, const float* wr, const float* bias, float* logits, float* topk_w, int* topk_ids,
              int T, int H, int E, int k, cudaStream_t s) {
  if (T <= 0) return KDB_OK;
  dim3 g1((T + kRouteTokTile - 1) / kRouteTokTile, (E + kRouteWarps * kRouteExpPerWarp - 1) / (kRouteWarps * kRouteExpPerWarp));
  moe_router_logits_kernel<<<g1, kRouteWarps * 32, 0, s>>>(static_cast<const __nv_bfloat16*>(x), wr, bias, logits, T,
                                                           H, E);
  int rc = cuda_status(cudaGetLastError());
  if (rc) return rc;
  const int blocks = (T * 32 + 255) / 256;
  const int per_lane = (E + 31) / 32;
  if (per_lane <= 2) moe_topk_kernel<2><<<blocks, 256, 0, s>>>(logits, topk_w, topk_ids, T, E, k);
  else if (per_lane <= 4) moe_topk_kernel<4><<<blocks, 256, 0, s>>>(logits, topk_w, topk_ids, T, E, k);
  else if (per_lane <= 8) moe_topk_kernel<8><<<blocks, 256, 0, s>>>(logits, topk_w, topk_ids, T, E, k);
  else moe_topk_kernel<32><<<blocks, 256, 0, s>>>(logits, topk_w, topk_ids, T, E, k);
  return cuda_status(cudaGetLastError());
}

int moe_plan(const int* ids, const float* topk_w, int T, int E, int k, int* chunk_counts, int* chunk_base,
             int* counts, int* offsets, int* mtile_start, int* perm_slot, int* slot_pos, int* perm_token,
             float* perm_w, cudaStream_t s) {
  const int C = (T + kPlanChunk - 1) / kPlanChunk;
  if (C == 0) {
    // no tokens: an empty plan
    cudaError_t e1 = cudaMemsetAsync(counts, 0, sizeof(int) * E, s);
    cudaError_t e2 = cudaMemsetAsync(offsets, 0, sizeof(int) * (E + 1), s);
    cudaError_t e3 = cudaMemsetAsync(mtile_start, 0, sizeof(int) * (E + 1), s);
    return cuda_status(e1 != cudaSuccess ? e1 : e2 != cudaSuccess ? e2 : e3);
  }
  moe_plan_count_kernel<<<C, kPlanChunk, sizeof(int) * E, s>>>(ids, T, E, k, chunk_counts);
  int rc = cuda_status(cudaGetLastError());
  if (rc) return rc;
  moe_plan_scan_kernel<<<1, ((E + 31) / 32) * 32, 0, s>>>(chunk_counts, C, E, chunk_base, counts, offsets, mtile_start);
  rc = cuda_status(cudaGetLastError());
  if (rc) return rc;
  moe_plan_scatter_kernel<<<C, 256, sizeof(int) * E, s>>>(ids, topk_w, T, E, k, chunk_base, perm_slot, slot_pos,
                                                          perm_token, perm_w);
  return cuda_status(cudaGetLastError());
}

int moe_gather_rows(const void* x, const int* perm_token, void* x_perm, int R, int H, int T, cudaStream_t s,
                    int div) {
  if (R <= 0) return KDB_OK;
  moe_gather_rows_kernel<<<(R + 7) / 8, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(x), perm_token,
                                                      static_cast<__nv_bfloat16*>(x_perm), R, H, T, div);
  return cuda_status(cudaGetLastError());
}

int moe_combine(const void* yperm, const int* slot_pos, const void* yshared, void* y, int T, int H, int k,
                cudaStream_t s, const float* slot_w) {
  if (T <= 0) return KDB_OK;
  const long long threads = static_cast<long long>(T) * (H / 8);
  moe_combine_kernel<<<static_cast<unsigned int>((threads + 255) / 256), 256, 0, s>>>(
      static_cast<const __nv_bfloat16*>(yperm), slot_pos, slot_w, static_cast<const __nv_bfloat16*>(yshared),
      static_cast<__nv_bfloat16*>(y), T, H, k);
  return cuda_status(cudaGetLastError());
}

int moe_pack_gate_up(const void* w, void* packed, int E, int I, int H, cudaStream_t s) {
  const long long rows = static_cast<long long>(E) * 2 * I;
  if (rows == 0) return KDB_OK;
  moe_pack_gate_up_kernel<<<static_cast<unsigned int>((rows + 7) / 8), 256, 0, s>>>(
      static_cast<const __nv_bfloat16*>(w), static_cast<__nv_bfloat16*>(packed), E, I, H);
  return cuda_status(cudaGetLastError());
}

}  // namespace kdb

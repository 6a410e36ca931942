// gemm_splitk_sm100.cuh — weight-streaming GEMM for small M (Y = X · Wᵀ with M <= 128) whose K split is
// reduced inside the same launch, through distributed shared memory.
//
// Shape: the weights are the MMA's M operand (MA parts of 128 rows per output tile), X's rows its N operand
// (NB rows, multiplied with N = rows rounded up to 16), as in gemm_swap_sm100.cuh.  With few rows every SM
// must stream a share of W, so K is split into S slices.  The S CTAs of one thread-block cluster compute
// the S slices of ONE output tile:
//   1. each CTA streams its slice of the tile's weight rows and token rows through a TMA ring and
//      accumulates MA x [128 x NB] fp32 in TMEM (one accumulator, one tile per CTA);
//   2. its epilogue warps stage the partial tile in shared memory (the ring is idle by then), fp32
//      [token][feature];
//   3. cluster barrier; every CTA then sums 1/S of the tile's elements over the S CTAs' partials, read
//      through distributed shared memory in slice order 0..S-1 (deterministic), and writes Y (bf16, or
//      fp32 for the router layer);
//   4. cluster barrier, so no CTA leaves while a peer still reads its shared memory.
// One launch, no global workspace and no partial round trip through HBM, which is what bounded the
// earlier two-launch form (GEMM writing fp32 partials + a reduction kernel) at these sizes.
//
// Every mbarrier wait is bounded (sm100_common.cuh); both cluster barriers are reached on every path, so a
// CTA whose wait gave up still meets its peers there.  No TMA multicast.
#pragma once

#include <cuda.h>
#include "gemm_sm100.cuh"
#include "gemm_swap_sm100.cuh"
#include "host_util.h"

namespace kdb {

template <int MA, int NB, int STAGES, int KC>
struct SplitKLayout {
  using Ring = SwapLayout<MA, NB, STAGES, KC>;
  static constexpr int kFeat = MA * 128;                            // output features of a tile
  static constexpr int kPartialBytes = NB * kFeat * 4;              // fp32 [NB tokens][kFeat]
  static constexpr int kRingBytes = STAGES * Ring::kStageBytes;
  static constexpr int kBarOffset = (kRingBytes > kPartialBytes ? kRingBytes : kPartialBytes);
  static constexpr int kBarBytes = (2 * STAGES + 2) * 8 + 16;
  static constexpr int kSmemBytes = kBarOffset + kBarBytes + 1024;
  static constexpr uint32_t kTmemCols = MA * NB <= 32 ? 32 : MA * NB <= 64 ? 64 : MA * NB <= 128 ? 128 : 256;
};

struct SplitKParams {
  int M, N, K;
  int f_tiles, t_tiles;    // output tiles: kFeat features x NB token rows; tile index = f * t_tiles + tt
  int splits;              // S = cluster size: CTA rank r takes k chunks [r * nkb_per, ...)
  int nkb_total, nkb_per;
  int b_kwrap;             // > 0: the token operand's k chunk wraps at b_kwrap ([W_hi | W_mid] weights)
  __nv_bfloat16* y;        // bf16 output, or
  float* y32;              // fp32 output (router layer) when not null
  long long ldy;
  bool vec_ok;             // 4 consecutive outputs of a row can be stored together
};

constexpr unsigned int kSiteSplitK = 0x130;

__device__ __forceinline__ float4 ld_dsmem_f4(uint32_t cluster_addr) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(cluster_addr)
               : "memory");
  return v;
}

template <int MA, int NB, int STAGES, int KC>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_splitk_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ TokenMaps tmB,
                       const SplitKParams p) {
  using L = SplitKLayout<MA, NB, STAGES, KC>;
  using R = typename L::Ring;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * R::kABytes;
  float* partial = reinterpret_cast<float*>(smem);   // reuses the ring once the MMAs are done
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kBarOffset);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* drain = tfull + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = warp_id_uniform();
  const uint32_t lane = lane_id();
  const int rank = static_cast<int>(cluster_ctarank());
  const int tile = blockIdx.x / p.splits;
  const int f = tile / p.t_tiles, tt = tile - f * p.t_tiles;
  const int row0 = tt * NB;
  const int n_valid = min(NB, p.M - row0);
  const int kb0 = rank * p.nkb_per;
  const int nkb = max(0, min(p.nkb_per, p.nkb_total - kb0));
  const int a_row = f * L::kFeat;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(tfull, 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
#pragma unroll
    for (int i = 0; i < 5; ++i) tma_prefetch_desc(&tmB.m[i]);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, L::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------------ TMA producer
      const uint64_t pol = l2_policy_evict_normal();
      const int bi = box_index(n_valid);
      const uint32_t chunk_bytes = R::kAChunk + (16u << bi) * kBK * 2;
      uint32_t stage = 0, phase = 0, armed_mask = 0, armed_phase = 0;
      for (int kb = 0; kb < nkb; kb += KC) {
        const int nc = min(KC, nkb - kb);
        if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, kSiteProdEmpty)) break;
        mbar_arrive_expect_tx(&full[stage], nc * chunk_bytes);
#pragma unroll
        for (int c = 0; c < KC; ++c) {
          if (c < nc) {
            const int kc = kb0 + kb + c;
#pragma unroll
            for (int a = 0; a < MA; ++a)
              tma_load_2d(sA + stage * R::kABytes + c * R::kAChunk + a * 128 * kBK * 2, &tmA, &full[stage], kc * kBK,
                          a_row + a * 128, pol);
            tma_load_2d(sB + stage * R::kBBytesMax + c * R::kBChunk, &tmB.m[bi], &full[stage],
                        (p.b_kwrap > 0 ? kc % p.b_kwrap : kc) * kBK, row0, pol);
          }
        }
        armed_mask |= 1u << stage;
        armed_phase = (armed_phase & ~(1u << stage)) | (phase << stage);
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
      for (int s = 0; s < STAGES; ++s)
        if (armed_mask & (1u << s)) mbar_wait_drain(&full[s], (armed_phase >> s) & 1u, kSiteDrainTma);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------------------------ MMA issuer
      const int n_mma = (n_valid + 15) & ~15;
      const uint32_t idesc = idesc_bf16_f32(128, n_mma);
      uint32_t stage = 0, phase = 0;
      bool ok = true, issued = false;
      for (int kb = 0; kb < nkb; kb += KC) {
        const int nc = min(KC, nkb - kb);
        if (!mbar_wait(&full[stage], phase, abort_flag, kSiteMmaFull)) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < KC; ++c) {
          if (c >= nc) break;
          const uint32_t a_addr = smem_u32(sA + stage * R::kABytes + c * R::kAChunk);
          const uint32_t b_addr = smem_u32(sB + stage * R::kBBytesMax + c * R::kBChunk);
#pragma unroll
          for (int kk = 0; kk < kBK / kUmmaK; ++kk) {
            const uint64_t bdesc = sdesc_sw128_kmajor(b_addr + kk * kUmmaK * 2);
#pragma unroll
            for (int a = 0; a < MA; ++a)
              mma_bf16(tmem_base + a * NB, sdesc_sw128_kmajor(a_addr + a * 128 * kBK * 2 + kk * kUmmaK * 2), bdesc,
                       idesc, (kb | c | kk) != 0);
          }
        }
        mma_commit(&empty[stage]);
        issued = true;
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (ok && issued) mma_commit(tfull);   // arrives once the accumulator is complete
      if (issued) {
        mma_commit(drain);
        mbar_wait_drain(drain, 0, kSiteDrainMma);
      }
      // an empty slice (nkb == 0) or a failed wait still releases the epilogue, which then stages zeros
      if (!(ok && issued)) mbar_arrive(tfull);
    }
  } else {
    // -------------------------------------------------------------------- epilogue: stage the partial
    const int quad = warp & 3;
    const int r = quad * 32 + static_cast<int>(lane);
    const bool ok = mbar_wait(tfull, 0, abort_flag, kSiteEpiTmemFull);
    const bool all_ok = __all_sync(0xffffffffu, ok);
    tc_fence_after();
    const bool use_acc = all_ok && nkb > 0 && *abort_flag == 0;
#pragma unroll 1
    for (int a = 0; a < MA; ++a) {
#pragma unroll 1
      for (int c0 = 0; c0 < n_valid; c0 += 32) {
        uint32_t v[32];
        if (use_acc) {
          tmem_ld_32x32b_x32(tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + a * NB + c0, v);
          tmem_ld_wait();
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = 0u;
        }
        const int n = min(32, n_valid - c0);
#pragma unroll
        for (int i = 0; i < 32; ++i)
          if (i < n) partial[(c0 + i) * L::kFeat + a * 128 + r] = __uint_as_float(v[i]);
      }
    }
  }

  // ---------------------------------------------------------------------- reduce across the cluster
  tc_fence_before();
  __syncthreads();
  __syncwarp();
  cluster_sync();   // every CTA's partial is staged
  {
    const int n_feat = min(L::kFeat, p.N - a_row);   // valid features of this tile
    const int groups = L::kFeat / 4;                   // 4 consecutive features per item
    const int items = n_valid * groups;
    const int per = (items + p.splits - 1) / p.splits;
    const int i0 = rank * per, i1 = min(items, i0 + per);
    const uint32_t base = smem_u32(partial);
    // two items per thread and pass, all their S loads in flight before the first add (the loads are
    // latency-bound); the adds then run in slice order
    const int stride = static_cast<int>(blockDim.x);
    for (int it = i0 + static_cast<int>(threadIdx.x); it < i1; it += 2 * stride) {
      float4 v[2][8];
      int tk[2], ft[2];
      bool live[2];
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int item = it + u * stride;
        tk[u] = item / groups;
        ft[u] = (item - tk[u] * groups) * 4;
        live[u] = item < i1 && ft[u] < n_feat;
        const uint32_t off = static_cast<uint32_t>((tk[u] * L::kFeat + ft[u]) * 4);
#pragma unroll
        for (int s = 0; s < 8; ++s)
          if (live[u] && s < p.splits) v[u][s] = ld_dsmem_f4(mapa_shared(base + off, static_cast<uint32_t>(s)));
      }
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        if (!live[u]) continue;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int s = 0; s < 8; ++s) {
          if (s < p.splits) {
            acc.x += v[u][s].x;
            acc.y += v[u][s].y;
            acc.z += v[u][s].z;
            acc.w += v[u][s].w;
          }
        }
        const int tok = tk[u], feat = ft[u];
        const long long row = row0 + tok;
        const int col = a_row + feat;
        const float o[4] = {acc.x, acc.y, acc.z, acc.w};
        if (p.y32) {
          float* dst = p.y32 + row * p.ldy + col;
          if (p.vec_ok && feat + 4 <= n_feat) {
            *reinterpret_cast<float4*>(dst) = acc;
          } else {
            for (int e = 0; e < 4; ++e)
              if (feat + e < n_feat) dst[e] = o[e];
          }
        } else {
          __nv_bfloat16* dst = p.y + row * p.ldy + col;
          if (p.vec_ok && feat + 4 <= n_feat) {
            uint2 pk;
            pk.x = pack_bf16x2(acc.x, acc.y);
            pk.y = pack_bf16x2(acc.z, acc.w);
            *reinterpret_cast<uint2*>(dst) = pk;
          } else {
            for (int e = 0; e < 4; ++e)
              if (feat + e < n_feat) dst[e] = __float2bfloat16_rn(o[e]);
          }
        }
      }
    }
  }
  __syncwarp();
  cluster_sync();   // no CTA leaves while a peer may still read its partial
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, L::kTmemCols);
  }
}

}  // namespace kdb

// gemm_swap_sm100.cuh — persistent warp-specialised tcgen05 GEMM with the weights as the M operand
// and a token block of per-tile size as the N operand ("swapped operands"), for the grouped expert
// GEMMs of the MoE layer.
//
// Why: the tokens routed to one expert rarely fill a multiple of 128 rows.  With tokens as M every
// expert's last tile is padded to 128 rows (a quarter of the prefill layer's MMA work); with tokens
// as N the MMA's N is rounded up only to 16.  For each tile:
//   A = MA x 128 weight rows (MA = 2 for gate_up: 128 gate rows + the matching 128 up rows),
//   B = n_valid <= NB token rows, loaded with the smallest of five TMA boxes (16..256 rows) that holds
//       them, multiplied with N = n_valid rounded up to 16,
//   D = MA accumulators of 128 TMEM lanes (weight rows) x NB columns (tokens), double buffered.
// Epilogue lane l of warp q owns weight row 32q + l of every accumulator, so gate and up of one
// intermediate feature meet in the same thread, and a warp's 32 lanes write 32 consecutive features of
// one token row (64-byte coalesced stores).
//
// Roles, bounded waits and the drain/teardown path are those of gemm_sm100.cuh.
#pragma once

#include <cuda.h>
#include "gemm_sm100.cuh"
#include "host_util.h"

namespace kdb {

// One tile of a swapped-operand GEMM: weight rows [a_row, a_row + 128*MA) (parts a_part_stride apart),
// token rows [b_row, b_row + n_valid), k slices [kb0, kb0 + nkb); f0 / row0 / split locate the output.
// b_kwrap > 0: the token operand's k chunk index wraps at b_kwrap (the weights hold [W_hi | W_mid] side by
// side along K, both multiplied by the same token row).
struct SwapTile {
  int a_row, a_part_stride, b_row, kb0, nkb, n_valid;
  int f0, row0, split;
  int b_kwrap = 0;
};


__host__ __device__ constexpr int box_index(int rows) {
  return rows <= 16 ? 0 : rows <= 32 ? 1 : rows <= 64 ? 2 : rows <= 128 ? 3 : 4;
}

// KC: 64-wide k chunks per pipeline stage.  Several chunks per stage ask HBM for KC adjacent 128-byte
// pieces of every weight row together rather than one per stage, which weight-streaming tiles need.
template <int MA, int NB, int STAGES, int KC = 1>
struct SwapLayout {
  static_assert(MA == 1 || MA == 2, "one or two 128-row weight blocks per tile");
  static_assert(NB == 32 || NB == 64 || NB == 128 || NB == 256, "token block of a tile");
  static_assert(MA * NB <= 256, "two accumulators of MA x NB columns must fit the 512 TMEM columns");
  static constexpr int kAChunk = MA * 128 * kBK * 2;       // one k chunk of the weight parts
  static constexpr int kBChunk = NB * kBK * 2;             // one k chunk of the token block
  static constexpr int kABytes = KC * kAChunk;
  static constexpr int kBBytesMax = KC * kBChunk;
  static constexpr int kStageBytes = kABytes + kBBytesMax;
  static constexpr int kBarOffset = STAGES * kStageBytes;
  static constexpr int kBarBytes = (2 * STAGES + 5) * 8 + 16;
  static constexpr int kSmemBytes = kBarOffset + kBarBytes + 1024;
  static constexpr int kAccCols = MA * NB;    // TMEM columns of one accumulator set
  static constexpr uint32_t kTmemCols = (2 * kAccCols <= 256) ? 256 : 512;
};

template <class Sched, class Epi, int MA, int NB, int STAGES, int KC = 1>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_swap_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ TokenMaps tmB,
                     const typename Sched::Params sp, const typename Epi::Params ep) {
  using L = SwapLayout<MA, NB, STAGES, KC>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * L::kABytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kBarOffset);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = warp_id_uniform();
  const uint32_t lane = lane_id();

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 128);
    }
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

  Sched sched(sp);
  const int ntiles = sched.num_tiles();

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------------ TMA producer
      const uint64_t pol_w = l2_policy_evict_normal();
      const uint64_t pol_t = l2_policy_evict_normal();
      uint32_t stage = 0, phase = 0;
      uint32_t armed_mask = 0, armed_phase = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < ntiles; t += gridDim.x) {
        const auto ti = sched.tile(t);
        const int bi = box_index(ti.n_valid);
        const uint32_t chunk_bytes = L::kAChunk + (16u << bi) * kBK * 2;
        for (int kb = 0; kb < ti.nkb; kb += KC) {   // one stage = nc <= KC k chunks of this tile
          const int nc = min(KC, ti.nkb - kb);
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, kSiteProdEmpty)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[stage], nc * chunk_bytes);
#pragma unroll
          for (int c = 0; c < KC; ++c) {
            if (c < nc) {
              const int kc = (ti.kb0 + kb + c) * kBK;
#pragma unroll
              for (int a = 0; a < MA; ++a)
                tma_load_2d(sA + stage * L::kABytes + c * L::kAChunk + a * 128 * kBK * 2, &tmA, &full[stage], kc,
                            ti.a_row + a * ti.a_part_stride, pol_w);
            }
          }
#pragma unroll
          for (int c = 0; c < KC; ++c)
            if (c < nc)
              tma_load_2d(sB + stage * L::kBBytesMax + c * L::kBChunk, &tmB.m[bi], &full[stage],
                          (ti.b_kwrap > 0 ? (ti.kb0 + kb + c) % ti.b_kwrap : ti.kb0 + kb + c) * kBK, ti.b_row,
                          pol_t);
          armed_mask |= 1u << stage;
          armed_phase = (armed_phase & ~(1u << stage)) | (phase << stage);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      for (int s = 0; s < STAGES; ++s)
        if (armed_mask & (1u << s)) mbar_wait_drain(&full[s], (armed_phase >> s) & 1u, kSiteDrainTma);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------------------------ MMA issuer
      uint32_t stage = 0, phase = 0;
      bool issued = false, ok = true;
      int it = 0;
      for (int t = blockIdx.x; ok && t < ntiles; t += gridDim.x, ++it) {
        const auto ti = sched.tile(t);
        const int n_mma = (ti.n_valid + 15) & ~15;
        const uint32_t idesc = idesc_bf16_f32(128, n_mma);
        const uint32_t acc = it & 1, aph = (it >> 1) & 1;
        if (!mbar_wait(&tempty[acc], aph ^ 1u, abort_flag, kSiteMmaTmemEmpty)) break;
        tc_fence_after();
        const uint32_t d_base = tmem_base + acc * L::kAccCols;
        for (int kb = 0; kb < ti.nkb; kb += KC) {
          const int nc = min(KC, ti.nkb - kb);
          if (!mbar_wait(&full[stage], phase, abort_flag, kSiteMmaFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int c = 0; c < KC; ++c) {
            if (c >= nc) break;
            const uint32_t a_addr = smem_u32(sA + stage * L::kABytes + c * L::kAChunk);
            const uint32_t b_addr = smem_u32(sB + stage * L::kBBytesMax + c * L::kBChunk);
#pragma unroll
            for (int kk = 0; kk < kBK / kUmmaK; ++kk) {
              const uint64_t bdesc = sdesc_sw128_kmajor(b_addr + kk * kUmmaK * 2);
#pragma unroll
              for (int a = 0; a < MA; ++a)
                mma_bf16(d_base + a * NB, sdesc_sw128_kmajor(a_addr + a * 128 * kBK * 2 + kk * kUmmaK * 2), bdesc,
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
        if (ok) mma_commit(&tfull[acc]);
      }
      if (issued) {
        mma_commit(drain);
        mbar_wait_drain(drain, 0, kSiteDrainMma);
      }
    }
  } else {
    // -------------------------------------------------------------------- epilogue (128 threads)
    const int quad = warp & 3;   // TMEM lanes [32*quad, 32*quad+32): weight rows of this warp
    int it = 0;
    for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ++it) {
      const uint32_t acc = it & 1, aph = (it >> 1) & 1;
      const bool ok = mbar_wait(&tfull[acc], aph, abort_flag, kSiteEpiTmemFull);
      if (!__all_sync(0xffffffffu, ok)) break;
      tc_fence_after();
      const auto ti = sched.tile(t);
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + acc * L::kAccCols;
      Epi::template run<NB>(ep, ti, quad * 32 + static_cast<int>(lane), taddr);
      tc_fence_before();
      mbar_arrive(&tempty[acc]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, L::kTmemCols);
  }
}

}  // namespace kdb

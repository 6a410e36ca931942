// gemm_sm100.cuh — persistent warp-specialised tcgen05 GEMM core, D = A · Bᵀ with A[rows, K] and
// B[cols, K] both K-major bf16, fp32 accumulation in tensor memory.
//
// One CTA per SM loops over output tiles handed out by a scheduler policy.  Roles:
//   warp 0, lane 0   TMA producer: fills a STAGES-deep ring of (A, B) k-slices in shared memory
//   warp 1, lane 0   MMA issuer: tcgen05.mma (128 x BN x 16) into one of two TMEM accumulators
//   warps 2..5       epilogue: tcgen05.ld of the finished accumulator, then the epilogue policy
// The two TMEM accumulators let the epilogue of tile i overlap the main loop of tile i+1.
//
// Policies:
//   Sched::Params, Sched(params), int num_tiles(), TileInfo tile(int t)
//     TileInfo has a_row, b_row (TMA row coordinates), nkb (number of 64-wide k slices), a_kwrap
//     (0, or the number of k slices after which A's k coordinate starts again at 0, so one A tile
//     multiplies B's k range [0, nkb*64) as [A | A | ...]), and the fields the epilogue needs.
//   Epi::Params, static void run(params, tile_info, row_in_tile, taddr_row)
//     row_in_tile in [0, 128); taddr_row addresses TMEM lane row_in_tile, column 0 of the tile.
//
// All waits are bounded (sm100_common.cuh).  On a timeout every role leaves its loop, the producer
// waits for its TMA copies in flight, the MMA issuer waits for its MMAs in flight, and the
// allocating warp frees the TMEM before the CTA exits.
#pragma once

#include <cuda.h>
#include "sm100_common.cuh"

namespace kdb {

constexpr int kBK = 64;       // bf16 elements per k slice: one 128-byte swizzle row
constexpr int kUmmaK = 16;    // K of one kind::f16 tcgen05.mma
constexpr int kGemmThreads = 192;

// Sites reported with KDB_ERR_TIMEOUT.
enum : unsigned int {
  kSiteProdEmpty = 0x101,
  kSiteMmaTmemEmpty = 0x102,
  kSiteMmaFull = 0x103,
  kSiteEpiTmemFull = 0x104,
  kSiteDrainTma = 0x105,
  kSiteDrainMma = 0x106,
};

template <int BM, int BN, int STAGES>
struct GemmLayout {
  static_assert(BM == 128, "one CTA owns 128 TMEM lanes");
  static_assert(BN % 32 == 0 && BN >= 32 && BN <= 256, "tcgen05 N for M=128 is a multiple of 16 up to 256");
  static constexpr int kABytes = BM * kBK * 2;
  static constexpr int kBBytes = BN * kBK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kBarOffset = STAGES * kStageBytes;
  // barriers: full[S], empty[S], tfull[2], tempty[2], drain ; then tmem slot, abort flag
  static constexpr int kBarBytes = (2 * STAGES + 5) * 8 + 16;
  static constexpr int kSmemBytes = kBarOffset + kBarBytes + 1024;   // + slack for 1024-B alignment
  static constexpr uint32_t kTmemCols = (2 * BN <= 32) ? 32 : (2 * BN <= 64) ? 64 : (2 * BN <= 128) ? 128
                                       : (2 * BN <= 256) ? 256 : 512;
  static constexpr uint32_t kIdesc = idesc_bf16_f32(BM, BN);
};

// Bounded wait used only while draining after an abort: ignores the abort flag.
__device__ __forceinline__ bool mbar_wait_drain(uint64_t* bar, uint32_t parity, unsigned int site) {
  const uint64_t t0 = globaltimer();
  while (!mbar_test(bar, parity)) {
    if (globaltimer() - t0 > KDB_WAIT_NS) {
      report(KDB_ERR_TIMEOUT, site);
      return false;
    }
  }
  return true;
}

template <class Sched, class Epi, int BM, int BN, int STAGES>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_tn_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const typename Sched::Params sp, const typename Epi::Params ep) {
  using L = GemmLayout<BM, BN, STAGES>;
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
    tma_prefetch_desc(&tmB);
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
      const uint64_t pol_a = l2_policy_evict_normal();
      const uint64_t pol_b = l2_policy_evict_normal();
      uint32_t stage = 0, phase = 0;
      uint32_t armed_mask = 0, armed_phase = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < ntiles; t += gridDim.x) {
        const auto ti = sched.tile(t);
        for (int kb = 0; kb < ti.nkb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, kSiteProdEmpty)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[stage], L::kStageBytes);
          const int a_kb = ti.a_kwrap > 0 ? kb % ti.a_kwrap : kb;   // A's k coordinate may wrap
          tma_load_2d(sA + stage * L::kABytes, &tmA, &full[stage], a_kb * kBK, ti.a_row, pol_a);
          tma_load_2d(sB + stage * L::kBBytes, &tmB, &full[stage], kb * kBK, ti.b_row, pol_b);
          armed_mask |= 1u << stage;
          armed_phase = (armed_phase & ~(1u << stage)) | (phase << stage);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // Every armed stage must have landed before the CTA may exit (a no-op on the normal path,
      // where the MMA issuer consumed them all).
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
        const uint32_t acc = it & 1, aph = (it >> 1) & 1;
        if (!mbar_wait(&tempty[acc], aph ^ 1u, abort_flag, kSiteMmaTmemEmpty)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = 0; kb < ti.nkb; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag, kSiteMmaFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(sA + stage * L::kABytes);
          const uint32_t b_addr = smem_u32(sB + stage * L::kBBytes);
#pragma unroll
          for (int kk = 0; kk < kBK / kUmmaK; ++kk) {
            mma_bf16(d_tmem, sdesc_sw128_kmajor(a_addr + kk * kUmmaK * 2),
                     sdesc_sw128_kmajor(b_addr + kk * kUmmaK * 2), L::kIdesc, (kb | kk) != 0);
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
    const int quad = warp & 3;   // TMEM lanes [32*quad, 32*quad+32) are reachable from this warp
    const int row_in_tile = quad * 32 + static_cast<int>(lane);
    int it = 0;
    for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ++it) {
      const uint32_t acc = it & 1, aph = (it >> 1) & 1;
      // tcgen05.ld is warp-collective: the whole warp leaves together if any lane gave up.
      const bool ok = mbar_wait(&tfull[acc], aph, abort_flag, kSiteEpiTmemFull);
      if (!__all_sync(0xffffffffu, ok)) break;
      tc_fence_after();
      const auto ti = sched.tile(t);
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + acc * BN;
      Epi::run(ep, ti, row_in_tile, taddr);
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

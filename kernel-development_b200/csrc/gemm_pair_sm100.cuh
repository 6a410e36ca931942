// gemm_pair_sm100.cuh — persistent tcgen05 GEMM on CTA pairs (cta_group::2): one 256 x BN output tile
// per pair of SMs.
//
// CTA rank r (0 or 1) of a 2-CTA cluster loads its own 128 rows of A and half of B's BN rows; the even
// CTA (the leader) issues 256 x BN x 16 MMAs that read both CTAs' shared memory and write each CTA's
// 128 rows of the accumulator into that CTA's TMEM.  Compared with one CTA per 128 x BN tile, every SM
// stages half as many B bytes per FLOP, which relieves the shared-memory and L2 bandwidth that bounds
// the single-CTA kernel.
//
// Signalling (all mbarrier waits bounded as in sm100_common.cuh):
//   full[s]    leader's only: the leader arms it for both CTAs' bytes; both CTAs' TMA copies complete
//              on it (cta_group::2 copies may signal the peer's barrier; no multicast)
//   empty[s]   both CTAs: the leader's MMA completion arrives on both (multicast tcgen05.commit)
//   tfull[a]   both CTAs: accumulator a is complete (multicast tcgen05.commit)
//   tempty[a]  leader's only: all 256 epilogue threads of the pair have read accumulator a
// The pair meets at cluster barriers after initialisation and before TMEM is freed, so no CTA signals
// a barrier of a peer that has not started or has already left.
#pragma once

#include <cuda.h>
#include "gemm_sm100.cuh"

namespace kdb {

template <int BN, int STAGES>
struct PairLayout {
  static_assert(BN % 32 == 0 && BN >= 64 && BN <= 256, "pair MMA N: multiple of 16 up to 256");
  static constexpr int kABytes = 128 * kBK * 2;          // this CTA's 128 A rows
  static constexpr int kBBytes = (BN / 2) * kBK * 2;     // this CTA's half of B
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr uint32_t kPairTx = 2 * kStageBytes;   // bytes landing on the leader's full barrier
  static constexpr int kBarOffset = STAGES * kStageBytes;
  static constexpr int kBarBytes = (2 * STAGES + 5) * 8 + 16;
  static constexpr int kSmemBytes = kBarOffset + kBarBytes + 1024;
  static constexpr uint32_t kTmemCols = (2 * BN <= 256) ? 256 : 512;
  static constexpr uint32_t kIdesc = idesc_bf16_f32(256, BN);
};

template <class Sched, class Epi, int BN, int STAGES>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_tn_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                        const typename Sched::Params sp, const typename Epi::Params ep) {
  using L = PairLayout<BN, STAGES>;
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
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 2 * 128);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, L::kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();   // both CTAs' barriers exist before either signals the other
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const uint32_t full_lead = mapa_shared(smem_u32(full), 0);
  const uint32_t tempty_lead = mapa_shared(smem_u32(tempty), 0);

  Sched sched(sp);
  const int ntiles = sched.num_tiles();
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------------ TMA producer (both CTAs)
      const uint64_t pol = l2_policy_evict_normal();
      uint32_t stage = 0, phase = 0;
      uint32_t armed_mask = 0, armed_phase = 0;
      bool ok = true;
      for (int t = pair; ok && t < ntiles; t += npairs) {
        const auto ti = sched.tile(t);
        for (int kb = 0; kb < ti.nkb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, kSiteProdEmpty)) {
            ok = false;
            break;
          }
          if (leader) mbar_arrive_expect_tx(&full[stage], L::kPairTx);
          const int a_kb = ti.a_kwrap > 0 ? kb % ti.a_kwrap : kb;
          tma_load_2d_pair(sA + stage * L::kABytes, &tmA, full_lead + 8u * stage, a_kb * kBK,
                           ti.a_row + 128 * static_cast<int>(rank), pol);
          tma_load_2d_pair(sB + stage * L::kBBytes, &tmB, full_lead + 8u * stage, kb * kBK,
                           ti.b_row + (BN / 2) * static_cast<int>(rank), pol);
          armed_mask |= 1u << stage;
          armed_phase = (armed_phase & ~(1u << stage)) | (phase << stage);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (leader) {
        for (int s = 0; s < STAGES; ++s)
          if (armed_mask & (1u << s)) mbar_wait_drain(&full[s], (armed_phase >> s) & 1u, kSiteDrainTma);
      } else if (!ok && armed_mask) {
        // the peer cannot test the leader's barriers: give copies in flight a bounded time to land
        const uint64_t t0 = globaltimer();
        while (globaltimer() - t0 < 200000ull) {
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      // ------------------------------------------------------------------ MMA issuer (leader)
      uint32_t stage = 0, phase = 0;
      bool issued = false, ok = true;
      int it = 0;
      for (int t = pair; ok && t < ntiles; t += npairs, ++it) {
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
            mma_bf16_pair(d_tmem, sdesc_sw128_kmajor(a_addr + kk * kUmmaK * 2),
                          sdesc_sw128_kmajor(b_addr + kk * kUmmaK * 2), L::kIdesc, (kb | kk) != 0);
          }
          mma_commit_pair(&empty[stage], 0x3);
          issued = true;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (ok) mma_commit_pair(&tfull[acc], 0x3);
      }
      if (issued) {
        mma_commit_pair(drain, 0x1);
        mbar_wait_drain(drain, 0, kSiteDrainMma);
      }
    }
  } else {
    // -------------------------------------------------------------------- epilogue (both CTAs)
    const int quad = warp & 3;
    const int row_in_tile = quad * 32 + static_cast<int>(lane);
    int it = 0;
    for (int t = pair; t < ntiles; t += npairs, ++it) {
      const uint32_t acc = it & 1, aph = (it >> 1) & 1;
      const bool ok = mbar_wait(&tfull[acc], aph, abort_flag, kSiteEpiTmemFull);
      if (!__all_sync(0xffffffffu, ok)) break;
      tc_fence_after();
      auto ti = sched.tile(t);
      ti.m0 += 128 * static_cast<int>(rank);   // this CTA's rows of the pair's 256-row tile
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + acc * BN;
      Epi::run(ep, ti, row_in_tile, taddr);
      tc_fence_before();
      if (leader) mbar_arrive(&tempty[acc]);
      else mbar_arrive_cluster(tempty_lead + 8u * acc);
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();   // no CTA leaves while its peer may still signal it
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, L::kTmemCols);
  }
}

}  // namespace kdb

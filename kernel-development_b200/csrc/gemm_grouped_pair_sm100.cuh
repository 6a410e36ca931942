// gemm_grouped_pair_sm100.cuh — grouped expert GEMM on CTA pairs (cta_group::2): the weights are the M
// operand (256 rows per pair, 128 per CTA) and up to 512 tokens of ONE expert are the N operand.
//
// Why this shape.  The expert GEMMs of a prefill layer sit at the HBM/tensor ridge: every expert sees about
// as many tokens as the ridge intensity, so the kernel must stream each expert's weights from HBM once while
// keeping the tensor pipe busy.  Two measured limits set the design:
//   * an SM's TMA path delivers roughly 80-90 GB/s from L2 (32-64 KB per stage), so a 128 x 256 single-CTA
//     tile (48 KB per 4.2 MFLOP) cannot feed the tensor pipe, while a 256 x 256 pair tile (32 KB per CTA per
//     4.2 MFLOP) can;
//   * an expert's weight tile read by two different tiles at different times is read from HBM twice, so all
//     tokens of an expert (up to 512) go through one tile: one pass over the weights per expert.
// N > 256 is issued as two MMAs per k step into two 256-column TMEM slots; a tile of <= 256 tokens uses one
// slot, so consecutive small tiles still double-buffer the accumulator.
//
// Per stage each CTA stages its 128 weight rows (one 128-row box, or two 64-row boxes: gate_up puts 64 gate
// rows and the 64 matching up rows of its features in one 128-row operand) and its half of each token
// group: tokens [0, m1) split m1/2 per CTA, then tokens [m1, n) split the same way (m1 = min(n16, 256),
// n16 = tokens rounded up to 16).
//
// Signalling follows gemm_pair_sm100.cuh (all waits bounded): full[s] (leader's, both CTAs' copies land on
// it), empty[s] (both CTAs, multicast commit), tfull[slot] (both CTAs, multicast commit), tempty[slot]
// (leader's, 512 epilogue arrivals).  Each epilogue group votes (bar.red.or over its 128 threads) after each
// bounded wait, so its named barriers are reached by all four of its warps or by none.
#pragma once

#include <cuda.h>
#include "gemm_sm100.cuh"
#include "gemm_swap_sm100.cuh"
#include "host_util.h"

namespace kdb {

constexpr int kGpTokens = 512;     // tokens of one tile at most
constexpr int kGpSlotCols = 256;   // TMEM columns of one accumulator slot

// One pair tile.  CTA r stages weight rows a_row + r * a_rank_stride (+ a_box_stride for its second box).
struct GpTile {
  int a_row, a_box_stride, a_rank_stride;
  int b_row;      // first token row of the tile (also its first output row)
  int n_valid;    // tokens, 1..512
  int nkb;        // 64-wide k chunks
  int f0;         // first output feature of the pair tile
};

template <int ABOXES, int STAGES, int EPI_BYTES>
struct GpLayout {
  static_assert(ABOXES == 1 || ABOXES == 2, "one 128-row or two 64-row weight boxes per CTA");
  static constexpr int kABoxRows = 128 / ABOXES;
  static constexpr int kABytes = 128 * kBK * 2;           // this CTA's 128 weight rows
  static constexpr int kBRegion = 128 * kBK * 2;          // this CTA's <= 128 rows of tokens [0, 256)
  static constexpr int kBRegion2 = (kGpTokens - kGpSlotCols) / 2 * kBK * 2;   // its rows of tokens [256, n)
  static constexpr int kStageBytes = kABytes + kBRegion + kBRegion2;
  static constexpr int kEpiOffset = STAGES * kStageBytes;
  static constexpr int kBarOffset = kEpiOffset + EPI_BYTES;
  static constexpr int kBarBytes = (2 * STAGES + 5) * 8 + 16;
  static constexpr int kSmemBytes = kBarOffset + kBarBytes + 1024;
  static constexpr uint32_t kTmemCols = 2 * kGpSlotCols;
};

// Token split of a tile: m1 columns in slot A (tokens [0, m1)), m2 in slot B (tokens [m1, m1 + m2)).
struct GpSplit {
  int m1, m2;
  __device__ explicit GpSplit(int n_valid) {
    const int n16 = (n_valid + 15) & ~15;
    m1 = n16 < kGpSlotCols ? n16 : kGpSlotCols;
    m2 = n16 - m1;
  }
};

// Two epilogue groups of four warps (warps 2-5 and 6-9; each group covers all four TMEM lane quarters)
// take alternate 32-token chunks of an accumulator.  Group g uses named barriers 1 + 2g (vote) and
// 2 + 2g (data exchange), 128 threads each.
constexpr int kGpThreads = 64 + 2 * 128;

// All 128 threads of an epilogue group agree on `ok`: false if any thread's wait failed.
__device__ __forceinline__ bool epi_vote_all(bool ok, int grp) {
  uint32_t bad = ok ? 0u : 1u, any;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.or.pred q, %2, 128, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(any)
      : "r"(bad), "r"(1 + 2 * grp)
      : "memory");
  return any == 0u;
}

__device__ __forceinline__ void epi_bar_sync(int grp) {
  asm volatile("bar.sync %0, 128;" ::"r"(2 + 2 * grp) : "memory");
}

template <class Sched, class Epi, int ABOXES, int STAGES>
__global__ void __launch_bounds__(kGpThreads, 1)
    gemm_grouped_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ TokenMaps tmB,
                             const typename Sched::Params sp, const typename Epi::Params ep) {
  using L = GpLayout<ABOXES, STAGES, 2 * Epi::kSmemBytes>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* epi_smem = smem + L::kEpiOffset;
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
      mbar_init(&tempty[a], 2 * 256);   // both CTAs' epilogue threads
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
#pragma unroll
    for (int i = 0; i < 5; ++i) tma_prefetch_desc(&tmB.m[i]);
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
        const GpTile ti = sched.tile(t);
        const GpSplit sp2(ti.n_valid);
        const int h1 = sp2.m1 / 2, h2 = sp2.m2 / 2;
        const int bi1 = box_index(h1), bi2 = box_index(h2 > 0 ? h2 : 1);
        const uint32_t bytes =
            2u * (L::kABytes + (16u << bi1) * kBK * 2 + (h2 > 0 ? (16u << bi2) * kBK * 2 : 0u));
        const int a_row = ti.a_row + static_cast<int>(rank) * ti.a_rank_stride;
        const int b1 = ti.b_row + static_cast<int>(rank) * h1;
        const int b2 = ti.b_row + sp2.m1 + static_cast<int>(rank) * h2;
        for (int kb = 0; kb < ti.nkb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, kSiteProdEmpty)) {
            ok = false;
            break;
          }
          if (leader) mbar_arrive_expect_tx(&full[stage], bytes);
          uint8_t* st = smem + stage * L::kStageBytes;
          const uint32_t bar = full_lead + 8u * stage;
#pragma unroll
          for (int b = 0; b < ABOXES; ++b)
            tma_load_2d_pair(st + b * L::kABoxRows * kBK * 2, &tmA, bar, kb * kBK, a_row + b * ti.a_box_stride, pol);
          tma_load_2d_pair(st + L::kABytes, &tmB.m[bi1], bar, kb * kBK, b1, pol);
          if (h2 > 0) tma_load_2d_pair(st + L::kABytes + L::kBRegion, &tmB.m[bi2], bar, kb * kBK, b2, pol);
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
      uint32_t ph = 0;   // bit s: parity of the number of tiles that used slot s so far
      int next = 0;
      bool issued = false, ok = true;
      for (int t = pair; ok && t < ntiles; t += npairs) {
        const GpTile ti = sched.tile(t);
        const GpSplit sp2(ti.n_valid);
        const int sa = next, sb = next ^ 1;
        const bool two = sp2.m2 > 0;
        if (!mbar_wait(&tempty[sa], ((ph >> sa) & 1u) ^ 1u, abort_flag, kSiteMmaTmemEmpty)) break;
        if (two && !mbar_wait(&tempty[sb], ((ph >> sb) & 1u) ^ 1u, abort_flag, kSiteMmaTmemEmpty)) break;
        tc_fence_after();
        const uint32_t da = tmem_base + sa * kGpSlotCols, db = tmem_base + sb * kGpSlotCols;
        const uint32_t id1 = idesc_bf16_f32(256, sp2.m1);
        const uint32_t id2 = idesc_bf16_f32(256, two ? sp2.m2 : 16);
        for (int kb = 0; kb < ti.nkb; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag, kSiteMmaFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem + stage * L::kStageBytes);
          const uint32_t b1_addr = a_addr + L::kABytes, b2_addr = b1_addr + L::kBRegion;
#pragma unroll
          for (int kk = 0; kk < kBK / kUmmaK; ++kk) {
            const uint64_t adesc = sdesc_sw128_kmajor(a_addr + kk * kUmmaK * 2);
            const uint32_t acc = (kb | kk) != 0;
            mma_bf16_pair(da, adesc, sdesc_sw128_kmajor(b1_addr + kk * kUmmaK * 2), id1, acc);
            if (two) mma_bf16_pair(db, adesc, sdesc_sw128_kmajor(b2_addr + kk * kUmmaK * 2), id2, acc);
          }
          mma_commit_pair(&empty[stage], 0x3);
          issued = true;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        mma_commit_pair(&tfull[sa], 0x3);
        ph ^= 1u << sa;
        if (two) {
          mma_commit_pair(&tfull[sb], 0x3);
          ph ^= 1u << sb;
        } else {
          next ^= 1;
        }
      }
      if (issued) {
        mma_commit_pair(drain, 0x1);
        mbar_wait_drain(drain, 0, kSiteDrainMma);
      }
    }
  } else {
    // -------------------------------------------------------------------- epilogue (both CTAs)
    const int quad = warp & 3;   // TMEM lanes [32*quad, 32*quad + 32)
    const int grp = (warp - 2) >> 2;
    uint8_t* gsmem = epi_smem + grp * Epi::kSmemBytes;
    uint32_t ph = 0;   // as in the MMA issuer
    int next = 0;
    uint32_t chunk_seq = 0;
    bool live = true;
    Epi::init_smem(gsmem, quad * 32 + static_cast<int>(lane));
    epi_bar_sync(grp);
    for (int t = pair; live && t < ntiles; t += npairs) {
      const GpTile ti = sched.tile(t);
      const GpSplit sp2(ti.n_valid);
      const int nslots = sp2.m2 > 0 ? 2 : 1;
      int done_tok0[2] = {0, 0}, done_ncols[2] = {0, 0};
      for (int k = 0; k < nslots; ++k) {
        const int s = k == 0 ? next : next ^ 1;
        const bool ok = mbar_wait(&tfull[s], (ph >> s) & 1u, abort_flag, kSiteEpiTmemFull);
        if (!epi_vote_all(ok, grp)) {
          live = false;
          break;
        }
        tc_fence_after();
        const int tok0 = k == 0 ? 0 : sp2.m1;
        const int ncols = min(ti.n_valid - tok0, k == 0 ? sp2.m1 : sp2.m2);
        const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + s * kGpSlotCols;
        Epi::run(ep, ti, quad, static_cast<int>(lane), static_cast<int>(rank), grp, taddr, tok0, ncols, gsmem,
                 chunk_seq);
        tc_fence_before();
        if (leader) mbar_arrive(&tempty[s]);
        else mbar_arrive_cluster(tempty_lead + 8u * s);
        done_tok0[k] = tok0;
        done_ncols[k] = ncols;
        ph ^= 1u << s;
      }
      if (nslots == 1) next ^= 1;
      // work that needs no accumulator, once every slot of the tile is back with the MMA
      if (live)
        for (int k = 0; k < nslots; ++k)
          Epi::after_release(ep, ti, quad, static_cast<int>(lane), static_cast<int>(rank), grp, gsmem, done_tok0[k],
                             done_ncols[k]);
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

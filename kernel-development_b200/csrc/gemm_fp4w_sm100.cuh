// gemm_fp4w_sm100.cuh — grouped expert GEMM with NVFP4 weights dequantised in shared memory (w4a16).
//
// The weights stream from HBM as NVFP4 (E2M1 codes, one E4M3 scale per 16 elements; 4.5 bits per weight)
// and become tcgen05 operands only in shared memory:
//   producer (warp 0, one thread): one bulk copy per raw stage of two k chunks; prepare() stores, for each
//       weight tile (two 128-row parts) and 64-element k chunk, both parts' codes (2 x 4 KB) and scales
//       (2 x 512 B) contiguously and the chunks of a tile one after another, because each TMA operation
//       carries a fixed cost that dominated when a chunk took four small copies;
//   converter (warps 6-9): e2m1 x e4m3 -> f16 (cvt.rn.f16x2.e2m1x2, then one f16x2 multiply: both exact,
//       the product has at most 6 significant bits) into the 128-byte-swizzled K-major layout the MMA
//       reads; thread 0 also loads the stage's token rows (f16) with TMA;
//   MMA issuer (warp 1, one thread): M = 128 token rows (<= 64 real; the rest of the A tile is whatever
//       follows in shared memory and lands in TMEM lanes nobody reads) x N = 256 weight rows (both parts)
//       x K = 16 f16 MMAs into TMEM, double-buffered accumulators;
//   epilogue (warps 2-3 hold the token lanes): per-group global scale and the layer's output conversion
//       (Epi), one token row per thread, contiguous feature stores.
// Tokens as M and weights as N: 256 weight rows per instruction, half the MMA instructions per weight byte
// of a 128-row weight operand, and contiguous output rows in the epilogue.
// Tokens are f16 because a kind::f16 MMA takes both operands in one type: the bf16 activations convert to
// f16 exactly within f16's range (their 8 significant bits fit in 11), so the products are those of the
// bf16 computation.  Why not tcgen05's block-scaled MMA: it scales fp4/fp6/fp8 operands only, and w4a16
// keeps the activations in 16 bits.
//
// Signalling (all waits bounded): raw_full (TMA tx), raw_empty (converter), conv_full (converter's
// expect-tx for the tokens + its arrival after the weights are written and fenced for the async proxy),
// conv_empty (MMA commit), tfull / tempty (accumulators).  The converter warps vote after each wait so
// their named barrier is reached by all four or none.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include "gemm_sm100.cuh"
#include "gemm_swap_sm100.cuh"
#include "host_util.h"

namespace kdb {

constexpr int kFp4Threads = 320;       // warp 0 producer, 1 MMA, 2-5 epilogue, 6-9 converter
constexpr int kFp4Block = 4096;        // codes of one 128-row x 64-element weight part
constexpr int kFp4ScaleBlock = 512;    // its E4M3 scales (4 per row)
constexpr int kFp4Chunk = 2 * kFp4Block + 2 * kFp4ScaleBlock;   // one k chunk of a weight tile: 9 KB
constexpr int kFp4RawChunks = 2;       // k chunks per raw stage (one bulk copy)
constexpr int kFp4NB = 64;             // tokens per tile at most
constexpr unsigned int kSiteFp4Conv = 0x120;

// One tile: weight tile f (two 128-row parts) of expert `group` times <= 64 token rows.
struct Fp4Tile {
  int group, f, b_row, n_valid, f0;
};

template <int RSTAGES, int CSTAGES>
struct Fp4Layout {
  // conv stage: token rows (A, 64 rows = 8 KB; the MMA reads 128 rows, the upper 64 from the weight part
  // that follows) then the two 128-row weight parts (B, 256 rows x 64 f16 = 32 KB)
  static constexpr int kTokBytes = kFp4NB * kBK * 2;
  static constexpr int kWPart = 128 * kBK * 2;
  static constexpr int kConvStage = kTokBytes + 2 * kWPart;    // 40 KB, 1024-aligned
  static constexpr int kRawStage = kFp4RawChunks * kFp4Chunk;
  static constexpr int kRawOffset = CSTAGES * kConvStage;
  static constexpr int kBarOffset = kRawOffset + RSTAGES * kRawStage;
  static constexpr int kBarBytes = (2 * RSTAGES + 2 * CSTAGES + 5) * 8 + 16;
  static constexpr int kSmemBytes = kBarOffset + kBarBytes + 1024;
  static constexpr uint32_t kTmemCols = 512;                   // 2 accumulators x 256 weight columns
};

__host__ __device__ constexpr uint32_t idesc_f16_f32(int m, int n) {
  return (1u << 4)                                   // D format: f32 (A, B format 0: f16)
         | (static_cast<uint32_t>(n >> 3) << 17)     // N / 8
         | (static_cast<uint32_t>(m >> 4) << 24);    // M / 16
}

// Bulk (non-tensor) copy global -> this CTA's shared memory, completing `bytes` on `bar`.  Both addresses
// 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_load(void* smem_dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(smem_dst)),
               "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// All 128 converter threads agree on `ok` (named barrier 5).
__device__ __forceinline__ bool conv_vote_all(bool ok) {
  uint32_t bad = ok ? 0u : 1u, any;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.or.pred q, 5, 128, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(any)
      : "r"(bad)
      : "memory");
  return any == 0u;
}

__device__ __forceinline__ void conv_bar_sync() { asm volatile("bar.sync 6, 128;" ::: "memory"); }

// Eight E2M1 codes (one 32-bit word, element 0 in the low nibble) times one f16 scale -> four f16x2.
__device__ __forceinline__ uint4 dequant8(uint32_t word, uint32_t scale2) {
  uint32_t h0, h1, h2, h3;
  asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
      "mov.b32 {b0, b1, b2, b3}, %4;\n\t"
      "cvt.rn.f16x2.e2m1x2 %0, b0;\n\t"
      "cvt.rn.f16x2.e2m1x2 %1, b1;\n\t"
      "cvt.rn.f16x2.e2m1x2 %2, b2;\n\t"
      "cvt.rn.f16x2.e2m1x2 %3, b3;\n\t}"
      : "=r"(h0), "=r"(h1), "=r"(h2), "=r"(h3)
      : "r"(word));
  uint4 out;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(out.x) : "r"(h0), "r"(scale2));
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(out.y) : "r"(h1), "r"(scale2));
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(out.z) : "r"(h2), "r"(scale2));
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(out.w) : "r"(h3), "r"(scale2));
  return out;
}

// E4M3 byte -> {s, s} as f16x2.
__device__ __forceinline__ uint32_t e4m3_to_f16x2(uint32_t byte) {
  uint32_t pair;
  const uint16_t two = static_cast<uint16_t>(byte | (byte << 8));
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(pair) : "h"(two));
  return pair;
}

template <class Sched, class Epi, int RSTAGES, int CSTAGES>
__global__ void __launch_bounds__(kFp4Threads, 1)
    gemm_fp4w_kernel(const __grid_constant__ TokenMaps tmB, const uint8_t* __restrict__ blocks,
                     const typename Sched::Params sp, const typename Epi::Params ep) {
  using L = Fp4Layout<RSTAGES, CSTAGES>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* raw = smem + L::kRawOffset;
  uint64_t* raw_full = reinterpret_cast<uint64_t*>(smem + L::kBarOffset);
  uint64_t* raw_empty = raw_full + RSTAGES;
  uint64_t* conv_full = raw_empty + RSTAGES;
  uint64_t* conv_empty = conv_full + CSTAGES;
  uint64_t* tfull = conv_empty + CSTAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = warp_id_uniform();
  const uint32_t lane = lane_id();

  if (threadIdx.x == 0) {
    for (int s = 0; s < RSTAGES; ++s) {
      mbar_init(&raw_full[s], 1);
      mbar_init(&raw_empty[s], 1);
    }
    for (int s = 0; s < CSTAGES; ++s) {
      mbar_init(&conv_full[s], 2);    // converter: expect-tx arrival for the tokens + arrival after writing
      mbar_init(&conv_empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 128);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
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
  const int nkb = sp.nkb;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------------ weight producer
      uint32_t stage = 0, phase = 0, armed_mask = 0, armed_phase = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < ntiles; t += gridDim.x) {
        const Fp4Tile ti = sched.tile(t);
        const uint8_t* tile_src = blocks + (static_cast<long long>(ti.group) * sp.f_tiles + ti.f) * nkb * kFp4Chunk;
        for (int kb = 0; kb < nkb; kb += kFp4RawChunks) {
          const int nc = min(kFp4RawChunks, nkb - kb);
          if (!mbar_wait(&raw_empty[stage], phase ^ 1u, abort_flag, kSiteProdEmpty)) {
            ok = false;
            break;
          }
          uint8_t* st = raw + stage * L::kRawStage;
          mbar_arrive_expect_tx(&raw_full[stage], nc * kFp4Chunk);
          bulk_load(st, tile_src + static_cast<long long>(kb) * kFp4Chunk, nc * kFp4Chunk, &raw_full[stage]);
          armed_mask |= 1u << stage;
          armed_phase = (armed_phase & ~(1u << stage)) | (phase << stage);
          if (++stage == RSTAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      for (int s = 0; s < RSTAGES; ++s)
        if (armed_mask & (1u << s)) mbar_wait_drain(&raw_full[s], (armed_phase >> s) & 1u, kSiteDrainTma);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------------------------ MMA issuer
      uint32_t stage = 0, phase = 0;
      bool issued = false, ok = true;
      int it = 0;
      for (int t = blockIdx.x; ok && t < ntiles; t += gridDim.x, ++it) {
        const Fp4Tile ti = sched.tile(t);
        constexpr uint32_t idesc = idesc_f16_f32(128, 256);
        const uint32_t acc = it & 1, aph = (it >> 1) & 1;
        if (!mbar_wait(&tempty[acc], aph ^ 1u, abort_flag, kSiteMmaTmemEmpty)) break;
        tc_fence_after();
        const uint32_t d_base = tmem_base + acc * 256;
        for (int kb = 0; kb < nkb; ++kb) {
          if (!mbar_wait(&conv_full[stage], phase, abort_flag, kSiteMmaFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem + stage * L::kConvStage);   // token rows
          const uint32_t b_addr = a_addr + L::kTokBytes;                      // 256 weight rows
#pragma unroll
          for (int kk = 0; kk < kBK / kUmmaK; ++kk)
            mma_bf16(d_base, sdesc_sw128_kmajor(a_addr + kk * kUmmaK * 2), sdesc_sw128_kmajor(b_addr + kk * kUmmaK * 2),
                     idesc, (kb | kk) != 0);
          mma_commit(&conv_empty[stage]);
          issued = true;
          if (++stage == CSTAGES) {
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
  } else if (warp >= 6) {
    // -------------------------------------------------------------------- converter (128 threads)
    const int ct = threadIdx.x - 192;   // weight row of both parts this thread converts
    uint32_t rstage = 0, rphase = 0, cstage = 0, cphase = 0;
    bool live = true, armed = false;
    uint32_t armed_stage = 0, armed_ph = 0;
    for (int t = blockIdx.x; live && t < ntiles; t += gridDim.x) {
      const Fp4Tile ti = sched.tile(t);
      const int bi = box_index(ti.n_valid);
      for (int kb = 0; live && kb < nkb; kb += kFp4RawChunks) {
        const int nc = min(kFp4RawChunks, nkb - kb);
        bool ok = mbar_wait(&raw_full[rstage], rphase, abort_flag, kSiteFp4Conv);
        const uint8_t* rst = raw + rstage * L::kRawStage;
        for (int c = 0; c < nc; ++c) {
          ok = ok && mbar_wait(&conv_empty[cstage], cphase ^ 1u, abort_flag, kSiteFp4Conv);
          if (!conv_vote_all(ok)) {
            live = false;
            break;
          }
          uint8_t* cst = smem + cstage * L::kConvStage;
          if (ct == 0) {
            mbar_arrive_expect_tx(&conv_full[cstage], (16u << bi) * kBK * 2);
            tma_load_2d(cst, &tmB.m[bi], &conv_full[cstage], (kb + c) * kBK, ti.b_row, l2_policy_evict_normal());
            armed = true;
            armed_stage = cstage;
            armed_ph = cphase;
          }
          const uint8_t* rch = rst + c * kFp4Chunk;
#pragma unroll
          for (int a = 0; a < 2; ++a) {
            const uint4* crow = reinterpret_cast<const uint4*>(rch + a * kFp4Block + ct * 32);
            const uint4 c0 = crow[0], c1 = crow[1];
            const uint32_t sc = *reinterpret_cast<const uint32_t*>(rch + 2 * kFp4Block + a * kFp4ScaleBlock + ct * 4);
            const uint32_t words[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
            uint8_t* drow = cst + L::kTokBytes + a * L::kWPart + ct * 128;
#pragma unroll
            for (int j = 0; j < 8; ++j) {   // 16-byte chunk j = elements 8j..8j+7, scale j / 2
              const uint32_t s2 = e4m3_to_f16x2((sc >> (8 * (j >> 1))) & 0xffu);
              *reinterpret_cast<uint4*>(drow + ((j ^ (ct & 7)) << 4)) = dequant8(words[j], s2);
            }
          }
          fence_proxy_async_smem();
          conv_bar_sync();
          if (ct == 0) mbar_arrive(&conv_full[cstage]);
          if (++cstage == CSTAGES) {
            cstage = 0;
            cphase ^= 1u;
          }
        }
        if (!live) break;
        if (ct == 0) mbar_arrive(&raw_empty[rstage]);
        if (++rstage == RSTAGES) {
          rstage = 0;
          rphase ^= 1u;
        }
      }
    }
    // the token copy of the last armed stage must land before this CTA may leave (already complete
    // unless the MMA side gave up before consuming it)
    if (ct == 0 && armed) mbar_wait_drain(&conv_full[armed_stage], armed_ph, kSiteDrainTma);
  } else {
    // -------------------------------------------------------------------- epilogue (128 threads)
    const int quad = warp & 3;   // TMEM lanes = token rows 32 * quad .. + 31 (only quads 0, 1 hold tokens)
    int it = 0;
    for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ++it) {
      const uint32_t acc = it & 1, aph = (it >> 1) & 1;
      const bool ok = mbar_wait(&tfull[acc], aph, abort_flag, kSiteEpiTmemFull);
      if (!__all_sync(0xffffffffu, ok)) break;
      tc_fence_after();
      const Fp4Tile ti = sched.tile(t);
      if (quad * 32 < ti.n_valid) {
        const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + acc * 256;
        Epi::run(ep, ti, quad * 32 + static_cast<int>(lane), taddr);
      }
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

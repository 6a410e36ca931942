// gemm_fp4w_sm100.cuh — grouped expert GEMM with NVFP4 weights dequantised on chip into TMEM (w4a16).
//
// The weights stream from HBM as NVFP4 (E2M1 codes, one E4M3 scale per 16 elements; 4.5 bits per weight)
// and become f16 tcgen05 operands only on chip:
//   producer (warp 0, one thread): per raw stage of two k chunks, one bulk copy of their NVFP4 blocks and
//       one TMA copy per chunk of the tile's token rows (f16), all completing on the stage's barrier, so a
//       chunk's tokens arrive RSTAGES stages ahead together with its weights.  prepare() stores, for each
//       weight tile (two 128-row parts) and 64-element k chunk, both parts' codes (2 x 4 KB) and scales
//       (2 x 512 B) contiguously and the chunks of a tile one after another, because each TMA operation
//       carries a fixed cost that dominated when a chunk took four small copies.  (The tokens were once
//       loaded by the converter at the start of each chunk; the MMA then waited ~1.5 us on every chunk's
//       token copy with only CSTAGES chunks of slack, which capped each SM at ~16 GB/s of NVFP4.)
//   converter (warps 6-9): e2m1 x e4m3 -> f16 (cvt.rn.f16x2.e2m1x2, then one f16x2 multiply: both exact,
//       the product has at most 6 significant bits) written straight into TMEM with tcgen05.st (lane =
//       weight row, two k elements per 32-bit column), where the MMA takes its A operand.  Staging the f16
//       weights in TMEM keeps them out of shared memory, whose bandwidth (32 KB of f16 written and read per
//       9 KB of NVFP4) bounded the version that converted into a swizzled shared-memory tile;
//   MMA issuer (warp 1, one thread): A = 128 weight rows of each part from TMEM, B = the tile's tokens
//       (N = tokens rounded up to 16) from shared memory, K = 16 per instruction, double-buffered
//       accumulators (2 parts x 64 token columns each);
//   epilogue (warps 2-5): per-group global scale and the layer's output conversion (Epi), TMEM lane =
//       output feature, one token per column.
// Tokens are f16 because a kind::f16 MMA takes both operands in one type: the bf16 activations convert to
// f16 exactly within f16's range (their 8 significant bits fit in 11), so the products are those of the
// bf16 computation.  Why not tcgen05's block-scaled MMA: it scales fp4/fp6/fp8 operands only, and w4a16
// keeps the activations in 16 bits.
//
// Signalling (all waits bounded): raw_full (TMA tx of weights and tokens), raw_empty (two arrivals: the
// converter once it has read the stage's weights, the MMA commit once the MMAs reading its tokens are done),
// conv_full (the converter's arrival after its tcgen05.st of the weights completed and was fenced),
// conv_empty (MMA commit), tfull / tempty (accumulators).  The converter warps vote after each wait so their
// named barrier is reached by all four or none.
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
  static constexpr int kTokBytes = kFp4NB * kBK * 2;           // one chunk's token rows (B, 64 x 64 f16 = 8 KB)
  static constexpr int kRawWeights = kFp4RawChunks * kFp4Chunk;   // a raw stage: the NVFP4 blocks of two chunks,
  static constexpr int kRawStage = kRawWeights + kFp4RawChunks * kTokBytes;   // then their token rows
  static constexpr int kRawOffset = 0;
  static constexpr int kBarOffset = kRawOffset + RSTAGES * kRawStage;
  static constexpr int kBarBytes = (2 * RSTAGES + 2 * CSTAGES + 5) * 8 + 16;
  static constexpr int kSmemBytes = kBarOffset + kBarBytes + 1024;
  // TMEM: accumulators [0, 256) = 2 buffers x 2 weight parts x 64 token columns; then CSTAGES stages of the
  // dequantised weights, 2 parts x 32 columns (64 f16 of K packed two per 32-bit column) each
  static constexpr uint32_t kAccCols = 2 * kFp4NB;
  static constexpr uint32_t kACol0 = 2 * kAccCols;
  static constexpr uint32_t kTmemCols = 512;
  static_assert(kACol0 + CSTAGES * 64 <= kTmemCols, "TMEM holds the accumulators and the weight stages");
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

// 32 consecutive 32-bit TMEM columns of this warp's 32 lanes (lane i: v[0..31] of lane i).
__device__ __forceinline__ void tmem_st_32x32b_x32(uint32_t taddr, const uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
      "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]), "r"(v[17]), "r"(v[18]),
      "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]),
      "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
      : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem]: A is M = 128 lanes x K = 16 (eight 32-bit columns of packed f16 pairs).
__device__ __forceinline__ void mma_f16_tmem_a(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                               uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
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
      mbar_init(&raw_empty[s], 2);    // converter (weights read) + MMA commit (tokens read)
    }
    for (int s = 0; s < CSTAGES; ++s) {
      mbar_init(&conv_full[s], 1);
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
      const uint64_t pol_t = l2_policy_evict_normal();
      for (int t = blockIdx.x; ok && t < ntiles; t += gridDim.x) {
        const Fp4Tile ti = sched.tile(t);
        const uint8_t* tile_src = blocks + (static_cast<long long>(ti.group) * sp.f_tiles + ti.f) * nkb * kFp4Chunk;
        const int bi = box_index(ti.n_valid);
        const uint32_t tok_bytes = (16u << bi) * kBK * 2;
        for (int kb = 0; kb < nkb; kb += kFp4RawChunks) {
          const int nc = min(kFp4RawChunks, nkb - kb);
          if (!mbar_wait(&raw_empty[stage], phase ^ 1u, abort_flag, kSiteProdEmpty)) {
            ok = false;
            break;
          }
          uint8_t* st = raw + stage * L::kRawStage;
          mbar_arrive_expect_tx(&raw_full[stage], nc * (kFp4Chunk + tok_bytes));
          bulk_load(st, tile_src + static_cast<long long>(kb) * kFp4Chunk, nc * kFp4Chunk, &raw_full[stage]);
          for (int c = 0; c < nc; ++c)
            tma_load_2d(st + L::kRawWeights + c * L::kTokBytes, &tmB.m[bi], &raw_full[stage], (kb + c) * kBK, ti.b_row,
                        pol_t);
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
      uint32_t stage = 0, phase = 0, rstage = 0, rphase = 0;
      bool issued = false, ok = true;
      int it = 0;
      for (int t = blockIdx.x; ok && t < ntiles; t += gridDim.x, ++it) {
        const Fp4Tile ti = sched.tile(t);
        const uint32_t idesc = idesc_f16_f32(128, (ti.n_valid + 15) & ~15);
        const uint32_t acc = it & 1, aph = (it >> 1) & 1;
        if (!mbar_wait(&tempty[acc], aph ^ 1u, abort_flag, kSiteMmaTmemEmpty)) break;
        tc_fence_after();
        const uint32_t d_base = tmem_base + acc * L::kAccCols;
        for (int kb = 0; kb < nkb; ++kb) {
          const int c = kb % kFp4RawChunks;   // chunk within its raw stage (tiles start on a stage boundary)
          if (!mbar_wait(&conv_full[stage], phase, abort_flag, kSiteMmaFull) ||
              (c == 0 && !mbar_wait(&raw_full[rstage], rphase, abort_flag, kSiteMmaFull))) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t b_addr = smem_u32(raw + rstage * L::kRawStage + L::kRawWeights + c * L::kTokBytes);
          const uint32_t a_col = tmem_base + L::kACol0 + stage * 64;                  // weight parts
#pragma unroll
          for (int kk = 0; kk < kBK / kUmmaK; ++kk) {
            const uint64_t bdesc = sdesc_sw128_kmajor(b_addr + kk * kUmmaK * 2);
#pragma unroll
            for (int a = 0; a < 2; ++a)
              mma_f16_tmem_a(d_base + a * kFp4NB, a_col + a * 32 + kk * 8, bdesc, idesc, (kb | kk) != 0);
          }
          mma_commit(&conv_empty[stage]);
          issued = true;
          if (++stage == CSTAGES) {
            stage = 0;
            phase ^= 1u;
          }
          if (c == kFp4RawChunks - 1 || kb == nkb - 1) {   // the stage's tokens are read once these MMAs finish
            mma_commit(&raw_empty[rstage]);
            if (++rstage == RSTAGES) {
              rstage = 0;
              rphase ^= 1u;
            }
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
    const int ct = threadIdx.x - 192;
    const int wrow = (warp & 3) * 32 + static_cast<int>(lane);   // weight row (= TMEM lane) this thread converts
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
    uint32_t rstage = 0, rphase = 0, cstage = 0, cphase = 0;
    bool live = true;
    for (int t = blockIdx.x; live && t < ntiles; t += gridDim.x) {
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
          tc_fence_after();   // the MMAs that read this TMEM stage completed (conv_empty) before it is rewritten
          const uint8_t* rch = rst + c * kFp4Chunk;
#pragma unroll
          for (int a = 0; a < 2; ++a) {
            const uint4* crow = reinterpret_cast<const uint4*>(rch + a * kFp4Block + wrow * 32);
            const uint4 c0 = crow[0], c1 = crow[1];
            const uint32_t sc = *reinterpret_cast<const uint32_t*>(rch + 2 * kFp4Block + a * kFp4ScaleBlock + wrow * 4);
            const uint32_t words[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
            uint32_t v[32];   // 64 f16 of this row's chunk, k pairs packed per 32-bit column
#pragma unroll
            for (int j = 0; j < 8; ++j) {   // elements 8j..8j+7, scale j / 2
              const uint4 q = dequant8(words[j], e4m3_to_f16x2((sc >> (8 * (j >> 1))) & 0xffu));
              v[4 * j] = q.x;
              v[4 * j + 1] = q.y;
              v[4 * j + 2] = q.z;
              v[4 * j + 3] = q.w;
            }
            tmem_st_32x32b_x32(tmem_base + lane_off + L::kACol0 + cstage * 64 + a * 32, v);
          }
          tmem_st_wait();
          tc_fence_before();
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
  } else {
    // -------------------------------------------------------------------- epilogue (128 threads)
    const int quad = warp & 3;   // TMEM lanes = weight rows 32 * quad .. + 31 of both parts
    int it = 0;
    for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ++it) {
      const uint32_t acc = it & 1, aph = (it >> 1) & 1;
      const bool ok = mbar_wait(&tfull[acc], aph, abort_flag, kSiteEpiTmemFull);
      if (!__all_sync(0xffffffffu, ok)) break;
      tc_fence_after();
      const Fp4Tile ti = sched.tile(t);
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + acc * L::kAccCols;
      Epi::run(ep, ti, quad * 32 + static_cast<int>(lane), taddr);
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

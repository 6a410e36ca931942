// moe_ep.cu — device pieces of the expert-parallel MoE layer.
//
// With experts split over P ranks (rank r owns the Er = E/P experts [r*Er, (r+1)*Er)), a rank's
// routed rows, grouped by expert, are already grouped by owner rank, so one all-to-all moves them.
// What arrives at an owner is source-major: blocks (source s, local expert e), expert-minor.  The
// grouped GEMMs want expert-major rows, so the owner regroups them (and ungroups the results before
// they travel back).  Both directions are a block transpose of a P x Er table of row counts:
//
//   source-major offset of block (s, e):  so[s][e] = sum_{s' < s} sum_e' c[s'][e'] + sum_{e' < e} c[s][e']
//   expert-major offset of block (s, e):  eo[s][e] = sum_{e' < e} sum_s' c[s'][e'] + sum_{s' < s} c[s'][e]
//
// The regroup also writes the expert-major offsets[Er + 1] and the tile prefix mtile_start[Er + 1]
// (exclusive prefix of ceil(rows / kMoeTokenTile)) that the grouped GEMM schedule reads.  Counts stay on the device: nothing here synchronises.
//
// No counterpart kernel in the reference: its engines simulate one ep8 rank and compute only the
// routes to local experts (okc_problems/muse_moe_w4a16.toml:136); the exchange is new.
#include "host_util.h"
#include "moe.h"
#include "sm100_common.cuh"

namespace kdb {

// One CTA (Er <= 1024 threads): so/eo tables ([P][Er] each), offsets, mtile_start.
__global__ void __launch_bounds__(1024)
    moe_ep_table_kernel(const int* __restrict__ counts, int P, int Er, int* __restrict__ so, int* __restrict__ eo,
                        int* __restrict__ offsets, int* __restrict__ mtile_start) {
  __shared__ int warp_sum[32];
  __shared__ int carry;
  const int e = threadIdx.x;
  const int lane = e & 31, w = e >> 5, nw = (blockDim.x + 31) >> 5;

  // block-wide exclusive scan of v over threads, returns (exclusive prefix, total)
  auto scan = [&](int v, int* total) -> int {
    int x = v;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, x, off);
      if (lane >= off) x += y;
    }
    if (lane == 31) warp_sum[w] = x;
    __syncthreads();
    if (w == 0) {
      int ws = lane < nw ? warp_sum[lane] : 0;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, ws, off);
        if (lane >= off) ws += y;
      }
      warp_sum[lane] = ws;
    }
    __syncthreads();
    const int incl = x + (w > 0 ? warp_sum[w - 1] : 0);
    *total = warp_sum[nw - 1];
    __syncthreads();
    return incl - v;
  };

  // expert-major: column totals, their exclusive scan, then source prefix within each column
  int col = 0;
  if (e < Er)
    for (int s = 0; s < P; ++s) col += counts[s * Er + e];
  const int mt = (col + kMoeTokenTile - 1) / kMoeTokenTile;
  int total_rows = 0, total_mt = 0;
  const int ebase = scan(e < Er ? col : 0, &total_rows);
  const int mbase = scan(e < Er ? mt : 0, &total_mt);
  if (e < Er) {
    offsets[e] = ebase;
    mtile_start[e] = mbase;
    int run = ebase;
    for (int s = 0; s < P; ++s) {
      eo[s * Er + e] = run;
      run += counts[s * Er + e];
    }
  }
  if (e == 0) {
    offsets[Er] = total_rows;
    mtile_start[Er] = total_mt;
    carry = 0;
  }
  __syncthreads();
  // source-major: for each source row of the table, a scan over experts
  for (int s = 0; s < P; ++s) {
    int row_total = 0;
    const int c = e < Er ? counts[s * Er + e] : 0;
    const int pre = scan(c, &row_total);
    if (e < Er) so[s * Er + e] = carry + pre;
    __syncthreads();
    if (e == 0) carry += row_total;
    __syncthreads();
  }
}

// grid (P * Er, chunks): block (s, e) copies its rows; one warp per row, 16-byte vectors.
__global__ void __launch_bounds__(256)
    moe_ep_copy_kernel(const int* __restrict__ counts, const int* __restrict__ so, const int* __restrict__ eo,
                       int to_expert_major, const __nv_bfloat16* __restrict__ in, __nv_bfloat16* __restrict__ out,
                       int H) {
  const int b = blockIdx.x;
  const int n = counts[b];
  const int src0 = to_expert_major ? so[b] : eo[b];
  const int dst0 = to_expert_major ? eo[b] : so[b];
  const int warps = blockDim.x >> 5, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int vec = H / 8;
  for (int r = blockIdx.y * warps + warp; r < n; r += gridDim.y * warps) {
    const uint4* s = reinterpret_cast<const uint4*>(in + static_cast<long long>(src0 + r) * H);
    uint4* d = reinterpret_cast<uint4*>(out + static_cast<long long>(dst0 + r) * H);
    for (int v = lane; v < vec; v += 32) d[v] = __ldg(s + v);
  }
}

size_t moe_ep_regroup_scratch_bytes(int P, int Er) {
  const size_t one = (static_cast<size_t>(P) * Er * sizeof(int) + 255) / 256 * 256;
  return 2 * one;
}

int moe_ep_regroup(const int* counts, int P, int Er, int to_expert_major, const void* in, void* out, int H,
                   int* offsets, int* mtile_start, void* scratch, cudaStream_t s) {
  const size_t one = moe_ep_regroup_scratch_bytes(P, Er) / 2;
  int* so = static_cast<int*>(scratch);
  int* eo = reinterpret_cast<int*>(static_cast<char*>(scratch) + one);
  moe_ep_table_kernel<<<1, ((Er + 31) / 32) * 32, 0, s>>>(counts, P, Er, so, eo, offsets, mtile_start);
  int rc = cuda_status(cudaGetLastError());
  if (rc) return rc;
  if (!in || !out) return KDB_OK;   // tables only
  dim3 grid(P * Er, 16);
  moe_ep_copy_kernel<<<grid, 256, 0, s>>>(counts, so, eo, to_expert_major, static_cast<const __nv_bfloat16*>(in),
                                          static_cast<__nv_bfloat16*>(out), H);
  return cuda_status(cudaGetLastError());
}

}  // namespace kdb

// tma_stream.cu — the TMA streaming measurements behind b200.toml's tma_* entries.
//
// One CTA per SM; thread 0 keeps `stages` copies in flight (boxes of 64 bf16 x box_rows rows, `boxes` per
// stage), waiting on the oldest stage's mbarrier before reusing it.  Two modes:
//   hbm: each CTA streams its own 512 rows x 8192 columns (1.24 GB in all; every byte from HBM once);
//   l2:  every CTA streams the same 256 rows x 1024 columns 16 times (L2-resident after the first pass).
// Build and run (one B200):
//   nvcc -gencode arch=compute_100a,code=sm_100a -O3 -std=c++17 --expt-relaxed-constexpr \
//        -I kernel-development_b200/csrc -I include -o tma_stream kernel-development_b200/kdb200/gpus/tma_stream.cu
//   ./tma_stream
// Prints one line per configuration: mode, box rows, boxes per stage, stage KB, stages, GB/s, GB/s per SM.
#include "host_util.cu"
#include "sm100_common.cuh"

#include <algorithm>
#include <cstdio>
#include <vector>

using namespace kdb;

__global__ void __launch_bounds__(32, 1)
    tma_stream_kernel(const __grid_constant__ CUtensorMap tm, int stages, int boxes, int box_rows, int chunks,
                      int rows_per_cta, int shared_rows, int passes) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int stage_bytes = boxes * box_rows * 128;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + stages * stage_bytes);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + stages);
  if (threadIdx.x != 0) return;
  for (int s = 0; s < stages; ++s) mbar_init(&bars[s], 1);
  *abort_flag = 0;
  fence_mbar_init();
  tma_prefetch_desc(&tm);
  const uint64_t pol = l2_policy_evict_normal();
  const int row0 = shared_rows ? 0 : blockIdx.x * rows_per_cta;
  const int rowblocks = rows_per_cta / (boxes * box_rows);
  const int per_pass = rowblocks * chunks;
  const int total = passes * per_pass;
  for (int i = 0; i < total + stages; ++i) {
    const int s = i % stages;
    if (i >= stages && !mbar_wait(&bars[s], static_cast<uint32_t>((i / stages) - 1) & 1u, abort_flag, 0x901)) return;
    if (i < total) {
      const int j = i % per_pass;
      const int rb = j / chunks, k = j % chunks;
      mbar_arrive_expect_tx(&bars[s], stage_bytes);
      for (int b = 0; b < boxes; ++b)
        tma_load_2d(smem + s * stage_bytes + b * box_rows * 128, &tm, &bars[s], k * 64,
                    row0 + (rb * boxes + b) * box_rows, pol);
    }
  }
}

static int run_mode(bool l2, void* buf, size_t rows, int sms) {
  const int cols = l2 ? 1024 : 8192, chunks = cols / 64;
  const int rows_per_cta = l2 ? 256 : 512, passes = l2 ? 16 : 1;
  cudaEvent_t a, b;
  cudaEventCreate(&a);
  cudaEventCreate(&b);
  for (int box_rows : {64, 128, 256}) {
    CUtensorMap tm;
    if (make_tmap_bf16_2d(&tm, buf, cols, rows, cols, 64, box_rows)) return 1;
    for (int boxes : {1, 2, 4}) {
      const int stage_bytes = boxes * box_rows * 128;
      if (stage_bytes > 64 * 1024 || boxes * box_rows > rows_per_cta) continue;
      for (int stages : {1, 2, 3, 4, 6, 8, 12}) {
        const int smem = stages * stage_bytes + stages * 8 + 16 + 1024;
        if (smem > 210 * 1024) continue;
        std::vector<float> ts;
        for (int rep = 0; rep < 4; ++rep) {
          cudaEventRecord(a);
          tma_stream_kernel<<<sms, 32, smem>>>(tm, stages, boxes, box_rows, chunks, rows_per_cta, l2 ? 1 : 0, passes);
          cudaEventRecord(b);
          cudaEventSynchronize(b);
          float ms = 0;
          cudaEventElapsedTime(&ms, a, b);
          if (rep) ts.push_back(ms);
        }
        unsigned int st[4] = {0, 0, 0, 0};
        cudaMemcpyFromSymbol(st, g_status, sizeof(st));
        if (cudaGetLastError() != cudaSuccess || st[0]) {
          printf("error: status %u site %u\n", st[0], st[1]);
          return 1;
        }
        std::sort(ts.begin(), ts.end());
        const double bytes = static_cast<double>(sms) * passes * rows_per_cta * cols * 2;
        const double gbs = bytes / (ts[1] * 1e-3) / 1e9;
        printf("%s %d %d %d %d %.0f %.1f\n", l2 ? "l2" : "hbm", box_rows, boxes, stage_bytes / 1024, stages, gbs,
               gbs / sms);
      }
    }
  }
  return 0;
}

int main() {
  const int sms = num_sms();
  const size_t rows = static_cast<size_t>(sms) * 512, cols = 8192;
  void* buf = nullptr;
  if (cudaMalloc(&buf, rows * cols * 2) != cudaSuccess) return 1;
  cudaMemset(buf, 0, rows * cols * 2);
  cudaFuncSetAttribute(tma_stream_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 220 * 1024);
  printf("mode box_rows boxes stage_KB stages GBps GBps_per_SM\n");
  int rc = run_mode(false, buf, rows, sms);
  if (!rc) rc = run_mode(true, buf, rows, sms);
  cudaFree(buf);
  return rc;
}

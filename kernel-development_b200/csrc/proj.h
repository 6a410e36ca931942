// proj.h — internal launcher of the bf16 projection (the C-ABI wrapper lives in capi.cu).
#pragma once
#include <cuda_runtime.h>

namespace kdb {
// Y[M, N] (row stride ldy) = X[M, K] · W[N, K]ᵀ.  force_bn: 0 = pick per shape, else 64/128/192/224/256;
// cta_pair: 1 = 256-row tiles on 2-CTA clusters (widths 192/224/256), 0 = one CTA per 128-row tile.
// Automatic tile shape: width *bn (64..256) and *pair (1 = 256-row tiles on CTA pairs).
void pick_tile(long long M, long long N, long long sms, int* bn, int* pair);

// M <= 128 with automatic shape: weights as the M operand and a K split over a thread-block cluster,
// reduced in distributed shared memory in the same launch.  `workspace` is not used (proj_workspace_bytes
// is 0); the parameters remain for the C ABI's kdb_proj_bf16_ws.
int proj_bf16(const void* x, const void* w, void* y, long long M, long long N, long long K, long long ldy,
              int force_bn, int cta_pair, cudaStream_t stream, void* workspace = nullptr, size_t ws_bytes = 0);
size_t proj_workspace_bytes(long long M, long long N, long long K);

// fp32-weight projection (router layer): w_split = [bf16(W) | bf16(W - bf16(W))] (N x 2K) from
// proj_split_f32; Y fp32 [M, N] contiguous.  K % 64 == 0.
int proj_split_f32(const float* w, void* w_split, long long N, long long K, cudaStream_t stream);
size_t proj_f32w_workspace_bytes(long long M, long long N, long long K);
int proj_f32w(const void* x, const void* w_split, float* y, long long M, long long N, long long K, void* workspace,
              size_t ws_bytes, cudaStream_t stream);
}  // namespace kdb

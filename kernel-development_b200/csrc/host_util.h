// host_util.h — host-side helpers shared by the launchers: TMA tensor-map encoding through the
// driver entry point (no link-time dependency on libcuda), per-device SM counts, argument checks.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cstdint>

#include "kdb_status.h"

namespace kdb {

// Records the last CUDA error seen by a launcher (read with kdb_last_cuda_error()).
void set_cuda_error(cudaError_t e);
int cuda_status(cudaError_t e);   // KDB_OK or KDB_ERR_CUDA (and records e)

// Number of SMs of the current device (cached per device).
// SMs the persistent kernels size their grids for: the device's count, or the process-wide budget when
// one is set (set_sm_budget; 0 = no budget), e.g. to leave SMs to a collective running alongside.
int num_sms();
int set_sm_budget(int sms);   // returns the previous budget
int sm_budget();

// Encodes a 2-D bf16 tensor map over a row-major [rows, inner] matrix with row stride `ld`
// elements, box = [box_rows, box_inner] with the 128-byte swizzle.  Returns KDB_OK or an error.
int make_tmap_bf16_2d(CUtensorMap* map, const void* base, uint64_t inner, uint64_t rows, uint64_t ld,
                      uint32_t box_inner, uint32_t box_rows);

// Five tensor maps over one row-major bf16 [n_rows, k] matrix with boxes of 16, 32, 64, 128 and 256
// rows (64 columns), for operands whose row count varies per tile.
struct TokenMaps {
  CUtensorMap m[5];
};
int make_token_maps(TokenMaps* m, const void* rows, uint64_t n_rows, uint64_t k);

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace kdb

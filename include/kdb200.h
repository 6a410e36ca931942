/*
 * kdb200.h — C ABI of libkdb200.so, the B200 (sm_100a) kernels behind the bf16 projection and the
 * fused Mixture-of-Experts layer.
 *
 * Every entry point takes plain device pointers, sizes in elements, and a cudaStream_t passed as
 * `void*` (NULL = legacy default stream).  Entry points never allocate device memory and never
 * synchronise: scratch comes from a caller-provided workspace, so each call is capturable in a CUDA
 * graph.  They return KDB_OK (0) or one of the KDB_ERR_* codes in kdb_status.h; asynchronous device
 * errors (a bounded wait that timed out, a kernel's own bounds check) land in the device status
 * word read by kdb_status_read().
 *
 * The reference reaches these paths only through its problem-adapter boundary: the submission's
 * `prepare(weights) -> state` and `kernel_fn(data, state) -> out`, called by
 * kdev `OkcAdapter.prepare/call` (src/kdev/adapters/okc.py:501-515, 534-537).  The Python host
 * layer (kernel-development_b200/kdb200) exposes exactly those two functions on top of this ABI.
 */
#ifndef KDB200_H
#define KDB200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define KDB200_ABI_VERSION 1

/* ---------------------------------------------------------------------------------------------- */
/* Library and status                                                                              */
/* ---------------------------------------------------------------------------------------------- */

/* ABI version (KDB200_ABI_VERSION). */
int kdb_abi_version(void);

/* Static string for a KDB_* status code. */
const char* kdb_strerror(int code);

/* The last CUDA error code recorded by a failing entry point on this host thread (0 if none). */
int kdb_last_cuda_error(void);

/*
 * Reads (and, if `clear` != 0, clears) the current device's status word: out[0] = first error code
 * (0 = none), out[1] = site id, out[2] = block index, out[3] = number of reports.  Synchronises the
 * given stream; call it outside timed regions.  Replaces the reference's debug-counter read-back of
 * its bounded spins (okc-challenge/engines/sc_h.cu:75-90), without the trap.
 */
int kdb_status_read(uint32_t out[4], int clear, void* stream);

/* ---------------------------------------------------------------------------------------------- */
/* bf16 dense projection                                                                           */
/* ---------------------------------------------------------------------------------------------- */

/*
 * Y[m, n] = sum_k X[m, k] * W[n, k]   (Y = X · Wᵀ), bf16 inputs, fp32 accumulation, bf16 output
 * rounded to nearest-even.
 *   x: bf16 [m, k] row-major, 16-byte aligned;  w: bf16 [n, k] row-major, 16-byte aligned;
 *   y: bf16 [m, n] with row stride ldy >= n elements (a column slice of a wider matrix is allowed).
 *   k % 8 == 0 (TMA row-stride rule).  m, n, k <= 2^30.  k == 0 writes zeros.
 * Replaces the body of `kernel_fn(data, state)` for the reference's `muse_bf16_proj` problem
 * (src/kdev/adapters/okc.py:534-537; src/kdev/adapters/okc_problems/muse_bf16_proj.toml:1-8).
 */
int kdb_proj_bf16(const void* x, const void* w, void* y, int64_t m, int64_t n, int64_t k, int64_t ldy,
                  void* stream);

/* As kdb_proj_bf16 with the output tile width forced to 64, 128 or 256 (0 = automatic). */
int kdb_proj_bf16_cfg(const void* x, const void* w, void* y, int64_t m, int64_t n, int64_t k, int64_t ldy,
                      int tile_n, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* KDB200_H */

// Allocation-free entry points of the prism_cp_b200 kernel library (C ABI).
//
// This header has no counterpart in the reference framework. It declares the
// one routine of the library that allocates no device memory at all, for
// callers that cannot: a host program that links the library without
// PyTorch's caching allocator, a runtime that forbids cudaMalloc / cudaFree in
// the middle of a step because they synchronise the device, or code that runs
// on a memory budget reserved up front. Such a caller passes every input and
// output buffer; the routine's own working memory (per-block partial sums of
// the weight gradient) is a fixed array compiled into the library.
//
// Contract of prism_rmsnorm_bwd_noalloc:
//   * Computes dx and dw of y = x * rstd * w (RMSNorm), given dy and the
//     forward's per-row reciprocal norms rstd, on `stream`.
//   * dy, x, dx: contiguous bf16 [rows, n]; w: bf16 [n]; rstd: fp32 [rows];
//     dw: fp32 [n] (overwritten). dy, x, w and dx 16-byte aligned; rstd and dw
//     4-byte aligned.
//   * n is a multiple of 8 and at most PRISM_NOALLOC_MAX_N; rows >= 1.
//   * Scratch: PRISM_NOALLOC_SCRATCH_BYTES in one file-scope __device__ array,
//     held on every GPU that loads the library until the process exits. The
//     number of partial-sum blocks is capped so that blocks * n fits in it.
//   * Every call shares that array and leaves its contents behind. Each call
//     writes every scratch row it reads, so nothing must be cleared first, but
//     calls whose kernels overlap on the GPU (different streams or host
//     threads) race on the array: serialise them.
//   * The first call on a device resolves the array's device address with
//     cudaGetSymbolAddress (the host-side symbol is not a device pointer).
//     Make that first call before any stream capture.
//   * Calls no cudaMalloc, cudaFree or allocating library routine.
//   * Returns PRISM_NOALLOC_OK or one of the error codes below;
//     prism_noalloc_error_string gives the message.
#pragma once

#include <cuda_runtime.h>

#define PRISM_NOALLOC_SCRATCH_BYTES (4 << 20)
#define PRISM_NOALLOC_MAX_N 8192

#define PRISM_NOALLOC_OK 0
#define PRISM_NOALLOC_BAD_ARGUMENT 1   /* null or misaligned pointer, rows < 1, n not a multiple of 8 */
#define PRISM_NOALLOC_TOO_LARGE 2      /* n > PRISM_NOALLOC_MAX_N */
#define PRISM_NOALLOC_SETUP_FAILED 3   /* scratch address could not be resolved on the current device */
#define PRISM_NOALLOC_LAUNCH_FAILED 4  /* one of this call's kernel launches failed */
#define PRISM_NOALLOC_PENDING_ERROR 5  /* a CUDA error from earlier work was pending; nothing launched */

#ifdef __cplusplus
extern "C" {
#endif

const char* prism_noalloc_error_string(int code);

int prism_rmsnorm_bwd_noalloc(const void* dy, const void* x, const void* w, const float* rstd, void* dx, float* dw,
                              int rows, int n, cudaStream_t stream);

#ifdef __cplusplus
}
#endif

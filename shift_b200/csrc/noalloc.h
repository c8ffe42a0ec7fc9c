// Allocation-free C entry point of the RMSNorm backward.
//
// This entry point has no counterpart in the reference; it exists only in
// this library.  It serves callers that must not allocate device memory on
// the call path: code running inside an allocator or a memory-pool callback,
// runtimes that pre-plan every byte of device memory and forbid cudaMalloc
// after start-up, and C hosts that do not link PyTorch's caching allocator.
// Instead of per-call scratch, the kernel's cross-block partial sums live in
// one file-scope device array of fixed size that every GPU loading the
// library keeps until the process exits.
#pragma once

#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

// Capacity of the shared scratch array, in floats (1 MiB): the kernel uses
// one row of `hidden` floats per thread block, and the entry point launches
// at most 256 blocks, so hidden <= 1024 always fits.
#define SB_NOALLOC_SCRATCH_FLOATS (256 * 1024)

// RMSNorm backward without any device allocation.
//
//   dx[r, :] = rstd[r] * (g - xhat * mean(g * xhat)) (+ dres[r, :]),
//              g = dy[r, :] * w,  xhat = x[r, :] * rstd[r]
//   dw[:]    = sum_r dy[r, :] * xhat[r, :]            (overwritten, fp32)
//
// dy, x, w, dres, dx are bf16; rstd and dw are fp32; dres may be NULL.
// rows >= 0; hidden must be 256, 512 or 1024.  `stream` is a cudaStream_t
// (NULL = legacy default stream).  All pointers are device pointers on the
// current device.
//
// Returns 0 on success; 1 if the problem needs more scratch than
// SB_NOALLOC_SCRATCH_FLOATS or hidden is unsupported; 2 if the one-time
// set-up on this device failed; 3 if the launch failed; 4 if a required
// pointer is NULL or misaligned (dy, x, w, dx and a non-NULL dres must be
// 16-byte aligned because rows move as 16-byte vectors; rstd and dw 4-byte
// aligned), in which case nothing is launched.  The first call on
// each device performs that set-up (it looks up the scratch array's device
// address), so make the first call before any stream capture.  Every call
// shares the same scratch array: calls whose kernels overlap on the GPU
// (different streams without ordering) race on it and must be serialised by
// the caller.  Nothing in the scratch needs to start at zero: each call
// writes every element it later reads.
int sb_rmsnorm_bwd_noalloc(const void* dy, const void* x, const float* rstd, const void* w, const void* dres,
                           void* dx, float* dw, int rows, int hidden, void* stream);

#ifdef __cplusplus
}
#endif

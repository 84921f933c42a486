// Allocation-free C entry point for the RMSNorm backward pass.
//
// This entry point has no counterpart in the reference framework.  It exists for
// callers that cannot allocate device memory at the moment they call in: code that
// runs inside a memory pool it does not own, host runtimes with no allocator hook,
// or embedding applications that forbid cudaMalloc after start-up.  The regular
// Python/torch entry point (rmsnorm_bwd in norm.cu) allocates a per-block partial
// buffer and its result through torch; this one needs only the caller's buffers.
//
// Scratch: the per-block partial sums of dW live in a file-scope device array of
// SV4_NOALLOC_MAX_BLOCKS x SV4_NOALLOC_MAX_DIM floats (4 MiB).  Every GPU that loads
// the library keeps that array until the process exits.  All calls share it and it
// keeps the previous call's contents; each call overwrites the rows it reads, so
// nothing needs clearing between calls -- but two calls that overlap on the GPU (on
// different streams, or from different threads without ordering) race on it.
//
// Set-up: the first call on a device looks up the array's device address with that
// device current (cudaGetSymbolAddress), raises the partial kernel's shared-memory limit
// (cudaFuncSetAttribute) and caches both.  Make that first call before any stream capture
// starts on the device.
//
// Determinism: dw is summed in a fixed order (per-warp rows, then blocks), so repeated
// calls on the same inputs give bit-identical results.
//
// Errors: a CUDA error already pending on the calling thread is returned as its own code
// and left pending (this call does not consume it).
#pragma once

#include <cuda_runtime.h>

#define SV4_NOALLOC_MAX_DIM 8192
#define SV4_NOALLOC_MAX_BLOCKS 128

#ifdef __cplusplus
extern "C" {
#endif

// dy, x, dx: (rows, dim) bf16, row-major, 16-byte aligned.  w: (dim) fp32 RMSNorm weight.
// rstd: (rows) fp32, 1/rms saved by the forward pass.  dw: (dim) fp32 output (overwritten).
// stream: a cudaStream_t (nullptr = legacy default stream).
// Returns 0 on success, otherwise an error code (see sv4_noalloc_error_string).
int sv4_rmsnorm_bwd_noalloc(const void* dy, const void* x, const float* w, const float* rstd, void* dx,
                            float* dw, int rows, int dim, void* stream);

// Human-readable text for an error code returned above.
const char* sv4_noalloc_error_string(int code);

#ifdef __cplusplus
}
#endif

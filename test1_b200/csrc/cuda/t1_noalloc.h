// C interface of the allocation-free RMSNorm backward (no counterpart in the
// reference).  For callers that cannot allocate device memory: code inside a
// custom memory arena or a framework that owns every device allocation,
// loops that forbid allocation after start-up, and C/C++ programs that link
// this library without PyTorch's caching allocator.  The caller passes every
// input and output; the partial sums of dw live in a 2 MiB file-scope device
// array that every GPU loading the library holds until the process exits.
//
// All calls on one device share that array and it keeps the last call's
// contents, so calls whose GPU work overlaps (different streams, or host
// threads without ordering) race and can give a wrong dw: serialise them.
// The first call on each device looks up the array's device address
// (cudaGetSymbolAddress, with that device current); make it before any
// stream capture begins.  No call allocates or frees device memory.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

// Largest hidden size the scratch array serves.
#define T1_NOALLOC_MAX_H 8192

// Return codes.
#define T1_NOALLOC_OK 0
#define T1_NOALLOC_BAD_ARGUMENT 1   // null pointer, T < 0, H <= 0 or H % 8 != 0
#define T1_NOALLOC_TOO_LARGE 2      // H > T1_NOALLOC_MAX_H
#define T1_NOALLOC_NO_SCRATCH 3     // the scratch array's device address is unavailable
#define T1_NOALLOC_PENDING_ERROR 4  // a CUDA error from earlier work was already pending;
                                    // nothing was launched and the error is left in place
#define T1_NOALLOC_LAUNCH_ERROR 1000  // + cudaError_t of a failed launch

// x [T, H] row-major bf16, w [H], rstd [T] fp32 (from the forward),
// dy [T, H], residual_grad [T, H] or NULL; outputs dx [T, H] and dw [H].
//   dx = rstd * (dy*w - xhat * mean(dy*w * xhat)) [+ residual_grad],  xhat = x * rstd
//   dw = sum over rows of dy * xhat
// All pointers are device pointers; the work is enqueued on `stream`.
int t1_rmsnorm_bwd_noalloc(const __nv_bfloat16* dy, const __nv_bfloat16* x,
                           const __nv_bfloat16* w, const float* rstd,
                           const __nv_bfloat16* residual_grad, __nv_bfloat16* dx,
                           __nv_bfloat16* dw, int T, int H, cudaStream_t stream);

#ifdef __cplusplus
}
#endif

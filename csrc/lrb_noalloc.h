// C entry points of llm_research_b200._C that allocate no device memory.
//
// This interface has no counterpart in the reference framework.  It exists for
// callers that cannot allocate device memory at the point of the call:
//   * hosts that reserve all of HBM up front (weights, optimizer shards and
//     activation arenas sized to the 180 GB budget) and keep nothing free;
//   * code running on an allocator's out-of-memory / defragmentation path,
//     where allocating would re-enter the allocator that is being repaired;
//   * plain C or C++ runtimes without PyTorch's caching allocator, where a
//     cudaMalloc/cudaFree would synchronise the device in the middle of a step.
// Every buffer is supplied by the caller; scratch lives in a fixed-size
// static device array inside the shared object.
#pragma once

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

// Return codes.
#define LRB_NOALLOC_OK 0
#define LRB_NOALLOC_ERR_ARGS 1      // null pointer, misaligned pointer or non-positive size
#define LRB_NOALLOC_ERR_TOO_LARGE 2 // row width above LRB_RMSNORM_BWD_NOALLOC_MAX_D
#define LRB_NOALLOC_ERR_CUDA 3      // a CUDA runtime call or the launch failed

// Widest row accepted (the per-block shared-memory accumulator of 8 rows x d
// fp32 values must fit in 200 KiB).
#define LRB_RMSNORM_BWD_NOALLOC_MAX_D 6400
// Size of the static scratch array that holds per-block weight-gradient partials.
#define LRB_RMSNORM_BWD_NOALLOC_SCRATCH_FLOATS (1 << 20)

// RMSNorm backward for bf16 activations and weight, identical in math to the
// `rmsnorm_bwd` op of the extension:
//   dx = rstd * (dy*w - xhat * mean(dy*w*xhat)) [+ ds],   xhat = x * rstd
//   dw = sum over rows of dy * bf16(xhat)
// dy, x, ds (optional, may be NULL), dx: (rows, d) bf16, contiguous, 16-byte
// aligned; w: (d) bf16; rstd: (rows) fp32 from the forward; dw: (d) fp32.
// dx and dw are fully overwritten: neither needs to start at zero, and the
// scratch array is fully written before it is read in every call, so nothing
// has to be cleared between calls.
// `stream` is a cudaStream_t of the current device (NULL = legacy default).
// The first call on each device looks up the scratch array's address with that
// device current (a symbol lookup that may load the module); do that first
// call before any stream capture on that device.
// Calls that overlap in time on the same device (different streams or host
// threads) share the scratch array and race: serialise them.
// On error returns a LRB_NOALLOC_ERR_* code and, when errbuf is not NULL,
// writes a NUL-terminated message of at most errbuf_len bytes.
int lrb_rmsnorm_bwd_bf16_noalloc(const void* dy, const void* x, const void* w, const float* rstd, const void* ds,
                                 void* dx, float* dw, int64_t rows, int64_t d, void* stream, char* errbuf,
                                 int errbuf_len);

#ifdef __cplusplus
}
#endif

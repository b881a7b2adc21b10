// C entry points of the tensor-core reduction GEMM that allocate no memory.
//
// This interface has no counterpart in the reference framework; it exists for callers that
// must not allocate device memory at call time:
//   * code running inside a custom allocator or an out-of-memory handler, where a nested
//     allocation would recurse or fail;
//   * host applications (an MD engine's force callback, a plugin loaded through dlopen)
//     that own the device memory budget and forbid libraries from taking more;
//   * C or Fortran callers that link this library without the PyTorch caching allocator.
//
// The computation is the one of the allocating entry point: out[K1, N] = scale * X^T D with
// X (M, K1) and D (M, N) float32 row-major on the device, split over rows into partial
// blocks that a second kernel sums in a fixed order (deterministic). The partial blocks live
// in a fixed scratch array of XNN_GEMM_REDUCE_NOALLOC_SCRATCH_FLOATS floats (8 MiB) compiled
// into the library, one copy per device. A call whose partial blocks do not fit is rejected
// with XNN_NOALLOC_ERR_SCRATCH before anything is launched.
//
// Setup: the first call on a device (with that device current) looks up the scratch array's
// device address with cudaGetSymbolAddress, which may load the library's module on that
// device. Call xnn_gemm_reduce_noalloc_setup() once per device before any stream capture
// that will contain these launches, so that this lookup does not happen during capture.
//
// Concurrency: every call on one device shares the same scratch array and status word. Calls
// issued to one stream run in order and are safe; calls that can overlap on the device
// (different streams, or several host threads) race on the scratch and give wrong results.
//
// What must start at zero: nothing the caller passes. The scratch array needs no clearing
// (each call overwrites every partial block it later reads); `out` is fully written. The
// device status word starts at zero when the module loads and is set to a non-zero code when a kernel's
// bounded wait on the tensor cores gave up; it stays set until cleared.
#pragma once

#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

#define XNN_GEMM_REDUCE_NOALLOC_SCRATCH_FLOATS (2 * 1024 * 1024)

// Return codes: 0 on success, a positive cudaError_t value when the CUDA runtime failed,
// or one of these negative codes (nothing was launched).
#define XNN_NOALLOC_ERR_SCRATCH (-1)  // ctas * K1 * N floats exceed the scratch array
#define XNN_NOALLOC_ERR_SHAPE (-2)    // K1 not in [1, 128], or N neither a multiple of 16 in [16, 256]
                                      // nor a multiple of 32 in [288, 512] (wider N runs as two
                                      // halves, each a multiple of 16)
#define XNN_NOALLOC_ERR_LAYOUT (-3)   // ldx or ldd not a multiple of 4, or X / D not 16-byte aligned
#define XNN_NOALLOC_ERR_ROWS (-4)     // rows_per_cta negative or not a multiple of 32

// Looks up the scratch array on the current device. Idempotent; thread-safe.
int xnn_gemm_reduce_noalloc_setup(void);

// out = scale * X^T D on `stream` (asynchronous). rows_per_cta = 0 picks the smallest
// multiple of 32 (at least 256) that keeps the CTA count at or below 296 and the partial
// blocks inside the scratch array; otherwise it must be a positive multiple of 32.
int xnn_gemm_reduce_tf32x3_noalloc(int M, int K1, int N, const float* X, int ldx, const float* D, int ldd,
                                   int rows_per_cta, float scale, float* out, cudaStream_t stream);

// Copies the current device's status word to *value (synchronous; 0 = no wait gave up).
int xnn_gemm_reduce_noalloc_status(int* value);

// Sets the current device's status word back to 0 (synchronous).
int xnn_gemm_reduce_noalloc_clear_status(void);

// Human-readable text for a return code of the functions above.
const char* xnn_gemm_reduce_noalloc_error_string(int code);

#ifdef __cplusplus
}
#endif

// Allocation-free bias-gradient entry point (C ABI).
//
// This entry point has no counterpart in the reference. It exists for callers
// that cannot call cudaMalloc: a serving or training runtime that reserves all
// device memory for its own pool at start-up, a host framework whose plugin
// interface forbids allocating outside its allocator, or code that must not
// allocate after initialisation because cudaMalloc can synchronise the device.
// Such callers pass their input and output buffers and nothing else.
//
//   out[c] (+)= sum_m dy[m, c]     for bf16 dy [M, C] (row stride ld), fp32 out [C]
//
// Scratch. The two-stage reduction keeps its per-chunk partial sums in one
// file-scope device array of G2B_NOALLOC_SCRATCH_FLOATS floats (1 MiB), which
// every GPU that loads this library holds until the process exits. A call
// needs ceil(M / 128) * C floats of it; a larger request is rejected with
// G2B_NOALLOC_ERR_TOO_LARGE and a message on stderr, and nothing is launched.
// Every scratch element a call reads is written earlier in the same call, so
// nothing has to start at zero; the array keeps the last call's contents.
// All calls share the one array, so calls that overlap on the GPU (different
// streams, or different threads, on the same device) race: order them.
//
// Set-up. The first call on each device looks up the array's device address
// with cudaGetSymbolAddress while that device is current, and caches it; make
// that first call before any stream capture.
//
// Returns 0 on success or one of the negative codes below.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#define G2B_NOALLOC_SCRATCH_FLOATS (1 << 18)
#define G2B_NOALLOC_ERR_ARGS (-1)       /* null pointer, non-positive size, C or ld not a multiple of 8, misaligned dy */
#define G2B_NOALLOC_ERR_TOO_LARGE (-2)  /* ceil(M/128) * C exceeds G2B_NOALLOC_SCRATCH_FLOATS */
#define G2B_NOALLOC_ERR_SETUP (-3)      /* cudaGetDevice / cudaGetSymbolAddress failed */
#define G2B_NOALLOC_ERR_LAUNCH (-4)     /* kernel launch failed */

#ifdef __cplusplus
extern "C" {
#endif

int g2b_bias_grad_noalloc(const void* dy, int64_t ld, int M, int C, float* out, int accumulate,
                          cudaStream_t stream);

#ifdef __cplusplus
}
#endif

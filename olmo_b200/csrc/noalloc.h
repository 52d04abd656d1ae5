// Allocation-free entry point (this has no counterpart in the reference implementation).
//
// Who needs it: code that must not touch the device allocator while it runs — a caller inside a region where
// cudaMalloc/cudaFree are forbidden or would serialise the device (a latency-critical step loop that has frozen its
// memory pool, a host callback, a plug-in that is handed raw pointers and a stream but owns no allocator), and which
// therefore cannot supply the scratch vector that ob_sumsq_f32 asks for.
//
//   ob_sumsq_f32_noalloc(g, n, out, accumulate, stream):  out[0] (+)= sum_i g[i]^2   for a flat fp32 buffer on the
//   current device, the same result as ob_sumsq_f32 up to summation order.
//
// The per-block partial sums live in a file-scope device array inside the library instead of caller memory:
//   * size: OB_NOALLOC_MAX_PARTIALS floats (32 KiB); every GPU that loads the library holds it until the process exits;
//   * one partial covers OB_NOALLOC_QUANTUM consecutive elements, so n may be at most
//     OB_NOALLOC_MAX_PARTIALS * OB_NOALLOC_QUANTUM = 2^31 elements (8 GiB of fp32); a larger n is rejected with
//     OB_NOALLOC_ERR_TOO_LARGE and nothing is launched;
//   * the first call on a device looks up the array's device address (one cudaGetSymbolAddress, no allocation) and
//     caches it; make that first call outside any stream capture.  Host threads may make it concurrently (they store the
//     same address);
//   * `out` must not be null, and `g` must not be null unless n is 0 (OB_NOALLOC_ERR_NULL, nothing is launched);
//   * every call on a device shares the one array, which keeps the previous call's partials.  A call overwrites every
//     entry it later reads, so nothing needs clearing, but two calls whose kernels overlap on the GPU (different
//     streams without ordering) race on it — serialise them.
//
// The function calls no cudaMalloc/cudaFree and no allocating library routine.  Returns 0, or a negative code that
// ob_noalloc_strerror turns into text.
#pragma once

#include <cuda_runtime.h>

#define OB_NOALLOC_MAX_PARTIALS 8192
#define OB_NOALLOC_QUANTUM (1 << 18)

#define OB_NOALLOC_ERR_TOO_LARGE (-101)
#define OB_NOALLOC_ERR_ALIGNMENT (-102)
#define OB_NOALLOC_ERR_SYMBOL (-103)
#define OB_NOALLOC_ERR_LAUNCH (-104)
#define OB_NOALLOC_ERR_DEVICE (-105)
#define OB_NOALLOC_ERR_NULL (-106)

#ifdef __cplusplus
extern "C" {
#endif

int ob_sumsq_f32_noalloc(const float* g, long long n, float* out, int accumulate, cudaStream_t stream);
long long ob_sumsq_f32_noalloc_max_elements(void);
const char* ob_noalloc_strerror(int code);

#ifdef __cplusplus
}
#endif

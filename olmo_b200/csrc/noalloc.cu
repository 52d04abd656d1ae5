// Sum of squares of a flat fp32 buffer without any caller- or allocator-provided scratch: see noalloc.h.
#include "common.cuh"
#include "noalloc.h"

namespace ob {
namespace {

constexpr int NA_THREADS = 512;
constexpr int NA_MAX_DEVICES = 64;

// Partial sums, one per quantum of the input.  Lives in every GPU that loads this library.
static __device__ __align__(256) float g_noalloc_partials[OB_NOALLOC_MAX_PARTIALS];

// Block b reduces elements [b * QUANTUM, min(n, (b + 1) * QUANTUM)).
__global__ void __launch_bounds__(NA_THREADS)
na_partial_kernel(const float* __restrict__ g, long long n, float* __restrict__ partials) {
  __shared__ float red[32];
  const long long begin = static_cast<long long>(blockIdx.x) * OB_NOALLOC_QUANTUM;
  long long end = begin + OB_NOALLOC_QUANTUM;
  if (end > n) end = n;
  const long long nvec = (end - begin) >> 2;  // begin is a multiple of 4 elements, g is 16-byte aligned
  const float4* v = reinterpret_cast<const float4*>(g + begin);
  float s = 0.f;
  for (long long i = threadIdx.x; i < nvec; i += NA_THREADS) {
    const float4 a = v[i];
    s += a.x * a.x + a.y * a.y + a.z * a.z + a.w * a.w;
  }
  if (threadIdx.x == 0)
    for (long long i = begin + nvec * 4; i < end; ++i) s += g[i] * g[i];
  s = block_sum(s, red);
  if (threadIdx.x == 0) partials[blockIdx.x] = s;
}

__global__ void __launch_bounds__(NA_THREADS)
na_final_kernel(const float* __restrict__ partials, int nparts, float* __restrict__ out, int accumulate) {
  __shared__ float red[32];
  float s = 0.f;
  for (int i = threadIdx.x; i < nparts; i += NA_THREADS) s += partials[i];
  s = block_sum(s, red);
  if (threadIdx.x == 0) out[0] = accumulate ? out[0] + s : s;
}

// Device address of g_noalloc_partials per device ordinal.  In host code the array's name is only a handle for the
// runtime, not an address a kernel could use, so the address is obtained once per device with that device current.
// The table is filled without a lock: two host threads that make the first call on a device at the same time both look
// the address up and both store the same value.
float* g_partials_addr[NA_MAX_DEVICES] = {nullptr};

int scratch_for_current_device(float** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= NA_MAX_DEVICES) return OB_NOALLOC_ERR_DEVICE;
  if (g_partials_addr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_partials) != cudaSuccess || p == nullptr) return OB_NOALLOC_ERR_SYMBOL;
    g_partials_addr[dev] = static_cast<float*>(p);
  }
  *out = g_partials_addr[dev];
  return 0;
}

}  // namespace
}  // namespace ob

extern "C" long long ob_sumsq_f32_noalloc_max_elements(void) {
  return static_cast<long long>(OB_NOALLOC_MAX_PARTIALS) * OB_NOALLOC_QUANTUM;
}

extern "C" const char* ob_noalloc_strerror(int code) {
  switch (code) {
    case 0: return "ok";
    case OB_NOALLOC_ERR_TOO_LARGE: return "n exceeds ob_sumsq_f32_noalloc_max_elements(): the built-in scratch array cannot hold its partial sums";
    case OB_NOALLOC_ERR_ALIGNMENT: return "input pointer must be 16-byte aligned";
    case OB_NOALLOC_ERR_SYMBOL: return "cudaGetSymbolAddress failed for the built-in scratch array";
    case OB_NOALLOC_ERR_LAUNCH: return "kernel launch failed";
    case OB_NOALLOC_ERR_DEVICE: return "no current CUDA device, or its ordinal is out of range";
    case OB_NOALLOC_ERR_NULL: return "out is null, or g is null while n > 0";
    default: return "unknown error";
  }
}

extern "C" int ob_sumsq_f32_noalloc(const float* g, long long n, float* out, int accumulate, cudaStream_t stream) {
  using namespace ob;
  if (n < 0 || n > ob_sumsq_f32_noalloc_max_elements()) return OB_NOALLOC_ERR_TOO_LARGE;
  if (out == nullptr || (n > 0 && g == nullptr)) return OB_NOALLOC_ERR_NULL;  // a launch on a null pointer would fault the device
  if ((reinterpret_cast<uintptr_t>(g) & 15) != 0) return OB_NOALLOC_ERR_ALIGNMENT;
  float* partials = nullptr;
  const int rc = scratch_for_current_device(&partials);  // first call on a device: one symbol lookup, no allocation
  if (rc != 0) return rc;
  const int nparts = n == 0 ? 0 : static_cast<int>((n + OB_NOALLOC_QUANTUM - 1) / OB_NOALLOC_QUANTUM);
  if (nparts > 0) na_partial_kernel<<<nparts, NA_THREADS, 0, stream>>>(g, n, partials);
  na_final_kernel<<<1, NA_THREADS, 0, stream>>>(partials, nparts, out, accumulate);
  return cudaGetLastError() == cudaSuccess ? 0 : OB_NOALLOC_ERR_LAUNCH;
}

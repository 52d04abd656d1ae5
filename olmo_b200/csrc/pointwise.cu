// Bandwidth-bound pointwise kernels: SwiGLU forward/backward, embedding gather and its gradient scatter-add,
// bf16 <-> fp32 accumulate helpers.
#include "common.cuh"
#include "api.h"

namespace ob {
namespace {

__device__ __forceinline__ void ld8(const bf16* p, float (&f)[8]) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 t = unpack_bf16x2(w[j]);
    f[2 * j] = t.x;
    f[2 * j + 1] = t.y;
  }
}
__device__ __forceinline__ void st8(bf16* p, const float (&f)[8]) {
  uint4 o;
  o.x = pack_bf16x2(f[0], f[1]);
  o.y = pack_bf16x2(f[2], f[3]);
  o.z = pack_bf16x2(f[4], f[5]);
  o.w = pack_bf16x2(f[6], f[7]);
  *reinterpret_cast<uint4*>(p) = o;
}

// h[M, 2H] = [value | gate]  ->  out[M, H] = silu(gate) * value
__global__ void swiglu_fwd_kernel(const bf16* __restrict__ h, bf16* __restrict__ out, int M, int H) {
  const int vec_per_row = H >> 3;
  const size_t total = static_cast<size_t>(M) * vec_per_row;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const size_t row = i / vec_per_row;
    const int c = static_cast<int>(i % vec_per_row) * 8;
    float v[8], g[8], o[8];
    ld8(h + row * 2 * H + c, v);
    ld8(h + row * 2 * H + H + c, g);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      // portable model: silu(gate) is rounded to bf16 before the product
      const float s = __bfloat162float(__float2bfloat16_rn(g[j] / (1.f + __expf(-g[j]))));
      o[j] = s * v[j];
    }
    st8(out + row * H + c, o);
  }
}

// dh[M, 2H] from dout[M, H] and h:  dvalue = dout * silu(gate);  dgate = dout * value * sig * (1 + gate (1 - sig))
__global__ void swiglu_bwd_kernel(const bf16* __restrict__ dout, const bf16* __restrict__ h, bf16* __restrict__ dh, int M,
                                  int H) {
  const int vec_per_row = H >> 3;
  const size_t total = static_cast<size_t>(M) * vec_per_row;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const size_t row = i / vec_per_row;
    const int c = static_cast<int>(i % vec_per_row) * 8;
    float v[8], g[8], d[8], dv[8], dg[8];
    ld8(h + row * 2 * H + c, v);
    ld8(h + row * 2 * H + H + c, g);
    ld8(dout + row * H + c, d);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float sig = 1.f / (1.f + __expf(-g[j]));
      dv[j] = d[j] * g[j] * sig;
      dg[j] = d[j] * v[j] * sig * (1.f + g[j] * (1.f - sig));
    }
    st8(dh + row * 2 * H + c, dv);
    st8(dh + row * 2 * H + H + c, dg);
  }
}

// out[m, :] = table[ids[m], :]
__global__ void embedding_fwd_kernel(const long long* __restrict__ ids, const bf16* __restrict__ table,
                                     bf16* __restrict__ out, int M, int D, int V) {
  const int vec_per_row = D >> 3;
  for (int row = blockIdx.x; row < M; row += gridDim.x) {
    long long id = ids[row];
    if (id < 0 || id >= V) id = 0;  // out-of-range ids read row 0 instead of faulting
    const uint4* src = reinterpret_cast<const uint4*>(table + static_cast<size_t>(id) * D);
    uint4* dst = reinterpret_cast<uint4*>(out + static_cast<size_t>(row) * D);
    for (int i = threadIdx.x; i < vec_per_row; i += blockDim.x) dst[i] = src[i];
  }
}

// grad_table[ids[m], :] += dout[m, :]   (fp32 accumulation with vector reductions)
__global__ void embedding_bwd_kernel(const long long* __restrict__ ids, const bf16* __restrict__ dout,
                                     float* __restrict__ grad, int M, int D, int V) {
  const int vec_per_row = D >> 3;
  for (int row = blockIdx.x; row < M; row += gridDim.x) {
    const long long id = ids[row];
    if (id < 0 || id >= V) continue;
    float* g = grad + static_cast<size_t>(id) * D;
    const bf16* d = dout + static_cast<size_t>(row) * D;
    for (int i = threadIdx.x; i < vec_per_row; i += blockDim.x) {
      float f[8];
      ld8(d + i * 8, f);
      atomicAdd(reinterpret_cast<float4*>(g + i * 8), make_float4(f[0], f[1], f[2], f[3]));
      atomicAdd(reinterpret_cast<float4*>(g + i * 8 + 4), make_float4(f[4], f[5], f[6], f[7]));
    }
  }
}

// acc[i] += src[i] (bf16 -> fp32), n multiple of 8
__global__ void accum_bf16_to_f32_kernel(const bf16* __restrict__ src, float* __restrict__ acc, size_t nvec) {
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < nvec;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    float f[8];
    ld8(src + i * 8, f);
    float4 a = *reinterpret_cast<float4*>(acc + i * 8);
    float4 b = *reinterpret_cast<float4*>(acc + i * 8 + 4);
    a.x += f[0]; a.y += f[1]; a.z += f[2]; a.w += f[3];
    b.x += f[4]; b.y += f[5]; b.z += f[6]; b.w += f[7];
    *reinterpret_cast<float4*>(acc + i * 8) = a;
    *reinterpret_cast<float4*>(acc + i * 8 + 4) = b;
  }
}

// dst(bf16)[i] = src(fp32)[i], n multiple of 8
__global__ void cast_f32_to_bf16_kernel(const float* __restrict__ src, bf16* __restrict__ dst, size_t nvec) {
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < nvec;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const float4 a = *reinterpret_cast<const float4*>(src + i * 8);
    const float4 b = *reinterpret_cast<const float4*>(src + i * 8 + 4);
    const float f[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    st8(dst + i * 8, f);
  }
}

inline int grid_for(size_t work_items, int threads) {
  size_t g = (work_items + threads - 1) / threads;
  const size_t cap = 148 * 16;
  return static_cast<int>(g < cap ? (g == 0 ? 1 : g) : cap);
}

}  // namespace
}  // namespace ob

extern "C" int ob_swiglu_fwd(const void* h, void* out, int M, int H, cudaStream_t stream) {
  using namespace ob;
  if (M <= 0) return 0;
  if (H % 8 != 0) return -1;
  swiglu_fwd_kernel<<<grid_for(static_cast<size_t>(M) * (H / 8), 256), 256, 0, stream>>>((const bf16*)h, (bf16*)out, M, H);
  return cudaGetLastError() == cudaSuccess ? 0 : -11;
}

extern "C" int ob_swiglu_bwd(const void* dout, const void* h, void* dh, int M, int H, cudaStream_t stream) {
  using namespace ob;
  if (M <= 0) return 0;
  if (H % 8 != 0) return -1;
  swiglu_bwd_kernel<<<grid_for(static_cast<size_t>(M) * (H / 8), 256), 256, 0, stream>>>((const bf16*)dout, (const bf16*)h,
                                                                                     (bf16*)dh, M, H);
  return cudaGetLastError() == cudaSuccess ? 0 : -11;
}

extern "C" int ob_embedding_fwd(const long long* ids, const void* table, void* out, int M, int D, int V,
                                cudaStream_t stream) {
  using namespace ob;
  if (M <= 0) return 0;
  if (D % 8 != 0) return -1;
  embedding_fwd_kernel<<<M < 148 * 16 ? M : 148 * 16, 256, 0, stream>>>(ids, (const bf16*)table, (bf16*)out, M, D, V);
  return cudaGetLastError() == cudaSuccess ? 0 : -11;
}

extern "C" int ob_embedding_bwd(const long long* ids, const void* dout, float* grad, int M, int D, int V,
                                cudaStream_t stream) {
  using namespace ob;
  if (M <= 0) return 0;
  if (D % 8 != 0) return -1;
  embedding_bwd_kernel<<<M < 148 * 16 ? M : 148 * 16, 256, 0, stream>>>(ids, (const bf16*)dout, grad, M, D, V);
  return cudaGetLastError() == cudaSuccess ? 0 : -11;
}

extern "C" int ob_accum_bf16_to_f32(const void* src, float* acc, long long n, cudaStream_t stream) {
  using namespace ob;
  if (n <= 0) return 0;
  if (n % 8 != 0) return -1;
  accum_bf16_to_f32_kernel<<<grid_for(n / 8, 256), 256, 0, stream>>>((const bf16*)src, acc, n / 8);
  return cudaGetLastError() == cudaSuccess ? 0 : -11;
}

extern "C" int ob_cast_f32_to_bf16(const float* src, void* dst, long long n, cudaStream_t stream) {
  using namespace ob;
  if (n <= 0) return 0;
  if (n % 8 != 0) return -1;
  cast_f32_to_bf16_kernel<<<grid_for(n / 8, 256), 256, 0, stream>>>(src, (bf16*)dst, n / 8);
  return cudaGetLastError() == cudaSuccess ? 0 : -11;
}

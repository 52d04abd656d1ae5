// Fused cross-entropy (+ z-loss) over a wide vocabulary, and the fused optimizer / gradient-norm kernels that
// run on flat fp32 shards.
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

constexpr int CE_THREADS = 512;

// One CTA per row.  Pass 1: online (max, sum-exp) over the row.  Pass 2 (optional): overwrite the logits with
//   d/dlogit [ (CE + z_mult * lse^2) * grad_scale ] = grad_scale * ( softmax * (1 + 2 z_mult lse) - onehot ).
// Rows whose label equals ignore_index produce zero loss and zero gradient.
__global__ void __launch_bounds__(CE_THREADS)
ce_kernel(bf16* __restrict__ logits, const long long* __restrict__ labels, float* __restrict__ ce_out,
          float* __restrict__ z_out, int R, int V, int ld, long long ignore_index, float z_mult, float grad_scale,
          int write_grad) {
  __shared__ float red[32];
  const int nvec = V >> 3;
  for (int row = blockIdx.x; row < R; row += gridDim.x) {
    bf16* x = logits + static_cast<size_t>(row) * ld;
    const long long y = labels[row];
    if (y == ignore_index || y < 0 || y >= V) {
      if (threadIdx.x == 0) {
        ce_out[row] = 0.f;
        if (z_out != nullptr) z_out[row] = 0.f;
      }
      if (write_grad) {
        const uint4 z = make_uint4(0, 0, 0, 0);
        for (int i = threadIdx.x; i < nvec; i += CE_THREADS) *reinterpret_cast<uint4*>(x + i * 8) = z;
      }
      continue;
    }
    float m = -INFINITY, s = 0.f;
    for (int i = threadIdx.x; i < nvec; i += CE_THREADS) {
      float f[8];
      ld8(x + i * 8, f);
      float lm = f[0];
#pragma unroll
      for (int j = 1; j < 8; ++j) lm = fmaxf(lm, f[j]);
      if (lm > m) {
        s *= __expf(m - lm);
        m = lm;
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) s += __expf(f[j] - m);
    }
    const float gmax = block_max(m, red);
    s *= (m == -INFINITY) ? 0.f : __expf(m - gmax);
    const float gsum = block_sum(s, red);
    const float lse = gmax + logf(gsum);
    const float xy = __bfloat162float(x[y]);
    __syncthreads();  // every thread has read x[y] before pass 2 overwrites it
    if (threadIdx.x == 0) {
      ce_out[row] = lse - xy;
      if (z_out != nullptr) z_out[row] = lse * lse;
    }
    if (write_grad) {
      const float coef = grad_scale * (1.f + 2.f * z_mult * lse);
      const int yv = static_cast<int>(y >> 3), yj = static_cast<int>(y & 7);
      for (int i = threadIdx.x; i < nvec; i += CE_THREADS) {
        float f[8];
        ld8(x + i * 8, f);
#pragma unroll
        for (int j = 0; j < 8; ++j) f[j] = coef * __expf(f[j] - lse);
        if (i == yv) f[yj] -= grad_scale;
        st8(x + i * 8, f);
      }
    }
  }
}

// ---------------------------------------------------------------------------------------- optimizers

struct Segments {
  const long long* end;  // exclusive end offset of each segment inside the flat buffer, ascending
  const float* wd;       // weight decay of the segment
  const float* lr;       // learning rate of the segment
  int count;
};

__device__ __forceinline__ int find_segment(const Segments& s, long long idx) {
  int lo = 0, hi = s.count - 1;
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    if (idx < s.end[mid]) hi = mid;
    else lo = mid + 1;
  }
  return lo;
}

// AdamW with decoupled weight decay on a flat fp32 shard; optionally emits the bf16 copy used by the next gather.
// `gscale` is a device scalar (the clipping coefficient); gradients are multiplied by it on the fly.
__global__ void adamw_kernel(float* __restrict__ p, const float* __restrict__ g, float* __restrict__ m,
                             float* __restrict__ v, bf16* __restrict__ p_lowp, long long n, Segments seg, float beta1,
                             float beta2, float eps, float bias1, float bias2_sqrt, const float* __restrict__ gscale) {
  const float gs = (gscale != nullptr) ? *gscale : 1.f;
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x * 4;
  for (long long i0 = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) * 4; i0 < n; i0 += stride) {
    int sidx = find_segment(seg, i0);
    if (i0 + 4 <= n) {
      float4 pv = *reinterpret_cast<float4*>(p + i0);
      const float4 gv = *reinterpret_cast<const float4*>(g + i0);
      float4 mv = *reinterpret_cast<float4*>(m + i0);
      float4 vv = *reinterpret_cast<float4*>(v + i0);
      float* pp = reinterpret_cast<float*>(&pv);
      const float* gp = reinterpret_cast<const float*>(&gv);
      float* mp = reinterpret_cast<float*>(&mv);
      float* vp = reinterpret_cast<float*>(&vv);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        while (i0 + j >= seg.end[sidx] && sidx < seg.count - 1) ++sidx;
        const float lr = seg.lr[sidx], wd = seg.wd[sidx];
        const float gj = gp[j] * gs;
        pp[j] *= 1.f - lr * wd;
        mp[j] = beta1 * mp[j] + (1.f - beta1) * gj;
        vp[j] = beta2 * vp[j] + (1.f - beta2) * gj * gj;
        const float denom = sqrtf(vp[j]) / bias2_sqrt + eps;
        pp[j] -= (lr / bias1) * (mp[j] / denom);
      }
      *reinterpret_cast<float4*>(p + i0) = pv;
      *reinterpret_cast<float4*>(m + i0) = mv;
      *reinterpret_cast<float4*>(v + i0) = vv;
      if (p_lowp != nullptr) {
        uint2 o;
        o.x = pack_bf16x2(pp[0], pp[1]);
        o.y = pack_bf16x2(pp[2], pp[3]);
        *reinterpret_cast<uint2*>(p_lowp + i0) = o;
      }
    } else {
      for (long long i = i0; i < n; ++i) {
        while (i >= seg.end[sidx] && sidx < seg.count - 1) ++sidx;
        const float lr = seg.lr[sidx], wd = seg.wd[sidx];
        const float gj = g[i] * gs;
        float pj = p[i] * (1.f - lr * wd);
        const float mj = beta1 * m[i] + (1.f - beta1) * gj;
        const float vj = beta2 * v[i] + (1.f - beta2) * gj * gj;
        pj -= (lr / bias1) * (mj / (sqrtf(vj) / bias2_sqrt + eps));
        p[i] = pj;
        m[i] = mj;
        v[i] = vj;
        if (p_lowp != nullptr) p_lowp[i] = __float2bfloat16_rn(pj);
      }
    }
  }
}

// Lion with decoupled weight decay: update = sign(b1 m + (1-b1) g); p = p (1 - lr wd) - lr update; m = b2 m + (1-b2) g
__global__ void lionw_kernel(float* __restrict__ p, const float* __restrict__ g, float* __restrict__ m,
                             bf16* __restrict__ p_lowp, long long n, Segments seg, float beta1, float beta2,
                             const float* __restrict__ gscale) {
  const float gs = (gscale != nullptr) ? *gscale : 1.f;
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride) {
    const int sidx = find_segment(seg, i);
    const float lr = seg.lr[sidx], wd = seg.wd[sidx];
    const float gj = g[i] * gs;
    const float u = beta1 * m[i] + (1.f - beta1) * gj;
    const float sgn = (u > 0.f) ? 1.f : ((u < 0.f) ? -1.f : 0.f);
    const float pj = p[i] * (1.f - lr * wd) - lr * sgn;
    p[i] = pj;
    m[i] = beta2 * m[i] + (1.f - beta2) * gj;
    if (p_lowp != nullptr) p_lowp[i] = __float2bfloat16_rn(pj);
  }
}

constexpr int SQ_THREADS = 512;

__global__ void __launch_bounds__(SQ_THREADS)
sumsq_partial_kernel(const float* __restrict__ g, long long n, float* __restrict__ partials) {
  __shared__ float red[32];
  float s = 0.f;
  const long long nvec = n >> 2;
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < nvec; i += stride) {
    const float4 a = *reinterpret_cast<const float4*>(g + i * 4);
    s += a.x * a.x + a.y * a.y + a.z * a.z + a.w * a.w;
  }
  if (blockIdx.x == 0 && threadIdx.x == 0)
    for (long long i = nvec * 4; i < n; ++i) s += g[i] * g[i];
  s = block_sum(s, red);
  if (threadIdx.x == 0) partials[blockIdx.x] = s;
}

__global__ void __launch_bounds__(SQ_THREADS)
sumsq_final_kernel(const float* __restrict__ partials, int nparts, float* __restrict__ out, int accumulate) {
  __shared__ float red[32];
  float s = 0.f;
  for (int i = threadIdx.x; i < nparts; i += blockDim.x) s += partials[i];
  s = block_sum(s, red);
  if (threadIdx.x == 0) out[0] = accumulate ? out[0] + s : s;
}

// coef[0] = min(1, max_norm / (sqrt(sumsq[0]) + 1e-6))
__global__ void clip_coef_kernel(const float* __restrict__ sumsq, float max_norm, float* __restrict__ coef,
                                 float* __restrict__ norm_out) {
  const float norm = sqrtf(sumsq[0]);
  if (norm_out != nullptr) norm_out[0] = norm;
  coef[0] = fminf(max_norm / (norm + 1e-6f), 1.0f);
}

}  // namespace
}  // namespace ob

extern "C" int ob_cross_entropy(void* logits, const long long* labels, float* ce_out, float* z_out, int R, int V, int ld,
                                long long ignore_index, float z_mult, float grad_scale, int write_grad,
                                cudaStream_t stream) {
  using namespace ob;
  if (R <= 0) return 0;
  if (V % 8 != 0 || ld % 8 != 0) return -1;
  ce_kernel<<<R < 148 * 4 ? R : 148 * 4, CE_THREADS, 0, stream>>>((bf16*)logits, labels, ce_out, z_out, R, V, ld,
                                                                   ignore_index, z_mult, grad_scale, write_grad);
  return cudaGetLastError() == cudaSuccess ? 0 : -11;
}

extern "C" int ob_adamw(float* p, const float* g, float* m, float* v, void* p_lowp, long long n,
                        const long long* seg_end, const float* seg_wd, const float* seg_lr, int nseg, float beta1,
                        float beta2, float eps, int step, const float* gscale, cudaStream_t stream) {
  using namespace ob;
  if (n <= 0) return 0;
  if (nseg <= 0) return -1;
  const float bias1 = 1.f - powf(beta1, (float)step);
  const float bias2_sqrt = sqrtf(1.f - powf(beta2, (float)step));
  Segments seg{seg_end, seg_wd, seg_lr, nseg};
  long long blocks = (n / 4 + 255) / 256;
  if (blocks > 148 * 16) blocks = 148 * 16;
  if (blocks < 1) blocks = 1;
  adamw_kernel<<<(int)blocks, 256, 0, stream>>>(p, g, m, v, (bf16*)p_lowp, n, seg, beta1, beta2, eps, bias1, bias2_sqrt,
                                                gscale);
  return cudaGetLastError() == cudaSuccess ? 0 : -11;
}

extern "C" int ob_lionw(float* p, const float* g, float* m, void* p_lowp, long long n, const long long* seg_end,
                        const float* seg_wd, const float* seg_lr, int nseg, float beta1, float beta2,
                        const float* gscale, cudaStream_t stream) {
  using namespace ob;
  if (n <= 0) return 0;
  if (nseg <= 0) return -1;
  Segments seg{seg_end, seg_wd, seg_lr, nseg};
  long long blocks = (n + 255) / 256;
  if (blocks > 148 * 16) blocks = 148 * 16;
  lionw_kernel<<<(int)blocks, 256, 0, stream>>>(p, g, m, (bf16*)p_lowp, n, seg, beta1, beta2, gscale);
  return cudaGetLastError() == cudaSuccess ? 0 : -11;
}

extern "C" int ob_sumsq_num_partials(long long n) {
  long long blocks = (n / 4 + ob::SQ_THREADS - 1) / ob::SQ_THREADS;
  if (blocks > 148 * 4) blocks = 148 * 4;
  if (blocks < 1) blocks = 1;
  return (int)blocks;
}

// Sum of squares of a flat fp32 buffer; `partials` is scratch of ob_sumsq_num_partials(n) floats.
extern "C" int ob_sumsq_f32(const float* g, long long n, float* partials, float* out, int accumulate,
                            cudaStream_t stream) {
  using namespace ob;
  if (n <= 0) return 0;
  if ((reinterpret_cast<uintptr_t>(g) & 15) != 0) return -1;
  const int blocks = ob_sumsq_num_partials(n);
  sumsq_partial_kernel<<<blocks, SQ_THREADS, 0, stream>>>(g, n, partials);
  sumsq_final_kernel<<<1, SQ_THREADS, 0, stream>>>(partials, blocks, out, accumulate);
  return cudaGetLastError() == cudaSuccess ? 0 : -11;
}

extern "C" int ob_clip_coef(const float* sumsq, float max_norm, float* coef, float* norm_out, cudaStream_t stream) {
  ob::clip_coef_kernel<<<1, 1, 0, stream>>>(sumsq, max_norm, coef, norm_out);
  return cudaGetLastError() == cudaSuccess ? 0 : -11;
}

// Row-wise normalisation kernels (bandwidth bound; one CTA walks rows with 16-byte vector accesses).
//
//   norm_fwd : out = [res +] norm(x) [* w] [+ b]      norm = RMSNorm (fp32 statistics) or LayerNorm
//   norm_bwd : dx  = [dres +] d norm / dx,  per-CTA partial sums of dw (and db) go to a scratch matrix that
//              reduce_rows_f32 folds into the fp32 gradient.
// Rounding follows the portable model: the normalised value is rounded to bf16 before the affine transform.
#include "common.cuh"
#include "api.h"

namespace ob {
namespace {

constexpr int NT = 256;   // threads per CTA
constexpr int MAXV = 4;   // vectors of 8 bf16 per thread -> D <= 8192

__device__ __forceinline__ void load8(const bf16* p, float (&f)[8]) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 t = unpack_bf16x2(w[j]);
    f[2 * j] = t.x;
    f[2 * j + 1] = t.y;
  }
}

__device__ __forceinline__ void store8(bf16* p, const float (&f)[8]) {
  uint4 o;
  o.x = pack_bf16x2(f[0], f[1]);
  o.y = pack_bf16x2(f[2], f[3]);
  o.z = pack_bf16x2(f[4], f[5]);
  o.w = pack_bf16x2(f[6], f[7]);
  *reinterpret_cast<uint4*>(p) = o;
}

__device__ __forceinline__ float round_bf16(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

template <bool RMS>
__global__ void __launch_bounds__(NT) norm_fwd_kernel(const bf16* __restrict__ x, const bf16* __restrict__ res,
                                                      const bf16* __restrict__ w, const bf16* __restrict__ b,
                                                      bf16* __restrict__ out, float* __restrict__ rstd_out,
                                                      float* __restrict__ mean_out, int M, int D, int ldx, float eps) {
  __shared__ float red[32];
  const int nvec = D >> 3;
  for (int row = blockIdx.x; row < M; row += gridDim.x) {
    const bf16* xr = x + static_cast<size_t>(row) * ldx;
    float v[MAXV][8];
    float s = 0.f, ss = 0.f;
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
      const int vi = threadIdx.x + i * NT;
      if (vi < nvec) {
        load8(xr + vi * 8, v[i]);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          s += v[i][j];
          ss += v[i][j] * v[i][j];
        }
      }
    }
    float mean = 0.f, rstd;
    if (RMS) {
      ss = block_sum(ss, red);
      rstd = rsqrtf(ss / D + eps);
    } else {
      s = block_sum(s, red);
      mean = s / D;
      float var = 0.f;
#pragma unroll
      for (int i = 0; i < MAXV; ++i) {
        const int vi = threadIdx.x + i * NT;
        if (vi < nvec) {
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const float d = v[i][j] - mean;
            var += d * d;
          }
        }
      }
      var = block_sum(var, red);
      rstd = rsqrtf(var / D + eps);
    }
    if (threadIdx.x == 0) {
      if (rstd_out != nullptr) rstd_out[row] = rstd;
      if (!RMS && mean_out != nullptr) mean_out[row] = mean;
    }
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
      const int vi = threadIdx.x + i * NT;
      if (vi < nvec) {
        float y[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) y[j] = round_bf16((v[i][j] - mean) * rstd);
        if (w != nullptr) {
          float wv[8];
          load8(w + vi * 8, wv);
#pragma unroll
          for (int j = 0; j < 8; ++j) y[j] *= wv[j];
        }
        if (b != nullptr) {
          float bv[8];
          load8(b + vi * 8, bv);
#pragma unroll
          for (int j = 0; j < 8; ++j) y[j] += bv[j];
        }
        if (res != nullptr) {
          float rv[8];
          load8(res + static_cast<size_t>(row) * D + vi * 8, rv);
#pragma unroll
          for (int j = 0; j < 8; ++j) y[j] = round_bf16(y[j]) + rv[j];
        }
        store8(out + static_cast<size_t>(row) * D + vi * 8, y);
      }
    }
  }
}

// dx = [dres +] rstd * (g - mean(g) - xhat * mean(g * xhat)),  g = dy * w   (RMS: the mean(g) term is absent)
template <bool RMS>
__global__ void __launch_bounds__(NT) norm_bwd_kernel(const bf16* __restrict__ dy, const bf16* __restrict__ x,
                                                      const bf16* __restrict__ w, const float* __restrict__ rstd_in,
                                                      const float* __restrict__ mean_in, const bf16* __restrict__ dres,
                                                      bf16* __restrict__ dx, float* __restrict__ dw_part,
                                                      float* __restrict__ db_part, int M, int D, int ldx, int lddx) {
  __shared__ float red[32];
  const int nvec = D >> 3;
  float dw_acc[MAXV][8], db_acc[MAXV][8];
#pragma unroll
  for (int i = 0; i < MAXV; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) dw_acc[i][j] = db_acc[i][j] = 0.f;

  for (int row = blockIdx.x; row < M; row += gridDim.x) {
    const float rstd = rstd_in[row];
    const float mean = RMS ? 0.f : mean_in[row];
    float g[MAXV][8], xh[MAXV][8];
    float sg = 0.f, sgx = 0.f;
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
      const int vi = threadIdx.x + i * NT;
      if (vi < nvec) {
        float dyv[8], xv[8];
        load8(dy + static_cast<size_t>(row) * D + vi * 8, dyv);
        load8(x + static_cast<size_t>(row) * ldx + vi * 8, xv);
        float wv[8];
        if (w != nullptr) load8(w + vi * 8, wv);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          xh[i][j] = (xv[j] - mean) * rstd;
          dw_acc[i][j] += dyv[j] * round_bf16(xh[i][j]);
          db_acc[i][j] += dyv[j];
          g[i][j] = (w != nullptr) ? dyv[j] * wv[j] : dyv[j];
          sg += g[i][j];
          sgx += g[i][j] * xh[i][j];
        }
      }
    }
    sgx = block_sum(sgx, red) / D;
    if (!RMS) sg = block_sum(sg, red) / D;
    else sg = 0.f;
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
      const int vi = threadIdx.x + i * NT;
      if (vi < nvec) {
        float o[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) o[j] = rstd * (g[i][j] - sg - xh[i][j] * sgx);
        if (dres != nullptr) {
          float rv[8];
          load8(dres + static_cast<size_t>(row) * D + vi * 8, rv);
#pragma unroll
          for (int j = 0; j < 8; ++j) o[j] += rv[j];
        }
        store8(dx + static_cast<size_t>(row) * lddx + vi * 8, o);
      }
    }
  }
  if (dw_part != nullptr) {
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
      const int vi = threadIdx.x + i * NT;
      if (vi < nvec) {
        float* p = dw_part + static_cast<size_t>(blockIdx.x) * D + vi * 8;
        *reinterpret_cast<float4*>(p) = make_float4(dw_acc[i][0], dw_acc[i][1], dw_acc[i][2], dw_acc[i][3]);
        *reinterpret_cast<float4*>(p + 4) = make_float4(dw_acc[i][4], dw_acc[i][5], dw_acc[i][6], dw_acc[i][7]);
        if (db_part != nullptr) {
          float* q = db_part + static_cast<size_t>(blockIdx.x) * D + vi * 8;
          *reinterpret_cast<float4*>(q) = make_float4(db_acc[i][0], db_acc[i][1], db_acc[i][2], db_acc[i][3]);
          *reinterpret_cast<float4*>(q + 4) = make_float4(db_acc[i][4], db_acc[i][5], db_acc[i][6], db_acc[i][7]);
        }
      }
    }
  }
}

// out[d] (+)= sum_p part[p, d]
__global__ void reduce_rows_f32_kernel(const float* __restrict__ part, int nparts, int D, float* __restrict__ out,
                                       int accumulate) {
  const int d = blockIdx.x * blockDim.x + threadIdx.x;
  if (d >= D) return;
  float s = 0.f;
  for (int p = 0; p < nparts; ++p) s += part[static_cast<size_t>(p) * D + d];
  out[d] = accumulate ? out[d] + s : s;
}

}  // namespace
}  // namespace ob

extern "C" int ob_norm_rows_per_launch(int M) { return M < 1184 ? M : 1184; }  // 148 SMs x 8 CTAs

extern "C" int ob_norm_fwd(const void* x, const void* res, const void* w, const void* b, void* out, float* rstd,
                           float* mean, int M, int D, int ldx, float eps, int is_rms, cudaStream_t stream) {
  using namespace ob;
  if (M <= 0) return 0;
  if (D % 8 != 0 || D > 8 * NT * MAXV || ldx % 8 != 0) return -1;
  const int grid = M < 148 * 8 ? M : 148 * 8;
  if (is_rms)
    norm_fwd_kernel<true><<<grid, NT, 0, stream>>>((const bf16*)x, (const bf16*)res, (const bf16*)w, (const bf16*)b,
                                                   (bf16*)out, rstd, mean, M, D, ldx, eps);
  else
    norm_fwd_kernel<false><<<grid, NT, 0, stream>>>((const bf16*)x, (const bf16*)res, (const bf16*)w, (const bf16*)b,
                                                    (bf16*)out, rstd, mean, M, D, ldx, eps);
  return cudaGetLastError() == cudaSuccess ? 0 : -11;
}

// `dw_part` / `db_part` are scratch matrices of ob_norm_rows_per_launch(M) x D floats (may be null when the norm
// has no affine parameters).  Returns the number of partial rows written (> 0) or a negative error.
extern "C" int ob_norm_bwd(const void* dy, const void* x, const void* w, const float* rstd, const float* mean,
                           const void* dres, void* dx, float* dw_part, float* db_part, int M, int D, int ldx, int lddx,
                           int is_rms, cudaStream_t stream) {
  using namespace ob;
  if (M <= 0) return 0;
  if (D % 8 != 0 || D > 8 * NT * MAXV || ldx % 8 != 0 || lddx % 8 != 0) return -1;
  const int grid = ob_norm_rows_per_launch(M);
  if (is_rms)
    norm_bwd_kernel<true><<<grid, NT, 0, stream>>>((const bf16*)dy, (const bf16*)x, (const bf16*)w, rstd, mean,
                                                   (const bf16*)dres, (bf16*)dx, dw_part, db_part, M, D, ldx, lddx);
  else
    norm_bwd_kernel<false><<<grid, NT, 0, stream>>>((const bf16*)dy, (const bf16*)x, (const bf16*)w, rstd, mean,
                                                    (const bf16*)dres, (bf16*)dx, dw_part, db_part, M, D, ldx, lddx);
  return cudaGetLastError() == cudaSuccess ? grid : -11;
}

extern "C" int ob_reduce_rows_f32(const float* part, int nparts, int D, float* out, int accumulate,
                                  cudaStream_t stream) {
  using namespace ob;
  if (D <= 0 || nparts <= 0) return 0;
  reduce_rows_f32_kernel<<<(D + 255) / 256, 256, 0, stream>>>(part, nparts, D, out, accumulate);
  return cudaGetLastError() == cudaSuccess ? 0 : -11;
}

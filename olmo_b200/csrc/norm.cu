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

__device__ __forceinline__ void unpack8(const uint4& u, float (&f)[8]) {
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
// Backward.  NV = 16-byte vectors per thread (the CTA has D / (8 * NV) threads, at most 512), BIAS = also reduce db.
// Keeping NV small (1 for D <= 4096) holds the kernel near 64 registers so that several CTAs share an SM and the loads
// of different rows overlap; with one large CTA per SM the per-row reduction latency was the bound.
template <bool RMS, int NV, bool BIAS>
__global__ void __launch_bounds__(512) norm_bwd_kernel(const bf16* __restrict__ dy, const bf16* __restrict__ x,
                                                       const bf16* __restrict__ w, const float* __restrict__ rstd_in,
                                                       const float* __restrict__ mean_in, const bf16* __restrict__ dres,
                                                       bf16* __restrict__ dx, float* __restrict__ dw_part,
                                                       float* __restrict__ db_part, int M, int D, int ldx, int lddx) {
  __shared__ float red[32];
  const int nvec = D >> 3;
  const int nt = blockDim.x;
  float dw_acc[NV][8], db_acc[BIAS ? NV : 1][8];
  float wv[NV][8];
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int vi = threadIdx.x + i * nt;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      dw_acc[i][j] = 0.f;
      if (BIAS) db_acc[i][j] = 0.f;
      wv[i][j] = 1.f;
    }
    if (w != nullptr && vi < nvec) load8(w + vi * 8, wv[i]);
  }

  // The raw vectors of the next row are fetched before this row's reductions, so that a CTA always has two rows of
  // loads in flight (the block-wide sums would otherwise serialise memory latency and synchronisation).
  uint4 dy_raw[NV], x_raw[NV];
  {
    const int row = blockIdx.x;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int vi = threadIdx.x + i * nt;
      if (row < M && vi < nvec) {
        dy_raw[i] = *reinterpret_cast<const uint4*>(dy + static_cast<size_t>(row) * D + vi * 8);
        x_raw[i] = *reinterpret_cast<const uint4*>(x + static_cast<size_t>(row) * ldx + vi * 8);
      }
    }
  }
  for (int row = blockIdx.x; row < M; row += gridDim.x) {
    const float rstd = rstd_in[row];
    const float mean = RMS ? 0.f : mean_in[row];
    float g[NV][8], xh[NV][8];
    float sg = 0.f, sgx = 0.f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int vi = threadIdx.x + i * nt;
      if (vi < nvec) {
        float dyv[8], xv[8];
        unpack8(dy_raw[i], dyv);
        unpack8(x_raw[i], xv);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          xh[i][j] = (xv[j] - mean) * rstd;
          dw_acc[i][j] += dyv[j] * round_bf16(xh[i][j]);
          if (BIAS) db_acc[i][j] += dyv[j];
          g[i][j] = dyv[j] * wv[i][j];
          sg += g[i][j];
          sgx += g[i][j] * xh[i][j];
        }
      }
    }
    const int next = row + gridDim.x;
    uint4 res_raw[NV];
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int vi = threadIdx.x + i * nt;
      if (vi < nvec) {
        if (dres != nullptr) res_raw[i] = *reinterpret_cast<const uint4*>(dres + static_cast<size_t>(row) * D + vi * 8);
        if (next < M) {
          dy_raw[i] = *reinterpret_cast<const uint4*>(dy + static_cast<size_t>(next) * D + vi * 8);
          x_raw[i] = *reinterpret_cast<const uint4*>(x + static_cast<size_t>(next) * ldx + vi * 8);
        }
      }
    }
    sgx = block_sum(sgx, red) / D;
    if (!RMS) sg = block_sum(sg, red) / D;
    else sg = 0.f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int vi = threadIdx.x + i * nt;
      if (vi < nvec) {
        float o[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) o[j] = rstd * (g[i][j] - sg - xh[i][j] * sgx);
        if (dres != nullptr) {
          float rv[8];
          unpack8(res_raw[i], rv);
#pragma unroll
          for (int j = 0; j < 8; ++j) o[j] += rv[j];
        }
        store8(dx + static_cast<size_t>(row) * lddx + vi * 8, o);
      }
    }
  }
  if (dw_part != nullptr) {
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int vi = threadIdx.x + i * nt;
      if (vi < nvec) {
        float* p = dw_part + static_cast<size_t>(blockIdx.x) * D + vi * 8;
        *reinterpret_cast<float4*>(p) = make_float4(dw_acc[i][0], dw_acc[i][1], dw_acc[i][2], dw_acc[i][3]);
        *reinterpret_cast<float4*>(p + 4) = make_float4(dw_acc[i][4], dw_acc[i][5], dw_acc[i][6], dw_acc[i][7]);
        if (BIAS) {
          float* q = db_part + static_cast<size_t>(blockIdx.x) * D + vi * 8;
          *reinterpret_cast<float4*>(q) = make_float4(db_acc[i][0], db_acc[i][1], db_acc[i][2], db_acc[i][3]);
          *reinterpret_cast<float4*>(q + 4) = make_float4(db_acc[i][4], db_acc[i][5], db_acc[i][6], db_acc[i][7]);
        }
      }
    }
  }
}

template <bool RMS, int NV>
void launch_norm_bwd(int grid, int threads, cudaStream_t stream, const bf16* dy, const bf16* x, const bf16* w, const float* rstd,
                     const float* mean, const bf16* dres, bf16* dx, float* dw_part, float* db_part, int M, int D, int ldx, int lddx) {
  if (db_part != nullptr && dw_part != nullptr)
    norm_bwd_kernel<RMS, NV, true><<<grid, threads, 0, stream>>>(dy, x, w, rstd, mean, dres, dx, dw_part, db_part, M, D, ldx, lddx);
  else
    norm_bwd_kernel<RMS, NV, false><<<grid, threads, 0, stream>>>(dy, x, w, rstd, mean, dres, dx, dw_part, nullptr, M, D, ldx, lddx);
}


// out[d] (+)= sum_p part[p, d].  A block owns 32 columns; its 256 threads are 8 row lanes x 32 columns, every row lane
// sums each eighth row with four independent accumulators (a warp reads 128 contiguous bytes per row), and the eight
// lane sums are added in lane order, so the result does not depend on scheduling.
constexpr int RR_COLS = 32, RR_LANES = 8;
__global__ void __launch_bounds__(RR_COLS * RR_LANES)
reduce_rows_f32_kernel(const float* __restrict__ part, int nparts, int D, float* __restrict__ out, int accumulate) {
  __shared__ float lane_sum[RR_LANES][RR_COLS];
  const int c = threadIdx.x & (RR_COLS - 1), rl = threadIdx.x >> 5;
  const int d = blockIdx.x * RR_COLS + c;
  float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
  if (d < D) {
    int p = rl;
    for (; p + 3 * RR_LANES < nparts; p += 4 * RR_LANES) {
      a0 += part[static_cast<size_t>(p) * D + d];
      a1 += part[static_cast<size_t>(p + RR_LANES) * D + d];
      a2 += part[static_cast<size_t>(p + 2 * RR_LANES) * D + d];
      a3 += part[static_cast<size_t>(p + 3 * RR_LANES) * D + d];
    }
    for (; p < nparts; p += RR_LANES) a0 += part[static_cast<size_t>(p) * D + d];
  }
  lane_sum[rl][c] = (a0 + a1) + (a2 + a3);
  __syncthreads();
  if (rl == 0 && d < D) {
    float s = 0.f;
#pragma unroll
    for (int l = 0; l < RR_LANES; ++l) s += lane_sum[l][c];
    out[d] = accumulate ? out[d] + s : s;
  }
}

}  // namespace
}  // namespace ob

extern "C" int ob_norm_rows_per_launch(int M) { return M < 592 ? M : 592; }  // 148 SMs x 4 CTAs of the backward kernel

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
  // one vector per thread up to D = 4096 (<= 512 threads), two up to 8192
  const int nvec = D / 8;
  const int nv = nvec <= 512 ? 1 : (nvec <= 1024 ? 2 : 4);
  int threads = (nvec + nv - 1) / nv;
  threads = ((threads + 31) / 32) * 32;
  const bf16 *dyp = (const bf16*)dy, *xp = (const bf16*)x, *wp = (const bf16*)w, *rp = (const bf16*)dres;
  bf16* dxp = (bf16*)dx;
#define OB_NORM_BWD(RMS_, NV_) launch_norm_bwd<RMS_, NV_>(grid, threads, stream, dyp, xp, wp, rstd, mean, rp, dxp, dw_part, db_part, M, D, ldx, lddx)
  if (is_rms) {
    if (nv == 1) OB_NORM_BWD(true, 1); else if (nv == 2) OB_NORM_BWD(true, 2); else OB_NORM_BWD(true, 4);
  } else {
    if (nv == 1) OB_NORM_BWD(false, 1); else if (nv == 2) OB_NORM_BWD(false, 2); else OB_NORM_BWD(false, 4);
  }
#undef OB_NORM_BWD
  return cudaGetLastError() == cudaSuccess ? grid : -11;
}

extern "C" int ob_reduce_rows_f32(const float* part, int nparts, int D, float* out, int accumulate,
                                  cudaStream_t stream) {
  using namespace ob;
  if (D <= 0 || nparts <= 0) return 0;
  reduce_rows_f32_kernel<<<(D + RR_COLS - 1) / RR_COLS, RR_COLS * RR_LANES, 0, stream>>>(part, nparts, D, out, accumulate);
  return cudaGetLastError() == cudaSuccess ? 0 : -11;
}

// QK-norm + rotary embedding, fused, forward and backward.
//
// Input is the fused projection qkv[M, ldq] = [q (Wq cols) | k (Wk cols) | v].  Per token row:
//   q <- rope(rmsnorm(q) * wq),  k <- rope(rmsnorm(k) * wk)        (the norm spans all heads jointly)
// and the result is written to out[M, ldo] = [q | k]; v is read by attention from qkv directly.  With clip_qkv
// (OLMo-1) all three parts are clamped first and the clamped v is written to out as a third part, so that the
// un-clamped projection survives for the backward mask.
// RoPE is the rotate-half form: within a head, element j < hd/2 pairs with j + hd/2;
//   a' = a cos - b sin,  b' = b cos + a sin   in fp32, rounded to bf16 once.
// Each thread owns pairs of 8-element vectors (a-vector and its partner), so rotation needs no exchange.
#include "common.cuh"
#include "api.h"

namespace ob {
namespace {

constexpr int NT = 256;
constexpr int MAXP = 2;  // vector pairs per thread and per part -> width <= 8192

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
__device__ __forceinline__ void ldf8(const float* p, float (&f)[8]) {
  const float4 a = *reinterpret_cast<const float4*>(p);
  const float4 b = *reinterpret_cast<const float4*>(p + 4);
  f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w;
  f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
}
__device__ __forceinline__ float rbf(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }
__device__ __forceinline__ float clampf(float v, float c) { return fminf(fmaxf(v, -c), c); }

struct PartGeom {
  int col0;   // first column of the part inside qkv
  int width;  // Wq or Wk
};

// One part (q or k) of one row, forward.  NP = vector pairs per thread.
template <bool NORM, bool ROPE, int NP>
__device__ __forceinline__ void part_fwd(const bf16* __restrict__ in, bf16* __restrict__ out, const bf16* __restrict__ w,
                                         const float* __restrict__ cosr, const float* __restrict__ sinr, int width,
                                         int hd, float eps, float clip, float* rstd_out, float* red) {
  const int half = hd >> 1;
  const int ppv = half >> 3;  // vector pairs per head
  const int npairs = width >> 4;
  float a[NP][8], b[NP][8];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < NP; ++i) {
    const int p = threadIdx.x + i * NT;
    if (p < npairs) {
      const int col = (p / ppv) * hd + (p % ppv) * 8;
      ld8(in + col, a[i]);
      ld8(in + col + half, b[i]);
      if (clip > 0.f) {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          a[i][j] = clampf(a[i][j], clip);
          b[i][j] = clampf(b[i][j], clip);
        }
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) ss += a[i][j] * a[i][j] + b[i][j] * b[i][j];
    }
  }
  float rstd = 1.f;
  if (NORM) {
    ss = block_sum(ss, red);
    rstd = rsqrtf(ss / width + eps);
    if (threadIdx.x == 0 && rstd_out != nullptr) *rstd_out = rstd;
  }
#pragma unroll
  for (int i = 0; i < NP; ++i) {
    const int p = threadIdx.x + i * NT;
    if (p < npairs) {
      const int jj = (p % ppv) * 8;
      const int col = (p / ppv) * hd + jj;
      if (NORM) {
        float wa[8], wb[8];
        if (w != nullptr) {
          ld8(w + col, wa);
          ld8(w + col + half, wb);
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          a[i][j] = rbf(a[i][j] * rstd);
          b[i][j] = rbf(b[i][j] * rstd);
          if (w != nullptr) {
            a[i][j] = rbf(a[i][j] * wa[j]);
            b[i][j] = rbf(b[i][j] * wb[j]);
          }
        }
      }
      float oa[8], ob_[8];
      if (ROPE) {
        float c[8], s[8];
        ldf8(cosr + jj, c);
        ldf8(sinr + jj, s);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          oa[j] = a[i][j] * c[j] - b[i][j] * s[j];
          ob_[j] = b[i][j] * c[j] + a[i][j] * s[j];
        }
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          oa[j] = a[i][j];
          ob_[j] = b[i][j];
        }
      }
      st8(out + col, oa);
      st8(out + col + half, ob_);
    }
  }
}

// grid = (row walkers, 2): blockIdx.y == 0 handles the q part of a row, 1 the k part (and the clamped v copy).  The two
// parts are independent (separate norms), so giving each its own CTA halves the per-thread state and doubles the number
// of rows in flight.
template <bool NORM, bool ROPE, int NP>
__global__ void __launch_bounds__(NT)
qk_fwd_kernel(const bf16* __restrict__ qkv, bf16* __restrict__ qk_out, const bf16* __restrict__ wq, const bf16* __restrict__ wk,
              const float* __restrict__ cos_t, const float* __restrict__ sin_t, float* __restrict__ rstd_q,
              float* __restrict__ rstd_k, int M, int T, int pos_offset, int Wq, int Wk, int hd, int ldq, int ldo,
              float eps, float clip) {
  __shared__ float red[32];
  const int half = hd >> 1;
  const bool is_k = blockIdx.y == 1;
  const int col0 = is_k ? Wq : 0;
  const int width = is_k ? Wk : Wq;
  const bf16* w = is_k ? wk : wq;
  float* rstd_out = is_k ? rstd_k : rstd_q;
  for (int row = blockIdx.x; row < M; row += gridDim.x) {
    const int t = row % T + pos_offset;
    const float* cr = cos_t + static_cast<size_t>(t) * half;
    const float* sr = sin_t + static_cast<size_t>(t) * half;
    const bf16* in = qkv + static_cast<size_t>(row) * ldq;
    bf16* out = qk_out + static_cast<size_t>(row) * ldo;
    part_fwd<NORM, ROPE, NP>(in + col0, out + col0, w, cr, sr, width, hd, eps, clip, rstd_out ? rstd_out + row : nullptr, red);
    if (is_k && clip > 0.f) {  // clamped v becomes the third part of the output
      const bf16* v = in + Wq + Wk;
      bf16* vo = out + Wq + Wk;
      for (int i = threadIdx.x; i < (Wk >> 3); i += NT) {
        float f[8];
        ld8(v + i * 8, f);
#pragma unroll
        for (int j = 0; j < 8; ++j) f[j] = clampf(f[j], clip);
        st8(vo + i * 8, f);
      }
    }
  }
}

// One part of one row, backward, in place on the gradient buffer.
template <bool NORM, bool ROPE, int NP>
__device__ __forceinline__ void part_bwd(const bf16* __restrict__ in, bf16* __restrict__ grad, const bf16* __restrict__ w,
                                         const float* __restrict__ cosr, const float* __restrict__ sinr, int width,
                                         int hd, float clip, float rstd, float (&dw_a)[NP][8], float (&dw_b)[NP][8],
                                         float* red) {
  const int half = hd >> 1;
  const int ppv = half >> 3;
  const int npairs = width >> 4;
  float ga[NP][8], gb[NP][8], xa[NP][8], xb[NP][8];
  float sgx = 0.f;
#pragma unroll
  for (int i = 0; i < NP; ++i) {
    const int p = threadIdx.x + i * NT;
    if (p < npairs) {
      const int jj = (p % ppv) * 8;
      const int col = (p / ppv) * hd + jj;
      float da[8], db[8];
      ld8(grad + col, da);
      ld8(grad + col + half, db);
      if (ROPE) {
        float c[8], s[8];
        ldf8(cosr + jj, c);
        ldf8(sinr + jj, s);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          ga[i][j] = da[j] * c[j] + db[j] * s[j];
          gb[i][j] = db[j] * c[j] - da[j] * s[j];
        }
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          ga[i][j] = da[j];
          gb[i][j] = db[j];
        }
      }
      ld8(in + col, xa[i]);
      ld8(in + col + half, xb[i]);
      if (NORM) {
        float wa[8], wb[8];
        if (w != nullptr) {
          ld8(w + col, wa);
          ld8(w + col + half, wb);
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float ca = (clip > 0.f) ? clampf(xa[i][j], clip) : xa[i][j];
          const float cb = (clip > 0.f) ? clampf(xb[i][j], clip) : xb[i][j];
          const float ha = ca * rstd, hb = cb * rstd;
          dw_a[i][j] += ga[i][j] * rbf(ha);
          dw_b[i][j] += gb[i][j] * rbf(hb);
          if (w != nullptr) {
            ga[i][j] *= wa[j];
            gb[i][j] *= wb[j];
          }
          sgx += ga[i][j] * ha + gb[i][j] * hb;
        }
      }
    }
  }
  if (NORM) sgx = block_sum(sgx, red) / width;
#pragma unroll
  for (int i = 0; i < NP; ++i) {
    const int p = threadIdx.x + i * NT;
    if (p < npairs) {
      const int col = (p / ppv) * hd + (p % ppv) * 8;
      float oa[8], ob_[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        float va = ga[i][j], vb = gb[i][j];
        if (NORM) {
          const float ca = (clip > 0.f) ? clampf(xa[i][j], clip) : xa[i][j];
          const float cb = (clip > 0.f) ? clampf(xb[i][j], clip) : xb[i][j];
          va = rstd * (va - ca * rstd * sgx);
          vb = rstd * (vb - cb * rstd * sgx);
        }
        if (clip > 0.f) {  // clamp passes gradient only strictly inside (-clip, clip)
          if (fabsf(xa[i][j]) > clip) va = 0.f;
          if (fabsf(xb[i][j]) > clip) vb = 0.f;
        }
        oa[j] = va;
        ob_[j] = vb;
      }
      st8(grad + col, oa);
      st8(grad + col + half, ob_);
    }
  }
}

template <bool NORM, bool ROPE, int NP>
__global__ void __launch_bounds__(NT, NP == 1 ? 3 : 1)
qk_bwd_kernel(const bf16* __restrict__ qkv, bf16* __restrict__ dqkv, const bf16* __restrict__ wq,
              const bf16* __restrict__ wk, const float* __restrict__ cos_t, const float* __restrict__ sin_t,
              const float* __restrict__ rstd_q, const float* __restrict__ rstd_k, float* __restrict__ dwq_part,
              float* __restrict__ dwk_part, int M, int T, int pos_offset, int Wq, int Wk, int hd, int ldq, float clip) {
  __shared__ float red[32];
  const int half = hd >> 1;
  const int ppv = half >> 3;
  const bool is_k = blockIdx.y == 1;
  const int col0 = is_k ? Wq : 0;
  const int width = is_k ? Wk : Wq;
  const bf16* w = is_k ? wk : wq;
  const float* rstd_in = is_k ? rstd_k : rstd_q;
  float* dw_part = is_k ? dwk_part : dwq_part;
  float dwa[NP][8], dwb[NP][8];
#pragma unroll
  for (int i = 0; i < NP; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) dwa[i][j] = dwb[i][j] = 0.f;

  for (int row = blockIdx.x; row < M; row += gridDim.x) {
    const int t = row % T + pos_offset;
    const float* cr = cos_t + static_cast<size_t>(t) * half;
    const float* sr = sin_t + static_cast<size_t>(t) * half;
    const bf16* in = qkv + static_cast<size_t>(row) * ldq;
    bf16* g = dqkv + static_cast<size_t>(row) * ldq;
    part_bwd<NORM, ROPE, NP>(in + col0, g + col0, w, cr, sr, width, hd, clip, NORM ? rstd_in[row] : 1.f, dwa, dwb, red);
    if (is_k && clip > 0.f) {  // clamp passes no gradient where the projection was outside [-clip, clip]
      const bf16* v = in + Wq + Wk;
      bf16* dv = g + Wq + Wk;
      for (int i = threadIdx.x; i < (Wk >> 3); i += NT) {
        float f[8], d[8];
        ld8(v + i * 8, f);
        ld8(dv + i * 8, d);
#pragma unroll
        for (int j = 0; j < 8; ++j)
          if (fabsf(f[j]) > clip) d[j] = 0.f;
        st8(dv + i * 8, d);
      }
    }
  }
  if (NORM && dw_part != nullptr) {
#pragma unroll
    for (int i = 0; i < NP; ++i) {
      const int p = threadIdx.x + i * NT;
      const int col = (p / ppv) * hd + (p % ppv) * 8;
      if (p < (width >> 4)) {
        float* o = dw_part + static_cast<size_t>(blockIdx.x) * width + col;
        *reinterpret_cast<float4*>(o) = make_float4(dwa[i][0], dwa[i][1], dwa[i][2], dwa[i][3]);
        *reinterpret_cast<float4*>(o + 4) = make_float4(dwa[i][4], dwa[i][5], dwa[i][6], dwa[i][7]);
        *reinterpret_cast<float4*>(o + half) = make_float4(dwb[i][0], dwb[i][1], dwb[i][2], dwb[i][3]);
        *reinterpret_cast<float4*>(o + half + 4) = make_float4(dwb[i][4], dwb[i][5], dwb[i][6], dwb[i][7]);
      }
    }
  }
}

}  // namespace
}  // namespace ob

extern "C" int ob_qk_rows_per_launch(int M) { return M < 592 ? M : 592; }  // x 2 parts = 8 CTAs per SM

static int qk_check(int Wq, int Wk, int hd, int ldq) {
  if (hd % 16 != 0 || Wq % hd != 0 || Wk % hd != 0 || ldq % 8 != 0) return -1;
  if (Wq > 16 * ob::NT * ob::MAXP || Wk > 16 * ob::NT * ob::MAXP) return -1;
  return 0;
}

extern "C" int ob_qk_norm_rope_fwd(const void* qkv, void* qk_out, const void* wq, const void* wk, const float* cos_t,
                                   const float* sin_t, float* rstd_q, float* rstd_k, int M, int T, int pos_offset,
                                   int Wq, int Wk, int hd, int ldq, int ldo, float eps, float clip, int do_norm,
                                   int do_rope, cudaStream_t stream) {
  using namespace ob;
  if (M <= 0) return 0;
  if (qk_check(Wq, Wk, hd, ldq) != 0 || ldo % 8 != 0) return -1;
  const int grid = ob_qk_rows_per_launch(M);
  const dim3 grid2(grid, 2);
  const bool one = (Wq > Wk ? Wq : Wk) <= 16 * NT;  // one vector pair per thread suffices
#define OB_QK_FWD(N_, R_)                                                                                              \
  do {                                                                                                                 \
    if (one)                                                                                                           \
      qk_fwd_kernel<N_, R_, 1><<<grid2, NT, 0, stream>>>((const bf16*)qkv, (bf16*)qk_out, (const bf16*)wq, (const bf16*)wk, cos_t, \
                                                         sin_t, rstd_q, rstd_k, M, T, pos_offset, Wq, Wk, hd, ldq, ldo, eps, clip); \
    else                                                                                                               \
      qk_fwd_kernel<N_, R_, MAXP><<<grid2, NT, 0, stream>>>((const bf16*)qkv, (bf16*)qk_out, (const bf16*)wq, (const bf16*)wk,     \
                                                            cos_t, sin_t, rstd_q, rstd_k, M, T, pos_offset, Wq, Wk, hd, ldq, ldo,  \
                                                            eps, clip);                                                \
  } while (0)
  if (do_norm && do_rope) OB_QK_FWD(true, true);
  else if (do_norm) OB_QK_FWD(true, false);
  else if (do_rope) OB_QK_FWD(false, true);
  else OB_QK_FWD(false, false);
#undef OB_QK_FWD
  return cudaGetLastError() == cudaSuccess ? 0 : -11;
}

// In place on dqkv[M, ldq]: on entry its q|k columns hold gradients w.r.t. the rotated, normalised q and k and its
// v columns the gradient w.r.t. v; on exit all columns hold gradients w.r.t. the projection output.
// dwq_part / dwk_part: scratch of ob_qk_rows_per_launch(M) x Wq (x Wk) floats; returns the partial-row count.
extern "C" int ob_qk_norm_rope_bwd(const void* qkv, void* dqkv, const void* wq, const void* wk, const float* cos_t,
                                   const float* sin_t, const float* rstd_q, const float* rstd_k, float* dwq_part,
                                   float* dwk_part, int M, int T, int pos_offset, int Wq, int Wk, int hd, int ldq,
                                   float clip, int do_norm, int do_rope, cudaStream_t stream) {
  using namespace ob;
  if (M <= 0) return 0;
  if (qk_check(Wq, Wk, hd, ldq) != 0) return -1;
  const int grid = ob_qk_rows_per_launch(M);
  const dim3 grid2(grid, 2);
  const bool one = (Wq > Wk ? Wq : Wk) <= 16 * NT;
#define OB_QK_BWD(N_, R_)                                                                                              \
  do {                                                                                                                 \
    if (one)                                                                                                           \
      qk_bwd_kernel<N_, R_, 1><<<grid2, NT, 0, stream>>>((const bf16*)qkv, (bf16*)dqkv, (const bf16*)wq, (const bf16*)wk, cos_t,   \
                                                         sin_t, rstd_q, rstd_k, dwq_part, dwk_part, M, T, pos_offset, Wq, Wk, hd, \
                                                         ldq, clip);                                                   \
    else                                                                                                               \
      qk_bwd_kernel<N_, R_, MAXP><<<grid2, NT, 0, stream>>>((const bf16*)qkv, (bf16*)dqkv, (const bf16*)wq, (const bf16*)wk,       \
                                                            cos_t, sin_t, rstd_q, rstd_k, dwq_part, dwk_part, M, T, pos_offset,    \
                                                            Wq, Wk, hd, ldq, clip);                                    \
  } while (0)
  if (do_norm && do_rope) OB_QK_BWD(true, true);
  else if (do_norm) OB_QK_BWD(true, false);
  else if (do_rope) OB_QK_BWD(false, true);
  else OB_QK_BWD(false, false);
#undef OB_QK_BWD
  return cudaGetLastError() == cudaSuccess ? grid : -11;
}

// Single-token decode step against preallocated key/value windows (serving): two bandwidth-bound kernels that replace the
// dozens of small element-wise launches a module-level decode step makes per block.
//
//   decode_qkv        two CTAs per sequence (query; key and value): optional clip of the fused q|k|v projection, optional RMS norm of q and k over
//                     their full widths (the OLMo-2 "QK-norm"), rotary embedding of q and k at the sequence's own token
//                     index, q written out, the new key and value written into the window at the shared write column.
//   decode_attention  one CTA per (query head, sequence): softmax(q·Kᵀ·scale + bias)·V over the first `length` columns of
//                     the window; keys are stored already rotated.  Each warp streams every fourth column with one
//                     coalesced 256-byte load per key and per value, keeps a running (max, sum, output) triple, and the
//                     four warps are merged through shared memory.  Grouped-query attention reads the shared key head.
//
// Everything that changes from step to step (write column, per-sequence token index, bias) is read from device memory, so
// a captured CUDA graph of the step can be replayed.  Indices read from memory are clamped before use.
#include "common.cuh"
#include "api.h"

namespace ob {
namespace {

constexpr int DQ_THREADS = 256;
constexpr int DA_WARPS = 4;  // eight warps per CTA measured no faster (48 vs 45 us at 32 x 32 x 256)
constexpr int DA_HD = 128;

__device__ __forceinline__ void load8(const bf16* p, float (&f)[8]) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 v = unpack_bf16x2(w[i]);
    f[2 * i] = v.x;
    f[2 * i + 1] = v.y;
  }
}

__device__ __forceinline__ void store8(bf16* p, const float (&f)[8]) {
  uint4 u;
  u.x = pack_bf16x2(f[0], f[1]);
  u.y = pack_bf16x2(f[2], f[3]);
  u.z = pack_bf16x2(f[4], f[5]);
  u.w = pack_bf16x2(f[6], f[7]);
  *reinterpret_cast<uint4*>(p) = u;
}

// qkv [R, Wq + 2 Wk]; q_out [R, Wq]; caches [R, Hkv, window, hd]; cos/sin [table_len, hd/2] fp32.
// Grid (R, 2): CTA (r, 0) handles the query of sequence r, CTA (r, 1) its key and value, so the two row reductions of
// the QK-norm run side by side.
__global__ void __launch_bounds__(DQ_THREADS)
decode_qkv_kernel(const bf16* __restrict__ qkv, const bf16* __restrict__ wq, const bf16* __restrict__ wk, const float* __restrict__ cos_t,
                  const float* __restrict__ sin_t, const long long* __restrict__ rope_pos, const long long* __restrict__ write_col,
                  bf16* __restrict__ q_out, bf16* __restrict__ k_cache, bf16* __restrict__ v_cache, int Wq, int Wk, int hd, int window,
                  int table_len, float eps, float clip, int qk_norm, int rope) {
  extern __shared__ float row[];  // max(Wq, Wk) floats: this CTA's vector after the optional clip
  __shared__ float scratch[32];
  const int r = blockIdx.x;
  const bool is_q = blockIdx.y == 0;
  const int width = is_q ? Wq : Wk;
  const bf16* src = qkv + static_cast<size_t>(r) * (Wq + 2 * Wk) + (is_q ? 0 : Wq);
  const bf16* w = is_q ? wq : wk;
  const int col = static_cast<int>(min(max(write_col[0], 0LL), static_cast<long long>(window - 1)));
  const int tok = static_cast<int>(min(max(rope_pos[r], 0LL), static_cast<long long>(table_len - 1)));
  const int hkv = Wk / hd;
  const int half = hd >> 1;

  float ss = 0.f;
  for (int c = threadIdx.x; c < width / 8; c += DQ_THREADS) {
    float f[8];
    load8(src + c * 8, f);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      if (clip > 0.f) f[i] = fminf(fmaxf(f[i], -clip), clip);
      row[c * 8 + i] = f[i];
      ss += f[i] * f[i];
    }
  }
  if (!is_q) {  // the value goes to the window as it is (clipped): [r, head, col, :]
    for (int c = threadIdx.x; c < Wk / 8; c += DQ_THREADS) {
      float f[8];
      load8(src + Wk + c * 8, f);
      if (clip > 0.f) {
#pragma unroll
        for (int i = 0; i < 8; ++i) f[i] = fminf(fmaxf(f[i], -clip), clip);
      }
      const int e = c * 8, head = e / hd, d = e % hd;
      store8(v_cache + ((static_cast<size_t>(r) * hkv + head) * window + col) * hd + d, f);
    }
  }
  float rstd = 1.f;
  if (qk_norm) {
    ss = block_sum(ss, scratch);
    rstd = rsqrtf(ss / static_cast<float>(width) + eps);
  }
  __syncthreads();  // `row` complete

  const float* cs = cos_t + static_cast<size_t>(tok) * half;
  const float* sn = sin_t + static_cast<size_t>(tok) * half;
  for (int c = threadIdx.x; c < width / 8; c += DQ_THREADS) {
    const int e0 = c * 8;
    const int d0 = e0 % hd;
    const int partner0 = d0 < half ? e0 + half : e0 - half;
    float wv[8], wp[8], out[8];
    if (qk_norm) {
      load8(w + e0, wv);
      load8(w + partner0, wp);
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      float a = row[e0 + i], b = row[partner0 + i];
      if (qk_norm) {
        a = a * rstd * wv[i];
        b = b * rstd * wp[i];
      }
      if (rope) {
        const int j = (d0 + i) % half;
        const float rot = d0 < half ? -b : b;  // rotate_half: (-second half, first half)
        out[i] = a * cs[j] + rot * sn[j];
      } else {
        out[i] = a;
      }
    }
    if (is_q) {
      store8(q_out + static_cast<size_t>(r) * Wq + e0, out);
    } else {
      const int head = e0 / hd;
      store8(k_cache + ((static_cast<size_t>(r) * hkv + head) * window + col) * hd + d0, out);
    }
  }
}

// q [R, H, 128]; caches [R, Hkv, window, 128]; bias [R, window] (additive, bf16); out [R, H, 128].
__global__ void __launch_bounds__(DA_WARPS * 32)
decode_attention_kernel(const bf16* __restrict__ q, const bf16* __restrict__ k_cache, const bf16* __restrict__ v_cache,
                        const bf16* __restrict__ bias, bf16* __restrict__ out, int H, int Hkv, int window, int length, float scale) {
  __shared__ float s_m[DA_WARPS], s_l[DA_WARPS];
  __shared__ float s_acc[DA_WARPS][DA_HD];
  const int h = blockIdx.x, r = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int hk = h / (H / Hkv);
  const bf16* kbase = k_cache + (static_cast<size_t>(r) * Hkv + hk) * static_cast<size_t>(window) * DA_HD;
  const bf16* vbase = v_cache + (static_cast<size_t>(r) * Hkv + hk) * static_cast<size_t>(window) * DA_HD;
  const bf16* brow = bias + static_cast<size_t>(r) * window;

  // this lane's four dimensions of the query, pre-multiplied by the softmax scale
  float qv[4];
  {
    const uint2 u = *reinterpret_cast<const uint2*>(q + (static_cast<size_t>(r) * H + h) * DA_HD + lane * 4);
    const float2 a = unpack_bf16x2(u.x), b = unpack_bf16x2(u.y);
    qv[0] = a.x * scale; qv[1] = a.y * scale; qv[2] = b.x * scale; qv[3] = b.y * scale;
  }
  float m = -INFINITY, l = 0.f, acc[4] = {0.f, 0.f, 0.f, 0.f};
  constexpr int COLS = 4;  // columns per iteration: eight independent 256-byte loads in flight per warp
  for (int j0 = warp; j0 < length; j0 += DA_WARPS * COLS) {
    uint2 ku[COLS], vu[COLS];
    bool live[COLS];
#pragma unroll
    for (int c = 0; c < COLS; ++c) {
      const int j = j0 + c * DA_WARPS;
      live[c] = j < length;
      ku[c] = live[c] ? *reinterpret_cast<const uint2*>(kbase + static_cast<size_t>(j) * DA_HD + lane * 4) : make_uint2(0u, 0u);
      vu[c] = live[c] ? *reinterpret_cast<const uint2*>(vbase + static_cast<size_t>(j) * DA_HD + lane * 4) : make_uint2(0u, 0u);
    }
    float s[COLS];
#pragma unroll
    for (int c = 0; c < COLS; ++c) {
      const float2 a = unpack_bf16x2(ku[c].x), b = unpack_bf16x2(ku[c].y);
      s[c] = qv[0] * a.x + qv[1] * a.y + qv[2] * b.x + qv[3] * b.y;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
#pragma unroll
      for (int c = 0; c < COLS; ++c) s[c] += __shfl_xor_sync(0xffffffffu, s[c], o);
    }
    float m_new = m;
#pragma unroll
    for (int c = 0; c < COLS; ++c) {
      s[c] = live[c] ? s[c] + __bfloat162float(brow[j0 + c * DA_WARPS]) : -INFINITY;
      m_new = fmaxf(m_new, s[c]);
    }
    const float corr = __expf(m - m_new);  // 0 on the first iteration (m = -inf); column j0 is always live, so m_new is finite
    l *= corr;
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[i] *= corr;
#pragma unroll
    for (int c = 0; c < COLS; ++c) {
      const float p = __expf(s[c] - m_new);
      const float2 a = unpack_bf16x2(vu[c].x), b = unpack_bf16x2(vu[c].y);
      l += p;
      acc[0] += p * a.x;
      acc[1] += p * a.y;
      acc[2] += p * b.x;
      acc[3] += p * b.y;
    }
    m = m_new;
  }
  if (lane == 0) {
    s_m[warp] = m;
    s_l[warp] = l;
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) s_acc[warp][lane * 4 + i] = acc[i];
  __syncthreads();
  if (warp == 0) {
    float mx = -INFINITY;
#pragma unroll
    for (int w = 0; w < DA_WARPS; ++w) mx = fmaxf(mx, s_m[w]);
    float total = 0.f, o[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int w = 0; w < DA_WARPS; ++w) {
      const float f = (s_m[w] == -INFINITY) ? 0.f : __expf(s_m[w] - mx);  // a warp that saw no column contributes nothing
      total += s_l[w] * f;
#pragma unroll
      for (int i = 0; i < 4; ++i) o[i] += s_acc[w][lane * 4 + i] * f;
    }
    const float inv = total > 0.f ? 1.f / total : 0.f;
    uint2 u;
    u.x = pack_bf16x2(o[0] * inv, o[1] * inv);
    u.y = pack_bf16x2(o[2] * inv, o[3] * inv);
    *reinterpret_cast<uint2*>(out + (static_cast<size_t>(r) * H + h) * DA_HD + lane * 4) = u;
  }
}

}  // namespace
}  // namespace ob

extern "C" {

int ob_decode_qkv(const void* qkv, const void* wq, const void* wk, const float* cos_t, const float* sin_t, const long long* rope_pos,
                  const long long* write_col, void* q_out, void* k_cache, void* v_cache, int R, int Wq, int Wk, int hd, int window,
                  int table_len, float eps, float clip, int qk_norm, int rope, cudaStream_t stream) {
  using namespace ob;
  if (R < 1 || hd < 16 || hd % 16 != 0 || Wq % hd != 0 || Wk % hd != 0 || window < 1 || table_len < 1) return -1;
  if (qk_norm && (wq == nullptr || wk == nullptr)) return -1;
  const size_t smem = static_cast<size_t>(Wq > Wk ? Wq : Wk) * sizeof(float);
  if (smem > 96 * 1024) return -1;
  static bool configured = false;
  if (!configured) {
    if (cudaFuncSetAttribute(decode_qkv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 96 * 1024) != cudaSuccess) return -4;
    configured = true;
  }
  decode_qkv_kernel<<<dim3(R, 2), DQ_THREADS, smem, stream>>>(static_cast<const bf16*>(qkv), static_cast<const bf16*>(wq), static_cast<const bf16*>(wk),
                                                     cos_t, sin_t, rope_pos, write_col, static_cast<bf16*>(q_out), static_cast<bf16*>(k_cache),
                                                     static_cast<bf16*>(v_cache), Wq, Wk, hd, window, table_len, eps, clip, qk_norm, rope);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

int ob_decode_attention(const void* q, const void* k_cache, const void* v_cache, const void* bias, void* out, int R, int H, int Hkv, int hd,
                        int window, int length, float scale, cudaStream_t stream) {
  using namespace ob;
  if (hd != DA_HD || R < 1 || H < 1 || Hkv < 1 || H % Hkv != 0 || length < 1 || length > window) return -1;
  const dim3 grid(H, R);
  decode_attention_kernel<<<grid, DA_WARPS * 32, 0, stream>>>(static_cast<const bf16*>(q), static_cast<const bf16*>(k_cache),
                                                              static_cast<const bf16*>(v_cache), static_cast<const bf16*>(bias),
                                                              static_cast<bf16*>(out), H, Hkv, window, length, scale);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

}  // extern "C"

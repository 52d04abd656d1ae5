// Weight-only quantised inference kernels for 2-, 3-, 4- and 8-bit weights with 16-bit activations
// (per-group scale and zero point).  The 4-bit tensor-core paths live in w4a16.cu / w4a16_mma.cu; this file covers the
// other widths the reference's vendored AutoGPTQ kernels serve (its 2/3/4/8-bit vector-matrix products), with one
// template instead of one hand-unrolled kernel per width.
//
// Layout: a row of K weights is a little-endian bit stream, weight k in bits [k*B, (k+1)*B) of the row, stored as
// int32 words: qweight is [N, K*B/32].  A chunk of 32 consecutive weights is therefore exactly B words, whatever B is
// (3-bit weights straddle word boundaries inside a chunk, never across chunks).  scales [N, K/G] bf16 and zeros
// [N, K/G] uint8 as in w4a16.cu; W[n][k] = (q[n][k] - zeros[n][k/G]) * scales[n][k/G]; G is a multiple of 32.
#include "common.cuh"
#include "api.h"

namespace ob {
namespace {

constexpr int WN_WARPS = 8;

// The 32 weights of one chunk (B words) as floats.
template <int B>
__device__ __forceinline__ void unpack_chunk(const uint32_t (&w)[B], float zero, float scale, float (&out)[32]) {
  constexpr uint32_t mask = (B == 32) ? 0xFFFFFFFFu : ((1u << B) - 1u);
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    const int bit = i * B;
    const int word = bit >> 5, shift = bit & 31;
    uint32_t v = w[word] >> shift;
    if (shift + B > 32) v |= w[(word + 1) < B ? (word + 1) : word] << (32 - shift);
    out[i] = (static_cast<float>(v & mask) - zero) * scale;
  }
}

// y[m][n] = sum_k x[m][k] * W[n][k] for 1 <= M <= 8.  One warp per output row; a lane owns chunks of 32 weights strided
// by 32 lanes, so a warp's loads of one iteration cover 32*B consecutive words of the weight row.
template <int B, int M>
__global__ void __launch_bounds__(WN_WARPS * 32) wna16_gemv_kernel(const bf16* __restrict__ x, const uint32_t* __restrict__ qweight,
                                                                    const bf16* __restrict__ scales, const uint8_t* __restrict__ zeros,
                                                                    bf16* __restrict__ y, int N, int K, int group) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int chunks = K / 32;
  const int groups = K / group;
  const size_t row_words = static_cast<size_t>(K) * B / 32;
  for (int n = blockIdx.x * WN_WARPS + warp; n < N; n += gridDim.x * WN_WARPS) {
    const uint32_t* wrow = qweight + static_cast<size_t>(n) * row_words;
    const bf16* srow = scales + static_cast<size_t>(n) * groups;
    const uint8_t* zrow = zeros + static_cast<size_t>(n) * groups;
    float acc[M];
#pragma unroll
    for (int m = 0; m < M; ++m) acc[m] = 0.f;
    for (int c = lane; c < chunks; c += 32) {
      uint32_t w[B];
#pragma unroll
      for (int j = 0; j < B; ++j) w[j] = __ldg(wrow + static_cast<size_t>(c) * B + j);
      const int k0 = c * 32;
      const int g = k0 / group;
      float wf[32];
      unpack_chunk<B>(w, static_cast<float>(zrow[g]), __bfloat162float(srow[g]), wf);
#pragma unroll
      for (int m = 0; m < M; ++m) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint4 xv = *reinterpret_cast<const uint4*>(x + static_cast<size_t>(m) * K + k0 + j * 8);
          const bf16* xb = reinterpret_cast<const bf16*>(&xv);
#pragma unroll
          for (int i = 0; i < 8; ++i) acc[m] = fmaf(wf[j * 8 + i], __bfloat162float(xb[i]), acc[m]);
        }
      }
    }
#pragma unroll
    for (int m = 0; m < M; ++m) {
      const float v = warp_sum(acc[m]);
      if (lane == 0) y[static_cast<size_t>(m) * N + n] = __float2bfloat16(v);
    }
  }
}

// Reconstruct the bf16 matrix [N, K]; one thread per chunk of 32 weights (four 16-byte stores).
template <int B>
__global__ void wna16_dequant_kernel(const uint32_t* __restrict__ qweight, const bf16* __restrict__ scales, const uint8_t* __restrict__ zeros,
                                     bf16* __restrict__ out, long long total_chunks, int K, int group) {
  const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= total_chunks) return;
  const int chunks = K / 32;
  const long long n = idx / chunks;
  const int k0 = static_cast<int>(idx % chunks) * 32;
  const int groups = K / group;
  uint32_t w[B];
#pragma unroll
  for (int j = 0; j < B; ++j) w[j] = qweight[idx * B + j];
  float wf[32];
  unpack_chunk<B>(w, static_cast<float>(zeros[n * groups + k0 / group]), __bfloat162float(scales[n * groups + k0 / group]), wf);
#pragma unroll
  for (int v = 0; v < 4; ++v) {
    __align__(16) bf16 o[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i] = __float2bfloat16(wf[v * 8 + i]);
    *reinterpret_cast<uint4*>(out + n * K + k0 + v * 8) = *reinterpret_cast<const uint4*>(o);
  }
}

template <int B>
int launch_gemv(const void* x, const void* q, const void* s, const void* z, void* y, int M, int N, int K, int group, cudaStream_t stream) {
  const int blocks = (N + WN_WARPS - 1) / WN_WARPS;
  const bf16* xb = reinterpret_cast<const bf16*>(x);
  const uint32_t* qw = reinterpret_cast<const uint32_t*>(q);
  const bf16* sc = reinterpret_cast<const bf16*>(s);
  const uint8_t* zp = reinterpret_cast<const uint8_t*>(z);
  bf16* yb = reinterpret_cast<bf16*>(y);
#define OB_WN_CASE(MM) case MM: wna16_gemv_kernel<B, MM><<<blocks, WN_WARPS * 32, 0, stream>>>(xb, qw, sc, zp, yb, N, K, group); break;
  switch (M) {
    OB_WN_CASE(1) OB_WN_CASE(2) OB_WN_CASE(3) OB_WN_CASE(4) OB_WN_CASE(5) OB_WN_CASE(6) OB_WN_CASE(7) OB_WN_CASE(8)
    default: return -1;
  }
#undef OB_WN_CASE
  return cudaGetLastError() == cudaSuccess ? 0 : -11;
}

template <int B>
int launch_dequant(const void* q, const void* s, const void* z, void* out, int N, int K, int group, cudaStream_t stream) {
  const long long total = static_cast<long long>(N) * (K / 32);
  const int threads = 256;
  const long long blocks = (total + threads - 1) / threads;
  wna16_dequant_kernel<B><<<static_cast<unsigned>(blocks), threads, 0, stream>>>(
      reinterpret_cast<const uint32_t*>(q), reinterpret_cast<const bf16*>(s), reinterpret_cast<const uint8_t*>(z),
      reinterpret_cast<bf16*>(out), total, K, group);
  return cudaGetLastError() == cudaSuccess ? 0 : -11;
}

bool shapes_ok(int N, int K, int group, int bits) {
  return N > 0 && K > 0 && K % 32 == 0 && group > 0 && group % 32 == 0 && K % group == 0 && (bits == 2 || bits == 3 || bits == 4 || bits == 8);
}

}  // namespace
}  // namespace ob

// x [M, K] bf16 (1 <= M <= 8), qweight [N, K*bits/32] int32, scales [N, K/group] bf16, zeros [N, K/group] uint8 -> y [M, N] bf16.
extern "C" int ob_wna16_gemv(const void* x, const void* qweight, const void* scales, const void* zeros, void* y, int M, int N, int K,
                             int group, int bits, cudaStream_t stream) {
  using namespace ob;
  if (!shapes_ok(N, K, group, bits) || M < 1 || M > 8) return -1;
  if ((reinterpret_cast<uintptr_t>(x) & 15) != 0) return -2;
  switch (bits) {
    case 2: return launch_gemv<2>(x, qweight, scales, zeros, y, M, N, K, group, stream);
    case 3: return launch_gemv<3>(x, qweight, scales, zeros, y, M, N, K, group, stream);
    case 4: return launch_gemv<4>(x, qweight, scales, zeros, y, M, N, K, group, stream);
    default: return launch_gemv<8>(x, qweight, scales, zeros, y, M, N, K, group, stream);
  }
}

// Reconstruct W [N, K] bf16 (16-byte aligned) from the packed representation.
extern "C" int ob_wna16_dequant(const void* qweight, const void* scales, const void* zeros, void* out, int N, int K, int group, int bits,
                                cudaStream_t stream) {
  using namespace ob;
  if (!shapes_ok(N, K, group, bits)) return -1;
  if ((reinterpret_cast<uintptr_t>(out) & 15) != 0) return -2;
  switch (bits) {
    case 2: return launch_dequant<2>(qweight, scales, zeros, out, N, K, group, stream);
    case 3: return launch_dequant<3>(qweight, scales, zeros, out, N, K, group, stream);
    case 4: return launch_dequant<4>(qweight, scales, zeros, out, N, K, group, stream);
    default: return launch_dequant<8>(qweight, scales, zeros, out, N, K, group, stream);
  }
}

// 4-bit weight / 16-bit activation inference kernels (weight-only quantisation, per-group scale and zero point).
//
// Layout (chosen for this library, not AutoGPTQ's): a linear layer y = x · Wᵀ with W of shape [N, K] is stored as
//   qweight [N, K/8]  int32   eight consecutive K entries per word, entry i in bits 4i..4i+3
//   scales  [N, K/G]  bf16    one scale per group of G consecutive K entries
//   zeros   [N, K/G]  uint8   zero point (0..15) per group
// so that W[n][k] = (q[n][k] - zeros[n][k/G]) * scales[n][k/G].  Rows are K-contiguous, like every other weight in the
// library, which lets the reconstructed matrix feed the tcgen05 GEMM directly.  Activation ordering ("act-order") is
// expressed as a permutation of the K axis applied to x (gather kernel below); the groups of the stored matrix are
// contiguous in the permuted order, so the inner loops never look up a group index per element.
//
// Counterparts in the reference's vendored AutoGPTQ: q4 matmul / reconstruct / column remap CUDA kernels.
#include "common.cuh"
#include "api.h"

namespace ob {
namespace {

constexpr int GV_WARPS = 8;

__device__ __forceinline__ uint4 ldg_nc_v4(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}

__device__ __forceinline__ void unpack8(uint32_t word, float zero, float scale, float (&out)[8]) {
#pragma unroll
  for (int i = 0; i < 8; ++i) out[i] = (static_cast<float>((word >> (4 * i)) & 0xF) - zero) * scale;
}

// y[m][n] = Σ_k x[m][k] · W[n][k] for 1 <= M <= 8.  One warp per output row; a lane owns 32-weight (16-byte) chunks of
// the row, strided by 32 lanes, so that a warp's loads of one iteration cover 512 contiguous bytes of the weight row.
// The weight stream is the only HBM traffic that matters (x is a few KiB and stays in L1/L2).
template <int M>
__global__ void __launch_bounds__(GV_WARPS * 32) w4a16_gemv_kernel(const bf16* __restrict__ x, const uint32_t* __restrict__ qweight,
                                                                    const bf16* __restrict__ scales, const uint8_t* __restrict__ zeros,
                                                                    bf16* __restrict__ y, int N, int K, int group) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int chunks = K / 32;  // 16-byte chunks per row
  const int groups = K / group;
  for (int n = blockIdx.x * GV_WARPS + warp; n < N; n += gridDim.x * GV_WARPS) {
    const uint32_t* wrow = qweight + static_cast<size_t>(n) * (K / 8);
    const bf16* srow = scales + static_cast<size_t>(n) * groups;
    const uint8_t* zrow = zeros + static_cast<size_t>(n) * groups;
    float acc[M];
#pragma unroll
    for (int m = 0; m < M; ++m) acc[m] = 0.f;
    for (int c = lane; c < chunks; c += 32) {
      const uint4 w = ldg_nc_v4(wrow + c * 4);
      const int k0 = c * 32;
      const int g = k0 / group;  // a 32-entry chunk never straddles a group (group is a multiple of 32)
      const float s = __bfloat162float(srow[g]);
      const float z = static_cast<float>(zrow[g]);
      const uint32_t words[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float wf[8];
        unpack8(words[j], z, s, wf);
#pragma unroll
        for (int m = 0; m < M; ++m) {
          const uint4 xv = *reinterpret_cast<const uint4*>(x + static_cast<size_t>(m) * K + k0 + j * 8);
          const bf16* xb = reinterpret_cast<const bf16*>(&xv);
#pragma unroll
          for (int i = 0; i < 8; ++i) acc[m] = fmaf(wf[i], __bfloat162float(xb[i]), acc[m]);
        }
      }
    }
#pragma unroll
    for (int m = 0; m < M; ++m) {
      float v = acc[m];
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
      if (lane == 0) y[static_cast<size_t>(m) * N + n] = __float2bfloat16(v);
    }
  }
}

// Reconstruct the bf16 matrix [N, K]; one thread per packed word (8 weights -> one 16-byte store).
__global__ void w4a16_dequant_kernel(const uint32_t* __restrict__ qweight, const bf16* __restrict__ scales, const uint8_t* __restrict__ zeros,
                                     bf16* __restrict__ out, long long words, int K, int group) {
  const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= words) return;
  const int words_per_row = K / 8;
  const long long n = idx / words_per_row;
  const int k0 = static_cast<int>(idx % words_per_row) * 8;
  const int groups = K / group;
  const float s = __bfloat162float(scales[n * groups + k0 / group]);
  const float z = static_cast<float>(zeros[n * groups + k0 / group]);
  float wf[8];
  unpack8(qweight[idx], z, s, wf);
  __align__(16) bf16 o[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) o[i] = __float2bfloat16(wf[i]);
  *reinterpret_cast<uint4*>(out + n * K + k0) = *reinterpret_cast<const uint4*>(o);
}

// out[m][j] = x[m][perm[j]]: applies the activation-order permutation of the K axis.
__global__ void gather_columns_kernel(const bf16* __restrict__ x, const int* __restrict__ perm, bf16* __restrict__ out, int M, int K) {
  const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= static_cast<long long>(M) * K) return;
  const int m = static_cast<int>(idx / K), j = static_cast<int>(idx % K);
  out[idx] = x[static_cast<size_t>(m) * K + perm[j]];
}

template <int M>
void launch_gemv(const bf16* x, const uint32_t* q, const bf16* s, const uint8_t* z, bf16* y, int N, int K, int group, cudaStream_t stream) {
  const int blocks = min((N + GV_WARPS - 1) / GV_WARPS, 148 * 8);
  w4a16_gemv_kernel<M><<<blocks, GV_WARPS * 32, 0, stream>>>(x, q, s, z, y, N, K, group);
}

}  // namespace
}  // namespace ob

extern "C" {

int ob_w4a16_gemv(const void* x, const void* qweight, const void* scales, const void* zeros, void* y, int M, int N, int K, int group,
                  cudaStream_t stream) {
  using namespace ob;
  if (M < 1 || M > 8 || K % 32 != 0 || group % 32 != 0 || K % group != 0) return -1;
  const bf16* xp = static_cast<const bf16*>(x);
  const uint32_t* q = static_cast<const uint32_t*>(qweight);
  const bf16* s = static_cast<const bf16*>(scales);
  const uint8_t* z = static_cast<const uint8_t*>(zeros);
  bf16* yp = static_cast<bf16*>(y);
  switch (M) {
    case 1: launch_gemv<1>(xp, q, s, z, yp, N, K, group, stream); break;
    case 2: launch_gemv<2>(xp, q, s, z, yp, N, K, group, stream); break;
    case 3: launch_gemv<3>(xp, q, s, z, yp, N, K, group, stream); break;
    case 4: launch_gemv<4>(xp, q, s, z, yp, N, K, group, stream); break;
    case 5: launch_gemv<5>(xp, q, s, z, yp, N, K, group, stream); break;
    case 6: launch_gemv<6>(xp, q, s, z, yp, N, K, group, stream); break;
    case 7: launch_gemv<7>(xp, q, s, z, yp, N, K, group, stream); break;
    default: launch_gemv<8>(xp, q, s, z, yp, N, K, group, stream); break;
  }
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

int ob_w4a16_dequant(const void* qweight, const void* scales, const void* zeros, void* out, int N, int K, int group, cudaStream_t stream) {
  if (K % 8 != 0 || group % 8 != 0 || K % group != 0) return -1;
  const long long words = static_cast<long long>(N) * (K / 8);
  const int threads = 256;
  const long long blocks = (words + threads - 1) / threads;
  ob::w4a16_dequant_kernel<<<static_cast<unsigned>(blocks), threads, 0, stream>>>(
      static_cast<const uint32_t*>(qweight), static_cast<const ob::bf16*>(scales), static_cast<const uint8_t*>(zeros),
      static_cast<ob::bf16*>(out), words, K, group);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

int ob_gather_columns_bf16(const void* x, const int* perm, void* out, int M, int K, cudaStream_t stream) {
  const long long total = static_cast<long long>(M) * K;
  const int threads = 256;
  ob::gather_columns_kernel<<<static_cast<unsigned>((total + threads - 1) / threads), threads, 0, stream>>>(
      static_cast<const ob::bf16*>(x), perm, static_cast<ob::bf16*>(out), M, K);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

}  // extern "C"

// y = x · Wᵀ for 4-bit weights and a decode-sized activation batch (9..256 rows), on the tcgen05 tensor cores with the
// dequantisation fused into the operand staging: the packed weights are read from HBM exactly once (half a byte per
// weight) and never exist as a bf16 matrix in global memory.
//
// Roles are swapped with respect to the training GEMM: the *weights* are the 128-row A operand (so a CTA owns 128
// output features) and the *activations* are the B operand (UMMA N = the batch, padded to 32/64/128/256), i.e. the
// accumulator in TMEM is yᵀ: lane = output feature, column = batch row.
//
// Grid (features / 128, K splits), 320 threads per CTA:
//   warps 0..7  dequantise: threads r and r + 128 share weight row n0 + r, each owning half of every 64-wide K block.
//               A thread keeps the packed codes of the next four blocks in registers (the loads are the only long
//               latency of the loop), turns 16 bytes into 32 bf16 and writes them into row r of a 128 x 64 K-major
//               tile in the 128-byte-swizzled layout tcgen05 expects (16-byte chunk c of row r lives at chunk position
//               c ^ (r % 8)), then makes the writes visible to the async proxy and arrives on the stage's barrier.
//               After the K loop the same warps read TMEM (warp w may touch lanes 32·(w % 4)..; the two warps of a
//               lane quarter take alternate 32-column chunks) and store y: lanes are consecutive features, so a warp's
//               stores are contiguous.
//   warp 8      TMA producer of the activation tile (MB x 64, rows beyond M are zero-filled by the copy engine)
//   warp 9      MMA issuer (one lane), owns the TMEM allocation
// A stage is full when the eight dequantising warps (one arrival each, after a warp-wide sync) and the TMA transaction
// have arrived; it is released by tcgen05.commit.
// With K splits (chosen when there are too few 128-feature tiles to fill the GPU) every CTA covers a range of K blocks
// and adds its partial result to a zeroed fp32 workspace, which the caller converts to bf16.
// Every wait is bounded and reports through the status word; an aborting CTA still releases its TMEM.
//
// Counterpart in the reference's vendored AutoGPTQ: the Triton quant_matmul kernel (tensor-core path for batches).
#include <cstdlib>

#include "common.cuh"
#include "api.h"

namespace ob {

int make_tensor_map_bf16_2d(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer, uint64_t ld,
                            uint32_t box_inner, uint32_t box_outer);

namespace {

constexpr int WM_ROWS = 128;  // weight rows (output features) per CTA = UMMA M
constexpr int WM_BK = 64;     // K entries per stage: one 128-byte swizzled row
constexpr int WM_STAGES = 4;
constexpr int WM_DEQ_THREADS = 256;
constexpr int WM_THREADS = WM_DEQ_THREADS + 64;
constexpr int WM_AHEAD = 4;  // K blocks whose packed codes a thread holds in registers
constexpr int WM_A_BYTES = WM_ROWS * WM_BK * 2;  // 16 KiB

template <int MB>
struct WmCfg {
  static constexpr int B_BYTES = MB * WM_BK * 2;
  static constexpr int STAGE_BYTES = WM_A_BYTES + B_BYTES;
  static constexpr int SMEM_BYTES = 1024 + WM_STAGES * STAGE_BYTES + 256;
};

__device__ __forceinline__ uint4 ldg_stream_v4(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}

// Eight 4-bit codes of one word -> eight bf16, value = (code - zero) * scale rounded once, two values per instruction.
// A code c dropped into the low mantissa bits of bf16 128.0 (0x4300) reads 128 + c exactly; subtracting 128 + zero is
// exact and the product with the bf16 scale is rounded once, which is what the scalar fp32 formula gives.  The pairs
// come out as (c0,c4) (c1,c5) (c2,c6) (c3,c7); two byte permutes per pair of words restore K order.
__device__ __forceinline__ uint32_t bf16x2_sub_mul(uint32_t v, uint32_t zero_plus_128, uint32_t scale) {
  const __nv_bfloat162 r = __hmul2(__hsub2(*reinterpret_cast<const __nv_bfloat162*>(&v), *reinterpret_cast<const __nv_bfloat162*>(&zero_plus_128)),
                                   *reinterpret_cast<const __nv_bfloat162*>(&scale));
  return *reinterpret_cast<const uint32_t*>(&r);
}

__device__ __forceinline__ uint4 dequant_word(uint32_t word, uint32_t zero_plus_128, uint32_t scale) {
  const uint32_t a = bf16x2_sub_mul((word & 0x000F000Fu) | 0x43004300u, zero_plus_128, scale);          // c0, c4
  const uint32_t b = bf16x2_sub_mul(((word >> 4) & 0x000F000Fu) | 0x43004300u, zero_plus_128, scale);   // c1, c5
  const uint32_t c = bf16x2_sub_mul(((word >> 8) & 0x000F000Fu) | 0x43004300u, zero_plus_128, scale);   // c2, c6
  const uint32_t d = bf16x2_sub_mul(((word >> 12) & 0x000F000Fu) | 0x43004300u, zero_plus_128, scale);  // c3, c7
  uint4 o;
  o.x = __byte_perm(a, b, 0x5410);  // c0, c1
  o.y = __byte_perm(c, d, 0x5410);  // c2, c3
  o.z = __byte_perm(a, b, 0x7632);  // c4, c5
  o.w = __byte_perm(c, d, 0x7632);  // c6, c7
  return o;
}

template <int MB>
__global__ void __launch_bounds__(WM_THREADS, 2)
w4a16_mma_kernel(const __grid_constant__ CUtensorMap tma_x, const uint32_t* __restrict__ qweight, const bf16* __restrict__ scales,
                 const uint8_t* __restrict__ zeros, bf16* __restrict__ y, float* __restrict__ partial, int M, int N, int K, int group,
                 int blocks_per_split, int* __restrict__ status) {
  using Cfg = WmCfg<MB>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;                           // WM_STAGES x 16 KiB, each 1024-byte aligned
  uint8_t* sB = smem + WM_STAGES * WM_A_BYTES;  // WM_STAGES x B_BYTES (multiples of 4 KiB)
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + WM_STAGES * Cfg::STAGE_BYTES);
  uint64_t* empty_bar = full_bar + WM_STAGES;
  uint64_t* done_bar = empty_bar + WM_STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int n0 = static_cast<int>(blockIdx.x) * WM_ROWS;
  const int kb_begin = static_cast<int>(blockIdx.y) * blocks_per_split;
  const int kb_end = min(K / WM_BK, kb_begin + blocks_per_split);
  const int k_blocks = kb_end - kb_begin;  // >= 1 by construction of the grid

  if (threadIdx.x == 0) {
    for (int s = 0; s < WM_STAGES; ++s) {
      mbar_init(&full_bar[s], WM_DEQ_THREADS / 32 + 1);  // one arrival per dequantising warp + the TMA producer's expect_tx
      mbar_init(&empty_bar[s], 1);
    }
    mbar_init(done_bar, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 9) {
    tmem_alloc(tmem_slot, MB);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp < 8) {
    // ------------------------------------------------------------ dequantise into the A stages, then the epilogue
    const int r = threadIdx.x & (WM_ROWS - 1);  // row of the tile, TMEM lane of the result
    const int half = threadIdx.x >> 7;          // which 32 of the block's 64 K entries
    const int n = n0 + r;
    const int groups = K / group;
    const uint32_t* wrow = qweight + static_cast<size_t>(n) * (K / 8) + half * 4;
    const bf16* srow = scales + static_cast<size_t>(n) * groups;
    const uint8_t* zrow = zeros + static_cast<size_t>(n) * groups;
    const uint32_t row_off = static_cast<uint32_t>(r) * 128u;
    const uint32_t sw = static_cast<uint32_t>(r & 7);
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    uint4 ahead[WM_AHEAD];
    uint32_t ahead_sz[WM_AHEAD];  // the block's group scale (bf16 bits) and zero point, fetched with the codes
    auto load_sz = [&](int kb_abs) -> uint32_t {
      const int g = (kb_abs * WM_BK) / group;  // a 64-wide block never straddles a group
      return static_cast<uint32_t>(*reinterpret_cast<const uint16_t*>(srow + g)) | (static_cast<uint32_t>(zrow[g]) << 16);
    };
#pragma unroll
    for (int a = 0; a < WM_AHEAD; ++a) {
      if (a < k_blocks) {
        ahead[a] = ldg_stream_v4(wrow + static_cast<size_t>(kb_begin + a) * 8);
        ahead_sz[a] = load_sz(kb_begin + a);
      }
    }
    for (int kb0 = 0; kb0 < k_blocks && ok; kb0 += WM_AHEAD) {
#pragma unroll
      for (int a = 0; a < WM_AHEAD; ++a) {
        const int kb = kb0 + a;
        if (kb >= k_blocks) break;
        const uint4 codes = ahead[a];
        const uint32_t sz = ahead_sz[a];
        if (kb + WM_AHEAD < k_blocks) {
          ahead[a] = ldg_stream_v4(wrow + static_cast<size_t>(kb_begin + kb + WM_AHEAD) * 8);
          ahead_sz[a] = load_sz(kb_begin + kb + WM_AHEAD);
        }
        const uint32_t s16 = sz & 0xFFFFu;
        const uint32_t s = s16 | (s16 << 16);  // the group's bf16 scale in both halves
        const uint32_t z16 = 0x4300u | (sz >> 16);  // bf16 128 + zero (zero is 0..15)
        const uint32_t z = z16 | (z16 << 16);
        // the warp decides together: the arrival below is made by one lane on behalf of all 32
        if (!__all_sync(0xffffffffu, mbar_wait(&empty_bar[stage], phase ^ 1u, abort_flag, status, ST_TIMEOUT_PRODUCER))) {
          ok = false;
          break;
        }
        uint8_t* row = sA + stage * WM_A_BYTES + row_off;
        const uint32_t words[4] = {codes.x, codes.y, codes.z, codes.w};
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const uint32_t chunk = static_cast<uint32_t>(half * 4 + c);
          *reinterpret_cast<uint4*>(row + ((chunk ^ sw) << 4)) = dequant_word(words[c], z, s);
        }
        fence_proxy_async();  // generic-proxy stores -> visible to the tensor core's reads
        __syncwarp();         // every lane's stores and fence precede the warp's single arrival
        if (lane == 0) mbar_arrive(&full_bar[stage]);
        if (++stage == WM_STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
    if (ok && mbar_wait(done_bar, 0u, abort_flag, status, ST_TIMEOUT_EPILOGUE)) {
      tc_fence_after();
      const uint32_t t_addr = tmem_base + (static_cast<uint32_t>((warp & 3) * 32) << 16);
#pragma unroll 1
      for (int c = half; c < MB / 32; c += 2) {  // the two warps of a lane quarter take alternate column chunks
        if (c * 32 >= M) break;  // warp-uniform
        uint32_t acc[32];
        tmem_ld_32x32b_x32(t_addr + c * 32, acc);
        tmem_ld_wait();
        if (partial != nullptr) {
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int m = c * 32 + j;
            if (m < M) atomicAdd(partial + static_cast<size_t>(m) * N + n, __uint_as_float(acc[j]));
          }
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int m = c * 32 + j;
            if (m < M) y[static_cast<size_t>(m) * N + n] = __float2bfloat16_rn(__uint_as_float(acc[j]));
          }
        }
      }
    }
  } else if (warp == 8) {
    // ------------------------------------------------------------------------- activation tiles by TMA
    if (lane == 0) {
      prefetch_tensormap(&tma_x);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int kb = 0; kb < k_blocks; ++kb) {
        if (!mbar_wait(&empty_bar[stage], phase ^ 1u, abort_flag, status, ST_TIMEOUT_PRODUCER)) {
          ok = false;
          break;
        }
        mbar_expect_tx(&full_bar[stage], Cfg::B_BYTES);
        tma_load_2d(sB + stage * Cfg::B_BYTES, &tma_x, &full_bar[stage], (kb_begin + kb) * WM_BK, 0);
        if (++stage == WM_STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (!ok) {  // aborting: give copies already in flight a bounded time to land before shared memory is released
        const long long t0 = clock64();
        while (clock64() - t0 < 2000000LL) {
        }
      }
    }
  } else {
    // ----------------------------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc_bf16(WM_ROWS, MB, 0, 0);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int kb = 0; kb < k_blocks; ++kb) {
        if (!mbar_wait(&full_bar[stage], phase, abort_flag, status, ST_TIMEOUT_MMA)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t a_addr = smem_u32(sA + stage * WM_A_BYTES);
        const uint32_t b_addr = smem_u32(sB + stage * Cfg::B_BYTES);
#pragma unroll
        for (int k = 0; k < WM_BK / 16; ++k) {
          const uint64_t a_desc = make_smem_desc_sw128(a_addr + k * 32, 16, 1024);
          const uint64_t b_desc = make_smem_desc_sw128(b_addr + k * 32, 16, 1024);
          umma_f16_ss(tmem_base, a_desc, b_desc, idesc, (kb > 0 || k > 0) ? 1u : 0u);
        }
        umma_commit(&empty_bar[stage]);
        if (++stage == WM_STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (ok) umma_commit(done_bar);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem_base, MB);
  }
}

template <int MB>
int launch_mma(const CUtensorMap& tx, const uint32_t* q, const bf16* s, const uint8_t* z, bf16* y, float* partial, int M, int N, int K,
               int group, int splits, int blocks_per_split, int* status, cudaStream_t stream) {
  using Cfg = WmCfg<MB>;
  static bool configured = false;
  if (!configured) {
    if (cudaFuncSetAttribute(w4a16_mma_kernel<MB>, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM_BYTES) != cudaSuccess) return -4;
    configured = true;
  }
  const dim3 grid(N / WM_ROWS, splits);
  w4a16_mma_kernel<MB><<<grid, WM_THREADS, Cfg::SMEM_BYTES, stream>>>(tx, q, s, z, y, partial, M, N, K, group, blocks_per_split, status);
  return cudaGetLastError() == cudaSuccess ? 0 : -5;
}

}  // namespace
}  // namespace ob

extern "C" {

// 1 if ob_w4a16_gemm_small covers the shape: up to 256 activation rows, features in whole 128-row tiles, K in whole
// 64-entry blocks that never straddle a quantisation group.
int ob_w4a16_gemm_small_supported(int M, int N, int K, int group) {
  return (M >= 1 && M <= 256 && N % ob::WM_ROWS == 0 && K % ob::WM_BK == 0 && group % ob::WM_BK == 0 && K % group == 0) ? 1 : 0;
}

// Number of K splits the kernel wants for this shape: 1 when the 128-feature tiles alone fill the GPU, otherwise enough
// splits to reach the CTA target, each split keeping at least eight K blocks.  With more than one split the caller
// passes a zeroed fp32 [M, N] workspace and converts it to bf16 afterwards.
int ob_w4a16_gemm_small_splits(int N, int K) {
  // CTAs the launch should reach.  A CTA's K loop is latency-bound, so three per SM (two resident, one queued) measured
  // faster than one per SM (7.6 -> 6.7 ms per 7B decode step at 32 rows); OLMO_B200_W4_TARGET_CTAS overrides.
  static int target = 0;
  if (target == 0) {
    const char* env = getenv("OLMO_B200_W4_TARGET_CTAS");
    target = env != nullptr ? atoi(env) : 444;
    if (target < 1) target = 444;
  }
  const int tiles = N / ob::WM_ROWS;
  const int k_blocks = K / ob::WM_BK;
  if (tiles <= 0 || k_blocks <= 0 || tiles * 5 >= target * 4) return 1;
  int splits = (target + tiles - 1) / tiles;
  if (splits > k_blocks / 8) splits = k_blocks / 8;
  if (splits < 1) splits = 1;
  const int per = (k_blocks + splits - 1) / splits;
  return (k_blocks + per - 1) / per;  // no empty split
}

// y[M, N] (bf16, row pitch N) = x[M, K] (bf16, contiguous) · Wᵀ with W given as packed 4-bit codes.  `splits` must be
// the value of ob_w4a16_gemm_small_splits; when it is greater than 1 the result is *added* to `partial` (fp32 [M, N])
// and `y` is not written.
int ob_w4a16_gemm_small(const void* x, const void* qweight, const void* scales, const void* zeros, void* y, float* partial, int M, int N,
                        int K, int group, int splits, int* status, cudaStream_t stream) {
  using namespace ob;
  if (!ob_w4a16_gemm_small_supported(M, N, K, group)) return -1;
  const int k_blocks = K / WM_BK;
  if (splits < 1 || splits > k_blocks || (splits > 1) != (partial != nullptr)) return -1;
  const int per = (k_blocks + splits - 1) / splits;
  if ((k_blocks + per - 1) / per != splits) return -1;
  const int mb = M <= 32 ? 32 : (M <= 64 ? 64 : (M <= 128 ? 128 : 256));
  CUtensorMap tx;
  // rows beyond M are outside the tensor: the copy engine fills them with zeros, which is the padding of the batch
  int rc = make_tensor_map_bf16_2d(&tx, x, static_cast<uint64_t>(K), static_cast<uint64_t>(M), static_cast<uint64_t>(K), WM_BK,
                                   static_cast<uint32_t>(mb));
  if (rc != 0) return rc - 10;
  const uint32_t* q = static_cast<const uint32_t*>(qweight);
  const bf16* s = static_cast<const bf16*>(scales);
  const uint8_t* z = static_cast<const uint8_t*>(zeros);
  bf16* yp = static_cast<bf16*>(y);
  switch (mb) {
    case 32: return launch_mma<32>(tx, q, s, z, yp, partial, M, N, K, group, splits, per, status, stream);
    case 64: return launch_mma<64>(tx, q, s, z, yp, partial, M, N, K, group, splits, per, status, stream);
    case 128: return launch_mma<128>(tx, q, s, z, yp, partial, M, N, K, group, splits, per, status, stream);
    default: return launch_mma<256>(tx, q, s, z, yp, partial, M, N, K, group, splits, per, status, stream);
  }
}

}  // extern "C"

// y = x · Wᵀ in bf16 for a decode-sized activation batch (1..256 rows) on the tcgen05 tensor cores.
//
// With a handful of rows the product is a stream of the weight matrix: every byte of W is needed once, and the job of the
// kernel is to keep HBM busy.  The operand roles are therefore swapped with respect to the training GEMM: the *weights*
// are the 128-row A operand (a CTA owns 128 output features), the *activations* are the B operand (UMMA N = the batch,
// padded to 16/32/64/128/256; rows beyond M are zero-filled by the copy engine), and the accumulator in TMEM is yᵀ
// (lane = output feature, column = batch row).  Layers with few 128-feature tiles split K over several CTAs so that
// two CTAs per SM stream weights at once in a single wave; every split writes its own fp32 slab and a second kernel adds the
// slabs in split order (no atomics: the result does not depend on scheduling) and rounds to bf16.
//
// Roles per CTA (192 threads): warp 0 TMA producer (weight tile 128 x 64 and activation tile MB x 64 per stage, an
// four-stage ring), warp 1 MMA issuer (owns TMEM), warps 2..5 epilogue.  Every wait is bounded and reports through the
// status word; an aborting CTA still frees its TMEM.
#include "common.cuh"
#include "api.h"

namespace ob {

int make_tensor_map_bf16_2d(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer, uint64_t ld,
                            uint32_t box_inner, uint32_t box_outer);

namespace {

constexpr int SM_ROWS = 128;  // output features per CTA = UMMA M
constexpr int SM_BK = 64;     // K entries per stage: one 128-byte swizzled row
constexpr int SM_THREADS = 192;
constexpr int SM_A_BYTES = SM_ROWS * SM_BK * 2;  // 16 KiB

template <int MB>
struct SmCfg {
  static constexpr int B_BYTES = MB * SM_BK * 2;
  static constexpr int STAGE_BYTES = SM_A_BYTES + B_BYTES;
  static constexpr int STAGES = 4;  // two CTAs share an SM for MB <= 64: one streams while the other starts up or drains
  static constexpr int SMEM_BYTES = 1024 + STAGES * STAGE_BYTES + 256;
  static constexpr int TMEM_COLS = MB < 32 ? 32 : MB;
};

template <int MB>
__global__ void __launch_bounds__(SM_THREADS, 2)
gemm_smallm_kernel(const __grid_constant__ CUtensorMap tma_w, const __grid_constant__ CUtensorMap tma_x, bf16* __restrict__ y,
                   float* __restrict__ partial, int M, int N, int K, int kb_per_split, int* __restrict__ status) {
  using Cfg = SmCfg<MB>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + Cfg::STAGES * SM_A_BYTES;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + Cfg::STAGES * Cfg::STAGE_BYTES);
  uint64_t* empty_bar = full_bar + Cfg::STAGES;
  uint64_t* done_bar = empty_bar + Cfg::STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = static_cast<int>(blockIdx.x) * SM_ROWS;
  const int split = static_cast<int>(blockIdx.y);
  const int k_blocks = (K + SM_BK - 1) / SM_BK;
  const int kb0 = split * kb_per_split;
  const int kb1 = min(k_blocks, kb0 + kb_per_split);
  const int my_blocks = max(0, kb1 - kb0);

  if (threadIdx.x == 0) {
    for (int s = 0; s < Cfg::STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    mbar_init(done_bar, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, Cfg::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      prefetch_tensormap(&tma_w);
      prefetch_tensormap(&tma_x);
      int stage = 0;
      uint32_t phase = 0;
      for (int kb = 0; kb < my_blocks; ++kb) {
        if (!mbar_wait(&empty_bar[stage], phase ^ 1u, abort_flag, status, ST_TIMEOUT_PRODUCER)) break;
        mbar_expect_tx(&full_bar[stage], Cfg::STAGE_BYTES);
        const int k0 = (kb0 + kb) * SM_BK;
        tma_load_2d(sA + stage * SM_A_BYTES, &tma_w, &full_bar[stage], k0, n0);
        tma_load_2d(sB + stage * Cfg::B_BYTES, &tma_x, &full_bar[stage], k0, 0);
        if (++stage == Cfg::STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (*abort_flag) {  // give copies in flight time to land before the CTA's shared memory goes away
        const long long t0 = clock64();
        while (clock64() - t0 < 2000000LL) {
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc_bf16(SM_ROWS, MB, 0, 0);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int kb = 0; kb < my_blocks; ++kb) {
        if (!mbar_wait(&full_bar[stage], phase, abort_flag, status, ST_TIMEOUT_MMA)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t a_addr = smem_u32(sA + stage * SM_A_BYTES);
        const uint32_t b_addr = smem_u32(sB + stage * Cfg::B_BYTES);
#pragma unroll
        for (int k = 0; k < SM_BK / 16; ++k)
          umma_f16_ss(tmem_base, make_smem_desc_sw128(a_addr + k * 32, 16, 1024), make_smem_desc_sw128(b_addr + k * 32, 16, 1024), idesc,
                      (kb > 0 || k > 0) ? 1u : 0u);
        umma_commit(&empty_bar[stage]);
        if (++stage == Cfg::STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (ok) umma_commit(done_bar);
    }
  } else {
    // epilogue: warp w may read TMEM lanes 32 (w % 4) .. 32 (w % 4) + 31, i.e. 32 consecutive output features
    const int quarter = warp & 3;
    const int n = n0 + quarter * 32 + lane;
    bool ok = my_blocks > 0;
    if (ok) ok = mbar_wait(done_bar, 0, abort_flag, status, ST_TIMEOUT_EPILOGUE);
    if (ok) {
      tc_fence_after();
      __syncwarp();
      const uint32_t t_addr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16);
      constexpr int CH = MB < 16 ? MB : 16;
#pragma unroll 1
      for (int c0 = 0; c0 < MB; c0 += CH) {
        uint32_t r[16];
        tmem_ld_32x32b_x16(t_addr + c0, r);
        tmem_ld_wait();
        if (n < N) {
#pragma unroll
          for (int j = 0; j < CH; ++j) {
            const int m = c0 + j;
            if (m < M) {
              if (partial != nullptr) partial[(static_cast<size_t>(split) * M + m) * N + n] = __uint_as_float(r[j]);
              else y[static_cast<size_t>(m) * N + n] = __float2bfloat16_rn(__uint_as_float(r[j]));
            }
          }
        }
      }
    } else if (my_blocks == 0 && partial != nullptr && n < N) {
      for (int m = 0; m < M; ++m) partial[(static_cast<size_t>(split) * M + m) * N + n] = 0.f;  // an empty split contributes zero
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
  }
}

// y[i] = bf16(sum_s partial[s][i]), slabs added in split order.
__global__ void sum_splits_kernel(const float* __restrict__ partial, bf16* __restrict__ y, long long n, int splits) {
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n) return;
  float s = 0.f;
  for (int k = 0; k < splits; ++k) s += partial[static_cast<long long>(k) * n + i];
  y[i] = __float2bfloat16_rn(s);
}

template <int MB>
int launch_smallm(const CUtensorMap& tw, const CUtensorMap& tx, void* y, float* partial, int M, int N, int K, int splits, int* status,
                  cudaStream_t stream) {
  using Cfg = SmCfg<MB>;
  auto kern = gemm_smallm_kernel<MB>;
  static bool configured = false;
  if (!configured) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM_BYTES) != cudaSuccess) return -10;
    configured = true;
  }
  const int k_blocks = (K + SM_BK - 1) / SM_BK;
  const int kb_per = (k_blocks + splits - 1) / splits;
  dim3 grid((N + SM_ROWS - 1) / SM_ROWS, splits);
  kern<<<grid, SM_THREADS, Cfg::SMEM_BYTES, stream>>>(tw, tx, reinterpret_cast<bf16*>(y), splits > 1 ? partial : nullptr, M, N, K, kb_per, status);
  if (cudaGetLastError() != cudaSuccess) return -11;
  if (splits > 1) {
    const long long n = static_cast<long long>(M) * N;
    sum_splits_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, stream>>>(partial, reinterpret_cast<bf16*>(y), n, splits);
    if (cudaGetLastError() != cudaSuccess) return -11;
  }
  return 0;
}

int padded_rows(int M) { return M <= 16 ? 16 : M <= 32 ? 32 : M <= 64 ? 64 : M <= 128 ? 128 : 256; }

}  // namespace
}  // namespace ob

// Number of K splits the kernel wants for a layer (the caller provides `splits * M * N` floats of workspace when > 1).
extern "C" int ob_gemm_smallm_splits(int N, int K, int num_sms) {
  if (num_sms <= 0) num_sms = 148;
  const int tiles = (N + ob::SM_ROWS - 1) / ob::SM_ROWS;
  const int k_blocks = (K + ob::SM_BK - 1) / ob::SM_BK;
  int splits = (2 * num_sms) / tiles;  // two CTAs per SM, all resident at once: one wave, no tail
  if (splits > k_blocks / 8) splits = k_blocks / 8;  // at least eight K blocks (two rings) per CTA
  return splits < 1 ? 1 : splits;
}

// x [M, K] bf16 (row pitch ldx), w [N, K] bf16 (row pitch ldw), y [M, N] bf16 contiguous; 1 <= M <= 256.
extern "C" int ob_gemm_smallm(const void* x, const void* w, void* y, float* partial, int M, int N, int K, int ldx, int ldw, int splits,
                              int* status, cudaStream_t stream) {
  using namespace ob;
  if (M < 1 || M > 256 || N < 1 || K < 1 || splits < 1) return -1;
  if (splits > 1 && partial == nullptr) return -1;
  const int MB = padded_rows(M);
  CUtensorMap tw, tx;
  int rc = make_tensor_map_bf16_2d(&tw, w, (uint64_t)K, (uint64_t)N, (uint64_t)ldw, SM_BK, SM_ROWS);
  if (rc != 0) return rc;
  rc = make_tensor_map_bf16_2d(&tx, x, (uint64_t)K, (uint64_t)M, (uint64_t)ldx, SM_BK, MB);
  if (rc != 0) return rc;
  switch (MB) {
    case 16: return launch_smallm<16>(tw, tx, y, partial, M, N, K, splits, status, stream);
    case 32: return launch_smallm<32>(tw, tx, y, partial, M, N, K, splits, status, stream);
    case 64: return launch_smallm<64>(tw, tx, y, partial, M, N, K, splits, status, stream);
    case 128: return launch_smallm<128>(tw, tx, y, partial, M, N, K, splits, status, stream);
    default: return launch_smallm<256>(tw, tx, y, partial, M, N, K, splits, status, stream);
  }
}

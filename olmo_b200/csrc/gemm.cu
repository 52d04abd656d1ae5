// bf16 GEMM on the 5th-generation tensor cores (tcgen05.mma, accumulators in TMEM, operands staged by TMA).
//
//   D[M,N] = A · B   with fp32 accumulation, where each operand is either
//     K-major  : memory is [rows, K] with K contiguous            (x and W of a Linear forward), or
//     MN-major : memory is [K, rows] with the row index contiguous (the transposed operands of dgrad/wgrad).
//
// One persistent CTA per SM, 192 threads:
//   warp 0      TMA producer        (4-stage ring of 128x64 A tiles and 256x64 B tiles, 128B swizzle)
//   warp 1      MMA issuer          (one elected lane issues tcgen05.mma 128x256x16; owns the TMEM allocation)
//   warps 2..5  epilogue            (tcgen05.ld 32x32b from one of two 256-column accumulators -> global)
// The two TMEM accumulators let the epilogue of tile i overlap the main loop of tile i+1.
//
// A launch may carry a collective (CommTask, comm.cuh).  With `comm_ctas` == 0 the spare warps 6..15 of every CTA execute
// their CTA's share of it next to the tensor-core pipeline; with `comm_ctas` > 0 the first `comm_ctas` blocks of the grid execute it
// (comm.cuh: peer all-gather of the next unit's weights, or the gradient reduce-scatter of the previous unit) and
// exit; the remaining blocks are the persistent GEMM.  One launch therefore overlaps NVLink traffic with the math.
//
// Optional readiness flags: when `b_ready` is given, the producer waits (bounded) until
// b_ready[(first B row of the tile) / rows_per_flag ... (last row) / rows_per_flag] >= ready_value before it
// loads B.  The parameter all-gather that lands peer shards in local memory sets these flags chunk by chunk,
// which lets the consuming GEMM start before the whole weight has arrived.
#include "common.cuh"
#include "comm.cuh"
#include "api.h"

namespace ob {

namespace {

constexpr int BM = 128;
constexpr int BN = 256;
constexpr int BK = 64;
constexpr int STAGES = 4;
constexpr int A_BYTES = BM * BK * 2;  // 16 KiB
constexpr int B_BYTES = BN * BK * 2;  // 32 KiB
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int CHUNK_BYTES = 64 * BK * 2;  // one 64(mn) x 64(k) box of an MN-major operand
constexpr int NUM_THREADS = 192;       // six role warps
constexpr int NUM_THREADS_COMM = 512;  // launches that carry communication CTAs: more warps to hide NVLink latency
constexpr int TMEM_COLS = 512;
constexpr int SMEM_BYTES = 1024 + STAGES * STAGE_BYTES + 256;
constexpr int GROUP_M = 8;

struct TileCoord {
  int m, n;
};

__device__ __forceinline__ TileCoord tile_coord(int t, int tiles_m, int tiles_n) {
  // grouped raster: GROUP_M row-tiles share each column-tile while it is hot in L2
  const int group_size = GROUP_M * tiles_n;
  const int group = t / group_size;
  const int first_m = group * GROUP_M;
  const int rows = min(tiles_m - first_m, GROUP_M);
  const int in_group = t - group * group_size;
  return {first_m + in_group % rows, in_group / rows};
}

template <int A_MN, int B_MN, int EPI>
__global__ void __launch_bounds__(NUM_THREADS_COMM, 1)
gemm_bf16_kernel(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b,
                 void* __restrict__ Cptr, const bf16* __restrict__ Rptr, int M, int N, int K, int ldc, int vec_ok,
                 const int* __restrict__ b_ready, int rows_per_flag, int ready_value, int* __restrict__ status,
                 const __grid_constant__ CommTask comm_task, int comm_ctas) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ CommScratch comm_scratch;
  if (static_cast<int>(blockIdx.x) < comm_ctas) {  // communication role: no TMEM, no barriers
    const CommGroup g = {static_cast<int>(threadIdx.x), static_cast<int>(blockDim.x), 1};
    comm_run(comm_task, blockIdx.x, comm_ctas, &comm_scratch, g);
    return;
  }
  const int cta = static_cast<int>(blockIdx.x) - comm_ctas;
  const int num_ctas = static_cast<int>(gridDim.x) - comm_ctas;
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_BYTES;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* tfull_bar = empty_bar + STAGES;
  uint64_t* tempty_bar = tfull_bar + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty_bar + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int tiles_m = (M + BM - 1) / BM;
  const int tiles_n = (N + BN - 1) / BN;
  const int num_tiles = tiles_m * tiles_n;
  const int k_blocks = (K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull_bar[a], 1);
      mbar_init(&tempty_bar[a], 128);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      prefetch_tensormap(&tma_a);
      prefetch_tensormap(&tma_b);
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;
      bool ok = true;
      for (int t = cta; t < num_tiles && ok; t += num_ctas) {
        const TileCoord tc = tile_coord(t, tiles_m, tiles_n);
        const int m0 = tc.m * BM, n0 = tc.n * BN;
        if (b_ready != nullptr) {
          const int last_row = min(n0 + BN, N) - 1;
          for (int f = n0 / rows_per_flag; f <= last_row / rows_per_flag && ok; ++f)
            ok = flag_wait_ge(b_ready + f, ready_value, abort_flag, status);
          if (!ok) break;
        }
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1u, abort_flag, status, ST_TIMEOUT_PRODUCER)) {
            ok = false;
            break;
          }
          mbar_expect_tx(&full_bar[stage], STAGE_BYTES);
          uint8_t* a_dst = sA + stage * A_BYTES;
          uint8_t* b_dst = sB + stage * B_BYTES;
          const int k0 = kb * BK;
          if (A_MN) {
#pragma unroll
            for (int c = 0; c < BM / 64; ++c) tma_load_2d(a_dst + c * CHUNK_BYTES, &tma_a, &full_bar[stage], m0 + c * 64, k0);
          } else {
            tma_load_2d(a_dst, &tma_a, &full_bar[stage], k0, m0);
          }
          if (B_MN) {
#pragma unroll
            for (int c = 0; c < BN / 64; ++c) tma_load_2d(b_dst + c * CHUNK_BYTES, &tma_b, &full_bar[stage], n0 + c * 64, k0);
          } else {
            tma_load_2d(b_dst, &tma_b, &full_bar[stage], k0, n0);
          }
          ++issued;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) {
        // Aborting: give copies already in flight a bounded time to land before shared memory is released.
        const long long t0 = clock64();
        while (clock64() - t0 < 2000000LL) {
        }
      }
      (void)issued;
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc_bf16(BM, BN, A_MN, B_MN);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int t = cta; t < num_tiles && ok; t += num_ctas) {
        if (!mbar_wait(&tempty_bar[acc], acc_phase ^ 1u, abort_flag, status, ST_TIMEOUT_MMA)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!mbar_wait(&full_bar[stage], phase, abort_flag, status, ST_TIMEOUT_MMA)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(sA + stage * A_BYTES);
          const uint32_t b_addr = smem_u32(sB + stage * B_BYTES);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            // K-major: 16 bf16 = 32 B further along the swizzled row.  MN-major: two 8-row groups = 2 KiB further.
            const uint64_t a_desc = A_MN ? make_smem_desc_sw128(a_addr + k * 2048, CHUNK_BYTES, 1024)
                                         : make_smem_desc_sw128(a_addr + k * 32, 16, 1024);
            const uint64_t b_desc = B_MN ? make_smem_desc_sw128(b_addr + k * 2048, CHUNK_BYTES, 1024)
                                         : make_smem_desc_sw128(b_addr + k * 32, 16, 1024);
            umma_f16_ss(d_tmem, a_desc, b_desc, idesc, (kb > 0 || k > 0) ? 1u : 0u);
          }
          umma_commit(&empty_bar[stage]);  // stage reusable once these MMAs have read it
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(&tfull_bar[acc]);  // accumulator complete
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
    }
  } else if (warp < 6) {
    // --------------------------------------------------------------------- epilogue
    const int quarter = warp & 3;  // TMEM lanes [32*quarter, 32*quarter+32) are the ones this warp may read
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = cta; t < num_tiles; t += num_ctas) {
      const TileCoord tc = tile_coord(t, tiles_m, tiles_n);
      const int row = tc.m * BM + quarter * 32 + lane;
      const int n0 = tc.n * BN;
      if (!mbar_wait(&tfull_bar[acc], acc_phase, abort_flag, status, ST_TIMEOUT_EPILOGUE)) break;
      tc_fence_after();
      const uint32_t t_addr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + static_cast<uint32_t>(acc * BN);
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(t_addr + c * 32, r);
        tmem_ld_wait();
        const int col0 = n0 + c * 32;
        if (row < M && col0 < N) {
          const bool full = vec_ok && (col0 + 32 <= N);
          if (EPI == EPI_BF16 || EPI == EPI_BF16_ADD) {
            bf16* crow = reinterpret_cast<bf16*>(Cptr) + static_cast<size_t>(row) * ldc + col0;
            const bf16* rrow = (EPI == EPI_BF16_ADD) ? Rptr + static_cast<size_t>(row) * ldc + col0 : nullptr;
            if (full) {
#pragma unroll
              for (int v = 0; v < 4; ++v) {
                float f[8];
#pragma unroll
                for (int j = 0; j < 8; ++j) f[j] = __uint_as_float(r[v * 8 + j]);
                if (EPI == EPI_BF16_ADD) {
                  const uint4 rv = *reinterpret_cast<const uint4*>(rrow + v * 8);
                  const uint32_t ru[4] = {rv.x, rv.y, rv.z, rv.w};
#pragma unroll
                  for (int j = 0; j < 4; ++j) {
                    const float2 p = unpack_bf16x2(ru[j]);
                    f[2 * j] += p.x;
                    f[2 * j + 1] += p.y;
                  }
                }
                uint4 o;
                o.x = pack_bf16x2(f[0], f[1]);
                o.y = pack_bf16x2(f[2], f[3]);
                o.z = pack_bf16x2(f[4], f[5]);
                o.w = pack_bf16x2(f[6], f[7]);
                *reinterpret_cast<uint4*>(crow + v * 8) = o;
              }
            } else {
              for (int j = 0; j < 32 && col0 + j < N; ++j) {
                float f = __uint_as_float(r[j]);
                if (EPI == EPI_BF16_ADD) f += __bfloat162float(rrow[j]);
                crow[j] = __float2bfloat16_rn(f);
              }
            }
          } else {
            float* crow = reinterpret_cast<float*>(Cptr) + static_cast<size_t>(row) * ldc + col0;
            if (full) {
#pragma unroll
              for (int v = 0; v < 8; ++v) {
                float4 o;
                o.x = __uint_as_float(r[v * 4 + 0]);
                o.y = __uint_as_float(r[v * 4 + 1]);
                o.z = __uint_as_float(r[v * 4 + 2]);
                o.w = __uint_as_float(r[v * 4 + 3]);
                if (EPI == EPI_F32_ACCUM) {
                  const float4 old = *reinterpret_cast<const float4*>(crow + v * 4);
                  o.x += old.x;
                  o.y += old.y;
                  o.z += old.z;
                  o.w += old.w;
                }
                *reinterpret_cast<float4*>(crow + v * 4) = o;
              }
            } else {
              for (int j = 0; j < 32 && col0 + j < N; ++j) {
                const float f = __uint_as_float(r[j]);
                crow[j] = (EPI == EPI_F32_ACCUM) ? crow[j] + f : f;
              }
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&tempty_bar[acc]);
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
  } else if (comm_ctas == 0 && comm_task.kind != COMM_NONE) {
    // ------------------------------------------------ communication warps (6..15) of a launch that carries a collective
    const CommGroup g = {static_cast<int>(threadIdx.x) - NUM_THREADS, static_cast<int>(blockDim.x) - NUM_THREADS, 1};
    if (g.nthr >= 32) comm_run(comm_task, blockIdx.x, gridDim.x, &comm_scratch, g);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (fn == nullptr) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess || p == nullptr)
      return nullptr;
    fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

}  // namespace

// 2-D bf16 tensor map with 128-byte swizzle; `inner` is the contiguous extent, `ld` the row pitch in elements.
int make_tensor_map_bf16_2d(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer, uint64_t ld,
                            uint32_t box_inner, uint32_t box_outer) {
  EncodeTiledFn fn = get_encode_fn();
  if (fn == nullptr) return -1;
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0 || (ld * 2) % 16 != 0) return -2;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {ld * 2};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : -3;
}

// 2-D fp32 tensor map with 128-byte swizzle (used for reduce-add stores of fp32 tiles; box_inner * 4 must be 128).
int make_tensor_map_f32_2d(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer, uint64_t ld,
                           uint32_t box_inner, uint32_t box_outer) {
  EncodeTiledFn fn = get_encode_fn();
  if (fn == nullptr) return -1;
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0 || (ld * 4) % 16 != 0 || box_inner * 4 != 128) return -2;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {ld * 4};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : -3;
}

template <int A_MN, int B_MN, int EPI>
static int launch_gemm(const CUtensorMap& ta, const CUtensorMap& tb, void* C, const void* R, int M, int N, int K,
                       int ldc, int vec_ok, const int* b_ready, int rows_per_flag, int ready_value, int* status,
                       int num_sms, const CommTask& comm_task, int comm_ctas, cudaStream_t stream) {
  auto kern = gemm_bf16_kernel<A_MN, B_MN, EPI>;
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
    if (e != cudaSuccess) return -10;
    configured = true;
  }
  const int tiles = ((M + BM - 1) / BM) * ((N + BN - 1) / BN);
  if (comm_ctas < 0 || comm_ctas >= num_sms) return -12;
  const int gemm_ctas = tiles < num_sms - comm_ctas ? tiles : num_sms - comm_ctas;
  const bool carries = comm_ctas > 0 || comm_task.kind != COMM_NONE;
  kern<<<gemm_ctas + comm_ctas, carries ? NUM_THREADS_COMM : NUM_THREADS, SMEM_BYTES, stream>>>(ta, tb, C, reinterpret_cast<const bf16*>(R), M, N, K, ldc,
                                                                  vec_ok, b_ready, rows_per_flag, ready_value, status,
                                                                  comm_task, comm_ctas);
  return cudaGetLastError() == cudaSuccess ? 0 : -11;
}

}  // namespace ob

namespace ob {
int gemm2_dispatch(const void* A, const void* B, void* C, const void* R, int M, int N, int K, int lda, int ldb, int ldc,
                   int a_mn_major, int b_mn_major, int epi, int* status, int num_sms, const CommTask& comm_task, int comm_ctas,
                   cudaStream_t stream);
}
static int g_gemm_pair_mode = 0;  // 1: use the two-CTA (cta_group::2) kernel of gemm2.cu where it applies

extern "C" void ob_set_gemm_pair_mode(int on) { g_gemm_pair_mode = on; }
extern "C" int ob_get_gemm_pair_mode(void) { return g_gemm_pair_mode; }

static int gemm_dispatch(const void* A, const void* B, void* C, const void* R, int M, int N, int K, int lda, int ldb,
                         int ldc, int a_mn_major, int b_mn_major, int epi, const int* b_ready, int rows_per_flag,
                         int ready_value, int* status, int num_sms, const ob::CommTask& comm_task, int comm_ctas,
                         cudaStream_t stream) {
  using namespace ob;
  if (M <= 0 || N <= 0 || K <= 0) return 0;
  if (num_sms <= 0) num_sms = 148;
  if (g_gemm_pair_mode && b_ready == nullptr && M > 128 && num_sms >= 2 + comm_ctas) {
    const int rc2 = gemm2_dispatch(A, B, C, R, M, N, K, lda, ldb, ldc, a_mn_major, b_mn_major, epi, status, num_sms & ~1,
                                   comm_task, comm_ctas, stream);
    if (rc2 != -20) return rc2;
  }
  CUtensorMap ta, tb;
  int rc;
  // K-major operand: inner = K, outer = rows, box = 64 x rows-per-tile.  MN-major: inner = rows, outer = K, box 64 x 64.
  rc = a_mn_major ? make_tensor_map_bf16_2d(&ta, A, (uint64_t)M, (uint64_t)K, (uint64_t)lda, 64, BK)
                  : make_tensor_map_bf16_2d(&ta, A, (uint64_t)K, (uint64_t)M, (uint64_t)lda, BK, BM);
  if (rc != 0) return rc;
  rc = b_mn_major ? make_tensor_map_bf16_2d(&tb, B, (uint64_t)N, (uint64_t)K, (uint64_t)ldb, 64, BK)
                  : make_tensor_map_bf16_2d(&tb, B, (uint64_t)K, (uint64_t)N, (uint64_t)ldb, BK, BN);
  if (rc != 0) return rc;
  const int esize = (epi == EPI_BF16 || epi == EPI_BF16_ADD) ? 2 : 4;
  int vec_ok = ((reinterpret_cast<uintptr_t>(C) & 15) == 0) && ((static_cast<size_t>(ldc) * esize) % 16 == 0);
  if (epi == EPI_BF16_ADD) vec_ok = vec_ok && ((reinterpret_cast<uintptr_t>(R) & 15) == 0);
  if (num_sms <= 0) num_sms = 148;

#define OB_DISPATCH(AM, BMJ, E)                                                                                      \
  if (a_mn_major == AM && b_mn_major == BMJ && epi == E)                                                             \
    return launch_gemm<AM, BMJ, E>(ta, tb, C, R, M, N, K, ldc, vec_ok, b_ready, rows_per_flag, ready_value, status,  \
                                   num_sms, comm_task, comm_ctas, stream);
  OB_DISPATCH(0, 0, EPI_BF16)
  OB_DISPATCH(0, 0, EPI_BF16_ADD)
  OB_DISPATCH(0, 0, EPI_F32_STORE)
  OB_DISPATCH(0, 1, EPI_BF16)
  OB_DISPATCH(0, 1, EPI_BF16_ADD)
  OB_DISPATCH(1, 1, EPI_BF16)
  OB_DISPATCH(1, 1, EPI_F32_ACCUM)
  OB_DISPATCH(1, 1, EPI_F32_STORE)
  OB_DISPATCH(1, 0, EPI_BF16)
#undef OB_DISPATCH
  return -20;  // combination not instantiated
}

extern "C" int ob_gemm_bf16(const void* A, const void* B, void* C, const void* R, int M, int N, int K, int lda, int ldb,
                            int ldc, int a_mn_major, int b_mn_major, int epi, const int* b_ready, int rows_per_flag,
                            int ready_value, int* status, int num_sms, cudaStream_t stream) {
  ob::CommTask none = {};
  return gemm_dispatch(A, B, C, R, M, N, K, lda, ldb, ldc, a_mn_major, b_mn_major, epi, b_ready, rows_per_flag, ready_value,
                       status, num_sms, none, 0, stream);
}

// Same GEMM with `comm_ctas` blocks of the grid executing `*task` (layout of ob::CommTask, see comm.cuh) concurrently.
extern "C" int ob_gemm_bf16_comm(const void* A, const void* B, void* C, const void* R, int M, int N, int K, int lda,
                                 int ldb, int ldc, int a_mn_major, int b_mn_major, int epi, int* status, int num_sms,
                                 const void* task, int comm_ctas, cudaStream_t stream) {
  const ob::CommTask* t = reinterpret_cast<const ob::CommTask*>(task);
  if (t == nullptr || t->world > ob::COMM_MAX_WORLD) return -13;
  return gemm_dispatch(A, B, C, R, M, N, K, lda, ldb, ldc, a_mn_major, b_mn_major, epi, nullptr, 0, 0, status, num_sms, *t,
                       comm_ctas, stream);
}

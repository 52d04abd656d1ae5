// bf16 GEMM with tcgen05 `cta_group::2`: two CTAs of a thread-block cluster (one per SM of a pair) cooperate on a
// 256 x 256 output tile.  Each CTA stages its own 128 rows of A and its own 128-column half of B, the leader CTA issues
// one 256 x 256 x 16 MMA per K step for both, and each CTA ends up with its 128 x 256 half of the accumulator in its
// own TMEM.  Compared with the single-CTA kernel (gemm.cu) every SM loads a third less operand data per FLOP, which
// leaves room for a six-stage ring (192 KiB) and keeps the tensor pipe fed under L2 latency.
//
// Roles per CTA (512 threads when the launch carries a collective, else 192): warp 0 TMA producer, warp 1 MMA issuer
// (leader CTA only; owns the TMEM allocation in both CTAs), warps 2..5 epilogue, warps 6..15 communication (comm.cuh:
// every CTA moves its share of the collective with its spare warps; alternatively whole CTA pairs are set aside for it).
// Cross-CTA signalling: operand loads of both CTAs complete on the leader's `full` barrier (the `cta_group::2` form of
// the tensor copy takes a cluster address for its barrier; each CTA still fetches only its own tile); the leader's tcgen05.commit arrives
// on the `empty` / `accumulator full` barriers of both CTAs; epilogue threads of both CTAs arrive on the leader's
// `accumulator empty` barrier.  The cluster synchronises once after set-up and once before tear-down, so neither CTA
// can exit while its partner may still touch its shared memory, barriers or TMEM.
#include "common.cuh"
#include "comm.cuh"
#include "api.h"

namespace ob {

int make_tensor_map_bf16_2d(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer, uint64_t ld,
                            uint32_t box_inner, uint32_t box_outer);
int make_tensor_map_f32_2d(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer, uint64_t ld,
                           uint32_t box_inner, uint32_t box_outer);
int g_gemm2_tma_store = 1;  // 0: epilogue threads store their rows directly (kept for comparison, see ob_set_gemm_tma_store)

namespace {

constexpr int G2_BM = 128;   // rows per CTA (256 per pair)
constexpr int G2_BN = 256;   // columns per pair; each CTA stages 128 of them
constexpr int G2_BK = 64;
constexpr int G2_STAGES = 6;
constexpr int G2_A_BYTES = G2_BM * G2_BK * 2;        // 16 KiB
constexpr int G2_B_BYTES = (G2_BN / 2) * G2_BK * 2;  // 16 KiB
constexpr int G2_STAGE_BYTES = G2_A_BYTES + G2_B_BYTES;
constexpr int G2_CHUNK_BYTES = 64 * G2_BK * 2;
constexpr int G2_THREADS = 192;
constexpr int G2_THREADS_COMM = 512;
constexpr int G2_OUT_BYTES = 4096;  // one epilogue warp's staging tile: 32 rows x 128 bytes, 128-byte swizzle
constexpr int G2_OUT_TOTAL = 4 * 2 * G2_OUT_BYTES;  // four epilogue warps, double buffered
constexpr int G2_SMEM = 1024 + G2_STAGES * G2_STAGE_BYTES + G2_OUT_TOTAL + 256;
constexpr int G2_GROUP_M = 8;

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// shared::cluster address of the same shared-memory location in CTA `rank` of this cluster
__device__ __forceinline__ uint32_t map_to_cta(uint32_t smem_addr, uint32_t rank) {
  uint32_t out;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(out) : "r"(smem_addr), "r"(rank));
  return out;
}

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_alloc_2cta(uint32_t* smem_result, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_result)), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tmem_relinquish_2cta() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_2cta(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// TMA load whose completion bytes are credited to a barrier given by cluster address (the pair leader's barrier).
__device__ __forceinline__ void tma_load_2d_pair(void* smem_dst, const CUtensorMap* map, uint32_t bar_cluster_addr, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];"
      ::"r"(smem_u32(smem_dst)), "l"(map), "r"(bar_cluster_addr), "r"(x), "r"(y)
      : "memory");
}

__device__ __forceinline__ void umma_f16_ss_2cta(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n"
      " .reg .pred p;\n"
      " setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n"
      "}\n" ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive (once all MMAs issued so far by this thread have completed) on a barrier given by cluster address.
__device__ __forceinline__ void umma_commit_2cta(uint32_t bar_cluster_addr) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar_cluster_addr) : "memory");
}

__device__ __forceinline__ void mbar_arrive_cluster(uint32_t bar_cluster_addr) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(bar_cluster_addr) : "memory");
}

struct Tile2 {
  int m, n;
};

__device__ __forceinline__ Tile2 tile2_coord(int t, int tiles_m, int tiles_n) {
  const int group_size = G2_GROUP_M * tiles_n;
  const int group = t / group_size;
  const int first_m = group * G2_GROUP_M;
  const int rows = min(tiles_m - first_m, G2_GROUP_M);
  const int in_group = t - group * group_size;
  return {first_m + in_group % rows, in_group / rows};
}

template <int A_MN, int B_MN, int EPI>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(G2_THREADS_COMM, 1)
gemm2_bf16_kernel(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b,
                  const __grid_constant__ CUtensorMap tma_c, int use_tma_c,
                  void* __restrict__ Cptr, const bf16* __restrict__ Rptr, int M, int N, int K, int ldc, int vec_ok,
                  int* __restrict__ status, const __grid_constant__ CommTask comm_task, int comm_ctas) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ CommScratch comm_scratch;
  if (static_cast<int>(blockIdx.x) < comm_ctas) {  // communication pairs (comm_ctas is even): no TMEM, no barriers
    const CommGroup g = {static_cast<int>(threadIdx.x), static_cast<int>(blockDim.x), 1};
    comm_run(comm_task, blockIdx.x, comm_ctas, &comm_scratch, g);
    return;
  }
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int pair = (static_cast<int>(blockIdx.x) - comm_ctas) >> 1;
  const int num_pairs = (static_cast<int>(gridDim.x) - comm_ctas) >> 1;

  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + G2_STAGES * G2_A_BYTES;
  uint8_t* sOut = smem + G2_STAGES * G2_STAGE_BYTES;  // 1024-byte aligned, as the swizzle pattern of the staging tiles needs
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(sOut + G2_OUT_TOTAL);
  uint64_t* empty_bar = full_bar + G2_STAGES;
  uint64_t* tfull_bar = empty_bar + G2_STAGES;
  uint64_t* tempty_bar = tfull_bar + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty_bar + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int tiles_m = (M + 2 * G2_BM - 1) / (2 * G2_BM);
  const int tiles_n = (N + G2_BN - 1) / G2_BN;
  const int num_tiles = tiles_m * tiles_n;
  const int k_blocks = (K + G2_BK - 1) / G2_BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < G2_STAGES; ++s) {
      mbar_init(&full_bar[s], 1);   // used in the leader: one arrive.expect_tx per phase
      mbar_init(&empty_bar[s], 1);  // one commit arrival per phase, in each CTA
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull_bar[a], 1);
      mbar_init(&tempty_bar[a], 256);  // used in the leader: epilogue threads of both CTAs
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc_2cta(tmem_slot, 512);
    tmem_relinquish_2cta();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // partner's barriers are initialised and its TMEM is allocated
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer (both CTAs)
    if (lane == 0) {
      prefetch_tensormap(&tma_a);
      prefetch_tensormap(&tma_b);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int t = pair; t < num_tiles && ok; t += num_pairs) {
        const Tile2 tc = tile2_coord(t, tiles_m, tiles_n);
        const int m0 = tc.m * 2 * G2_BM + static_cast<int>(rank) * G2_BM;
        const int n0 = tc.n * G2_BN + static_cast<int>(rank) * (G2_BN / 2);
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1u, abort_flag, status, ST_TIMEOUT_PRODUCER)) {
            ok = false;
            break;
          }
          if (leader) mbar_expect_tx(&full_bar[stage], 2 * G2_STAGE_BYTES);
          const uint32_t bar = map_to_cta(smem_u32(&full_bar[stage]), 0);
          uint8_t* a_dst = sA + stage * G2_A_BYTES;
          uint8_t* b_dst = sB + stage * G2_B_BYTES;
          const int k0 = kb * G2_BK;
          if (A_MN) {
#pragma unroll
            for (int c = 0; c < G2_BM / 64; ++c) tma_load_2d_pair(a_dst + c * G2_CHUNK_BYTES, &tma_a, bar, m0 + c * 64, k0);
          } else {
            tma_load_2d_pair(a_dst, &tma_a, bar, k0, m0);
          }
          if (B_MN) {
#pragma unroll
            for (int c = 0; c < (G2_BN / 2) / 64; ++c) tma_load_2d_pair(b_dst + c * G2_CHUNK_BYTES, &tma_b, bar, n0 + c * 64, k0);
          } else {
            tma_load_2d_pair(b_dst, &tma_b, bar, k0, n0);
          }
          if (++stage == G2_STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) {
        const long long t0 = clock64();
        while (clock64() - t0 < 2000000LL) {
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------- MMA issuer (leader CTA only)
    if (leader && lane == 0) {
      constexpr uint32_t idesc = make_idesc_bf16(2 * G2_BM, G2_BN, A_MN, B_MN);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int t = pair; t < num_tiles && ok; t += num_pairs) {
        if (!mbar_wait(&tempty_bar[acc], acc_phase ^ 1u, abort_flag, status, ST_TIMEOUT_MMA)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * G2_BN);
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!mbar_wait(&full_bar[stage], phase, abort_flag, status, ST_TIMEOUT_MMA)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(sA + stage * G2_A_BYTES);
          const uint32_t b_addr = smem_u32(sB + stage * G2_B_BYTES);
#pragma unroll
          for (int k = 0; k < G2_BK / 16; ++k) {
            const uint64_t a_desc = A_MN ? make_smem_desc_sw128(a_addr + k * 2048, G2_CHUNK_BYTES, 1024)
                                         : make_smem_desc_sw128(a_addr + k * 32, 16, 1024);
            const uint64_t b_desc = B_MN ? make_smem_desc_sw128(b_addr + k * 2048, G2_CHUNK_BYTES, 1024)
                                         : make_smem_desc_sw128(b_addr + k * 32, 16, 1024);
            umma_f16_ss_2cta(d_tmem, a_desc, b_desc, idesc, (kb > 0 || k > 0) ? 1u : 0u);
          }
          // the stage becomes reusable in both CTAs once these MMAs have read it
          umma_commit_2cta(map_to_cta(smem_u32(&empty_bar[stage]), 0));
          umma_commit_2cta(map_to_cta(smem_u32(&empty_bar[stage]), 1));
          if (++stage == G2_STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit_2cta(map_to_cta(smem_u32(&tfull_bar[acc]), 0));
        umma_commit_2cta(map_to_cta(smem_u32(&tfull_bar[acc]), 1));
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
    }
  } else if (warp < 6) {
    // --------------------------------------------------------------------- epilogue (both CTAs)
    const int quarter = warp & 3;
    int acc = 0;
    uint32_t acc_phase = 0;
    uint32_t out_buf = 0;
    for (int t = pair; t < num_tiles; t += num_pairs) {
      const Tile2 tc = tile2_coord(t, tiles_m, tiles_n);
      const int row = tc.m * 2 * G2_BM + static_cast<int>(rank) * G2_BM + quarter * 32 + lane;
      const int n0 = tc.n * G2_BN;
      if (!mbar_wait(&tfull_bar[acc], acc_phase, abort_flag, status, ST_TIMEOUT_EPILOGUE)) break;
      tc_fence_after();
      __syncwarp();
      const uint32_t t_addr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + static_cast<uint32_t>(acc * G2_BN);
      if (use_tma_c) {
        // Output through shared memory: every epilogue warp packs its 32 rows of a 64-column (bf16) or 32-column (fp32)
        // slab into a 128-byte-swizzled staging tile and one lane hands it to the TMA unit, as a plain store or, for the
        // accumulating epilogue, as a reduce-add performed at the memory side (the old values are never loaded).  Rows and
        // columns beyond the matrix are clipped by the tensor map.  Two staging tiles per warp alternate.
        constexpr bool OUT16 = (EPI == EPI_BF16 || EPI == EPI_BF16_ADD);
        constexpr int SLAB = OUT16 ? 64 : 32;  // columns per TMA operation (128 bytes per row)
        const int row0 = tc.m * 2 * G2_BM + static_cast<int>(rank) * G2_BM + quarter * 32;
#pragma unroll 1
        for (int sl = 0; sl < G2_BN / SLAB; ++sl) {
          const int colS = n0 + sl * SLAB;
          uint8_t* buf = sOut + (quarter * 2 + (out_buf & 1)) * G2_OUT_BYTES;
          if (lane == 0) tma_store_wait_read<1>();  // the store issued from this buffer two slabs ago has read it
          __syncwarp();
          uint8_t* myrow = buf + lane * 128;
#pragma unroll
          for (int hc = 0; hc < SLAB / 32; ++hc) {
            uint32_t r[32];
            tmem_ld_32x32b_x32(t_addr + sl * SLAB + hc * 32, r);
            tmem_ld_wait();
            if (OUT16) {
              const int col0 = colS + hc * 32;
#pragma unroll
              for (int v = 0; v < 4; ++v) {
                float f[8];
#pragma unroll
                for (int j = 0; j < 8; ++j) f[j] = __uint_as_float(r[v * 8 + j]);
                if (EPI == EPI_BF16_ADD && row < M && col0 + v * 8 + 8 <= N) {
                  const uint4 rv = *reinterpret_cast<const uint4*>(Rptr + static_cast<size_t>(row) * ldc + col0 + v * 8);
                  const uint32_t ru[4] = {rv.x, rv.y, rv.z, rv.w};
#pragma unroll
                  for (int j = 0; j < 4; ++j) {
                    const float2 pr = unpack_bf16x2(ru[j]);
                    f[2 * j] += pr.x;
                    f[2 * j + 1] += pr.y;
                  }
                }
                uint4 o;
                o.x = pack_bf16x2(f[0], f[1]);
                o.y = pack_bf16x2(f[2], f[3]);
                o.z = pack_bf16x2(f[4], f[5]);
                o.w = pack_bf16x2(f[6], f[7]);
                const int chunk = hc * 4 + v;
                *reinterpret_cast<uint4*>(myrow + ((chunk ^ (lane & 7)) << 4)) = o;
              }
            } else {
#pragma unroll
              for (int v = 0; v < 8; ++v)
                *reinterpret_cast<uint4*>(myrow + ((v ^ (lane & 7)) << 4)) = make_uint4(r[v * 4 + 0], r[v * 4 + 1], r[v * 4 + 2], r[v * 4 + 3]);
            }
          }
          fence_proxy_async();
          __syncwarp();
          if (lane == 0 && row0 < M && colS < N) {
            if (EPI == EPI_F32_ACCUM) tma_reduce_add_2d(&tma_c, buf, colS, row0);
            else tma_store_2d(&tma_c, buf, colS, row0);
          }
          if (lane == 0) tma_store_commit();
          ++out_buf;
        }
        tc_fence_before();
        if (leader) mbar_arrive(&tempty_bar[acc]);
        else mbar_arrive_cluster(map_to_cta(smem_u32(&tempty_bar[acc]), 0));
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1u;
        }
        continue;
      }
#pragma unroll 1
      for (int c = 0; c < G2_BN / 32; ++c) {
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
                    const float2 pr = unpack_bf16x2(ru[j]);
                    f[2 * j] += pr.x;
                    f[2 * j + 1] += pr.y;
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
      // the accumulator may be overwritten once all 256 epilogue threads of the pair have drained it
      if (leader) mbar_arrive(&tempty_bar[acc]);
      else mbar_arrive_cluster(map_to_cta(smem_u32(&tempty_bar[acc]), 0));
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
    if (use_tma_c && lane == 0) tma_store_wait<0>();  // every store / reduce-add of this warp has been performed
  } else if (comm_ctas == 0 && comm_task.kind != COMM_NONE) {
    // ------------------------------------------------ communication warps (6..15) of a launch that carries a collective:
    // this CTA's share of the task, moved by plain peer loads while the six role warps above run the tiles
    const CommGroup g = {static_cast<int>(threadIdx.x) - G2_THREADS, static_cast<int>(blockDim.x) - G2_THREADS, 1};
    if (g.nthr >= 32) comm_run(comm_task, blockIdx.x, gridDim.x, &comm_scratch, g);
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // partner has finished everything that touches this CTA's memory
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_2cta(tmem_base, 512);
  }
}

template <int A_MN, int B_MN, int EPI>
int launch_gemm2(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tcm, int use_tma_c, void* C, const void* R, int M, int N, int K, int ldc, int vec_ok,
                 int* status, int num_sms, const CommTask& comm_task, int comm_ctas, cudaStream_t stream) {
  auto kern = gemm2_bf16_kernel<A_MN, B_MN, EPI>;
  static bool configured = false;
  if (!configured) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, G2_SMEM) != cudaSuccess) return -10;
    configured = true;
  }
  comm_ctas &= ~1;  // whole pairs
  if (comm_ctas < 0 || comm_ctas + 2 > num_sms) return -12;
  const int tiles = ((M + 2 * G2_BM - 1) / (2 * G2_BM)) * ((N + G2_BN - 1) / G2_BN);
  int pairs = (num_sms - comm_ctas) / 2;
  if (tiles < pairs) pairs = tiles;
  const bool carries = comm_ctas > 0 || comm_task.kind != COMM_NONE;
  kern<<<2 * pairs + comm_ctas, carries ? G2_THREADS_COMM : G2_THREADS, G2_SMEM, stream>>>(
      ta, tb, tcm, use_tma_c, C, reinterpret_cast<const bf16*>(R), M, N, K, ldc, vec_ok, status, comm_task, comm_ctas);
  return cudaGetLastError() == cudaSuccess ? 0 : -11;
}

}  // namespace

// Same contract as the single-CTA dispatcher in gemm.cu; returns -20 for a combination that is not instantiated.
int gemm2_dispatch(const void* A, const void* B, void* C, const void* R, int M, int N, int K, int lda, int ldb, int ldc,
                   int a_mn_major, int b_mn_major, int epi, int* status, int num_sms, const CommTask& comm_task, int comm_ctas,
                   cudaStream_t stream) {
  CUtensorMap ta, tb;
  int rc = a_mn_major ? make_tensor_map_bf16_2d(&ta, A, (uint64_t)M, (uint64_t)K, (uint64_t)lda, 64, G2_BK)
                      : make_tensor_map_bf16_2d(&ta, A, (uint64_t)K, (uint64_t)M, (uint64_t)lda, G2_BK, G2_BM);
  if (rc != 0) return rc;
  rc = b_mn_major ? make_tensor_map_bf16_2d(&tb, B, (uint64_t)N, (uint64_t)K, (uint64_t)ldb, 64, G2_BK)
                  : make_tensor_map_bf16_2d(&tb, B, (uint64_t)K, (uint64_t)N, (uint64_t)ldb, G2_BK, G2_BN / 2);
  if (rc != 0) return rc;
  const int esize = (epi == EPI_BF16 || epi == EPI_BF16_ADD) ? 2 : 4;
  int vec_ok = ((reinterpret_cast<uintptr_t>(C) & 15) == 0) && ((static_cast<size_t>(ldc) * esize) % 16 == 0);
  if (epi == EPI_BF16_ADD) vec_ok = vec_ok && ((reinterpret_cast<uintptr_t>(R) & 15) == 0);
  // output tiles leave through shared memory and the TMA unit when the output is 16-byte aligned with a 16-byte pitch
  CUtensorMap tcm = ta;
  int use_tma_c = vec_ok && (N % 8 == 0) && g_gemm2_tma_store;
  if (use_tma_c) {
    rc = esize == 2 ? make_tensor_map_bf16_2d(&tcm, C, (uint64_t)N, (uint64_t)M, (uint64_t)ldc, 64, 32)
                    : make_tensor_map_f32_2d(&tcm, C, (uint64_t)N, (uint64_t)M, (uint64_t)ldc, 32, 32);
    if (rc != 0) use_tma_c = 0;
  }
#define OB_DISPATCH2(AM, BMJ, E)                                                                                         \
  if (a_mn_major == AM && b_mn_major == BMJ && epi == E)                                                                 \
    return launch_gemm2<AM, BMJ, E>(ta, tb, tcm, use_tma_c, C, R, M, N, K, ldc, vec_ok, status, num_sms, comm_task, comm_ctas, stream);
  OB_DISPATCH2(0, 0, EPI_BF16)
  OB_DISPATCH2(0, 0, EPI_BF16_ADD)
  OB_DISPATCH2(0, 0, EPI_F32_STORE)
  OB_DISPATCH2(0, 1, EPI_BF16)
  OB_DISPATCH2(0, 1, EPI_BF16_ADD)
  OB_DISPATCH2(1, 1, EPI_BF16)
  OB_DISPATCH2(1, 1, EPI_F32_ACCUM)
  OB_DISPATCH2(1, 1, EPI_F32_STORE)
  OB_DISPATCH2(1, 0, EPI_BF16)
#undef OB_DISPATCH2
  return -20;
}

}  // namespace ob

extern "C" void ob_set_gemm_tma_store(int on) { ob::g_gemm2_tma_store = on; }

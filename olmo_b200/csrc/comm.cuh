// Peer-memory collectives as device functions, so that the same code runs either as a stand-alone kernel or as the
// "communication CTAs" of a GEMM launch (gemm.cu): the first `comm_ctas` blocks of the grid execute a CommTask while the
// remaining blocks compute tiles, which overlaps NVLink traffic with tensor-core work inside one kernel.
//
// Remote data is read through peer-mapped pointers (NVLink 5 via NVSwitch) in one of two ways, chosen per task:
//  * plain 16-byte loads issued by every thread of the CTA (mode 0), or
//  * untiled bulk-async copies (`cp.async.bulk`, never multicast) from the peer's memory into a ring of shared-memory
//    stages (mode COMM_MODE_BULK).  One thread keeps the whole ring (up to 192 KiB per CTA) in flight, which is what
//    lets a handful of communication CTAs saturate the links instead of dozens.
// Waits on a peer's flag or on a stage barrier are bounded (common.cuh) and report through the status word.
#pragma once

#include "common.cuh"

namespace ob {

constexpr int COMM_MAX_WORLD = 8;

enum : int { COMM_NONE = 0, COMM_ALL_GATHER = 1, COMM_REDUCE_SCATTER = 2 };
enum : int { COMM_MODE_BULK = 1, COMM_MODE_SELF = 2 };

struct CommTask {
  int kind;
  int world;
  int rank;
  int wait_value;                 // proceed with peer p once *wait_flags[p] >= wait_value (null flag: no wait)
  long long elems;                // all-gather: bf16 elements per peer region; reduce-scatter: fp32 elements of my slice
  long long dst_peer_stride;      // all-gather: elements between consecutive ranks' regions in dst
  const void* src[COMM_MAX_WORLD];
  const int* wait_flags[COMM_MAX_WORLD];
  void* dst;
  float scale;                    // reduce-scatter: dst += scale * sum_p src[p]
  float* sumsq_partials;          // reduce-scatter, optional: partial[c] += sum of squares of dst after CTA c's additions
  int* status;
  long long wait_cycles;          // budget of every flag wait in this task (0: library default)
  int mode;                       // bit 0 (COMM_MODE_BULK): bulk-async copies through shared memory;
                                  // bit 1 (COMM_MODE_SELF): an all-gather also copies this rank's own region
  int reserved;
};

__device__ __forceinline__ uint4 ld_peer_16(const void* p) {
  uint4 v;
  asm volatile("ld.global.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p) : "memory");
  return v;
}

// Every thread of the CTA calls this; returns false if the wait ran out (whole CTA agrees).
__device__ __forceinline__ bool comm_wait_peer(const CommTask& t, int p, int* smem_ok) {
  if (t.wait_flags[p] == nullptr) return true;
  __syncthreads();
  if (threadIdx.x == 0)
    *smem_ok = flag_wait_ge(t.wait_flags[p], t.wait_value, nullptr, t.status,
                            t.wait_cycles > 0 ? t.wait_cycles : OB_WAIT_BUDGET_CYCLES) ? 1 : 0;
  __syncthreads();
  return *smem_ok != 0;
}

// Copy every peer's region (except this rank's own, which is already in place) into dst.  16-byte granularity:
// `elems` must be a multiple of 8 bf16 elements and all bases 16-byte aligned.
__device__ __forceinline__ void comm_all_gather(const CommTask& t, int cta, int nctas, int* smem_ok) {
  const long long vecs = t.elems >> 3;  // 16-byte vectors per peer
  constexpr int UNROLL = 8;
  const long long tile = static_cast<long long>(blockDim.x) * UNROLL;  // vectors per CTA iteration
  for (int q = (t.mode & COMM_MODE_SELF) ? 0 : 1; q < t.world; ++q) {
    const int p = (t.rank + q) % t.world;  // start with the next rank so that peers are read evenly
    if (!comm_wait_peer(t, p, smem_ok)) return;
    const uint4* src = reinterpret_cast<const uint4*>(t.src[p]);
    uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<bf16*>(t.dst) + static_cast<long long>(p) * t.dst_peer_stride);
    for (long long base = static_cast<long long>(cta) * tile; base < vecs; base += static_cast<long long>(nctas) * tile) {
      uint4 v[UNROLL];
#pragma unroll
      for (int u = 0; u < UNROLL; ++u) {
        const long long i = base + static_cast<long long>(u) * blockDim.x + threadIdx.x;
        if (i < vecs) v[u] = ld_peer_16(src + i);
      }
#pragma unroll
      for (int u = 0; u < UNROLL; ++u) {
        const long long i = base + static_cast<long long>(u) * blockDim.x + threadIdx.x;
        if (i < vecs) dst[i] = v[u];
      }
    }
  }
}

// dst[i] += scale * (src[0][i] + src[1][i] + ... + src[W-1][i]) over my slice, summed in rank order (deterministic).
// `elems` must be a multiple of 4 fp32 elements.  Each thread keeps 8 sixteen-byte loads in flight (U = 8 / W vectors
// from each of the W ranks) because a communication CTA has few warps to hide NVLink latency with.
template <int W, int U>
struct RsTile {
  uint4 v[W][U];
  float4 d[U];
};

template <int W, int U>
__device__ __forceinline__ void rs_load(const CommTask& t, RsTile<W, U>& r, long long base, long long vecs) {
  const float4* dst = reinterpret_cast<const float4*>(t.dst);
#pragma unroll
  for (int u = 0; u < U; ++u) {
    const long long i = base + static_cast<long long>(u) * blockDim.x + threadIdx.x;
    if (i < vecs) {
#pragma unroll
      for (int p = 0; p < W; ++p) r.v[p][u] = ld_peer_16(reinterpret_cast<const uint4*>(t.src[p]) + i);
      r.d[u] = dst[i];
    }
  }
}

template <int W, int U>
__device__ __forceinline__ float rs_finish(const CommTask& t, RsTile<W, U>& r, long long base, long long vecs) {
  float4* dst = reinterpret_cast<float4*>(t.dst);
  float ss = 0.f;
#pragma unroll
  for (int u = 0; u < U; ++u) {
    const long long i = base + static_cast<long long>(u) * blockDim.x + threadIdx.x;
    if (i < vecs) {
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int p = 0; p < W; ++p) {
        acc.x += __uint_as_float(r.v[p][u].x);
        acc.y += __uint_as_float(r.v[p][u].y);
        acc.z += __uint_as_float(r.v[p][u].z);
        acc.w += __uint_as_float(r.v[p][u].w);
      }
      acc.x *= t.scale; acc.y *= t.scale; acc.z *= t.scale; acc.w *= t.scale;
      float4 d = r.d[u];
      d.x += acc.x; d.y += acc.y; d.z += acc.z; d.w += acc.w;
      dst[i] = d;
      ss += d.x * d.x + d.y * d.y + d.z * d.z + d.w * d.w;
    }
  }
  return ss;
}

// One tile of U vectors from each of the W ranks is in flight per thread.  (Keeping a second tile in registers does not
// help: a wait for the older tile's loads also waits for the younger one's, so each memory round trip still retires one
// tile; what counts is the number of bytes requested before the first use.)
template <int W, int U>
__device__ __forceinline__ float comm_rs_loop(const CommTask& t, int cta, int nctas) {
  const long long vecs = t.elems >> 2;
  const long long tile = static_cast<long long>(blockDim.x) * U;
  const long long stride = static_cast<long long>(nctas) * tile;
  float ss = 0.f;
  for (long long base = static_cast<long long>(cta) * tile; base < vecs; base += stride) {
    RsTile<W, U> r;
    rs_load<W, U>(t, r, base, vecs);
    ss += rs_finish<W, U>(t, r, base, vecs);
  }
  return ss;
}

__device__ __forceinline__ void comm_reduce_scatter(const CommTask& t, int cta, int nctas, int* smem_ok, float* red) {
  for (int p = 0; p < t.world; ++p)
    if (p != t.rank && !comm_wait_peer(t, p, smem_ok)) return;
  float ss;
  switch (t.world) {
    case 1: ss = comm_rs_loop<1, 8>(t, cta, nctas); break;
    case 2: ss = comm_rs_loop<2, 6>(t, cta, nctas); break;
    case 3: ss = comm_rs_loop<3, 4>(t, cta, nctas); break;
    case 4: ss = comm_rs_loop<4, 4>(t, cta, nctas); break;
    case 5: ss = comm_rs_loop<5, 3>(t, cta, nctas); break;
    case 6: ss = comm_rs_loop<6, 2>(t, cta, nctas); break;
    case 7: ss = comm_rs_loop<7, 2>(t, cta, nctas); break;
    default: ss = comm_rs_loop<8, 2>(t, cta, nctas); break;
  }
  if (t.sumsq_partials != nullptr) {
    ss = block_sum(ss, red);
    if (threadIdx.x == 0) t.sumsq_partials[cta] += ss;
  }
}


// ------------------------------------------------------------------------------------------------ bulk-async variants

constexpr int COMM_STAGE_BYTES = 32768;
constexpr int COMM_MAX_STAGES = 6;

__device__ __forceinline__ void bulk_load_g2s(void* smem_dst, const void* gsrc, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
               ::"r"(smem_u32(smem_dst)), "l"(gsrc), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void bulk_store_s2g(void* gdst, const void* smem_src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(gdst), "r"(smem_u32(smem_src)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void bulk_wait_group_read1() { asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); }

struct CommRing {
  uint8_t* data;     // 1024-byte aligned
  uint64_t* bars;    // 16 barriers behind the ring
  int stages;        // stages of COMM_STAGE_BYTES
};

__device__ __forceinline__ CommRing comm_ring(uint8_t* smem, int smem_bytes) {
  CommRing r;
  r.data = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem) + 1023) & ~uintptr_t(1023));
  const int avail = smem_bytes - static_cast<int>(r.data - smem) - 128;
  int s = avail / COMM_STAGE_BYTES;
  r.stages = s > COMM_MAX_STAGES ? COMM_MAX_STAGES : s;
  r.bars = reinterpret_cast<uint64_t*>(r.data + r.stages * COMM_STAGE_BYTES);
  return r;
}

// Gives loads that are still in flight a bounded time to land, so that the CTA never exits under them.
__device__ __forceinline__ void comm_drain(const CommRing& r, long long first, long long issued, int* status) {
  for (long long j = first; j < issued; ++j) {
    const int s = static_cast<int>(j % r.stages);
    const uint32_t parity = static_cast<uint32_t>((j / r.stages) & 1);
    const long long t0 = clock64();
    while (!mbar_try_wait(&r.bars[s], parity)) {
      if (clock64() - t0 > 400000000LL) {
        if (status != nullptr) atomicCAS(status, 0, (int)ST_TIMEOUT_DRAIN);
        break;
      }
    }
  }
}

// All-gather, one issuing thread per CTA: 16 KiB pieces of the peers' regions travel peer memory -> shared memory ->
// local `dst`, both hops as bulk-async copies.  With P source ranks (W-1, or W when this rank's own region is copied too),
// piece g of the task is piece g / P of the (g % P)-th source, so consecutive pieces come from different peers and every
// CTA reads all of them evenly.
__device__ __forceinline__ void comm_all_gather_bulk(const CommTask& t, int cta, int nctas, uint8_t* smem, int smem_bytes) {
  if (threadIdx.x != 0 || t.world < 2) return;
  constexpr int PIECE = 16384;
  CommRing r = comm_ring(smem, smem_bytes);
  const int S = r.stages * (COMM_STAGE_BYTES / PIECE);
  if (S < 2) {
    if (t.status != nullptr) atomicCAS(t.status, 0, (int)ST_BAD_ARGUMENT);
    return;
  }
  uint64_t* bars = r.bars;
  const int SS = S > 12 ? 12 : S;  // pieces in flight (the barrier area holds 16)
  const long long budget = t.wait_cycles > 0 ? t.wait_cycles : OB_WAIT_BUDGET_CYCLES;
  const int first = (t.mode & COMM_MODE_SELF) ? 0 : 1;
  const int sources = t.world - first;
  for (int q = first; q < t.world; ++q) {
    const int p = (t.rank + q) % t.world;
    if (t.wait_flags[p] != nullptr && !flag_wait_ge(t.wait_flags[p], t.wait_value, nullptr, t.status, budget)) return;
  }
  for (int s = 0; s < SS; ++s) mbar_init(&bars[s], 1);
  fence_barrier_init();
  fence_proxy_async();
  const long long bytes = t.elems * 2;
  const long long per_peer = (bytes + PIECE - 1) / PIECE;
  const long long total = per_peer * sources;
  const long long mine = total > cta ? (total - cta + nctas - 1) / nctas : 0;
  volatile int abort_local = 0;
  auto piece = [&](long long j, const uint8_t*& src, uint8_t*& dst, uint32_t& len) {
    const long long g = cta + j * nctas;
    const int p = (t.rank + first + static_cast<int>(g % sources)) % t.world;
    const long long off = (g / sources) * PIECE;
    const long long left = bytes - off;
    len = static_cast<uint32_t>(left < PIECE ? left : PIECE);
    src = reinterpret_cast<const uint8_t*>(t.src[p]) + off;
    dst = reinterpret_cast<uint8_t*>(t.dst) + static_cast<long long>(p) * t.dst_peer_stride * 2 + off;
  };
  auto issue = [&](long long j) {
    const uint8_t* src;
    uint8_t* dst;
    uint32_t len;
    piece(j, src, dst, len);
    const int s = static_cast<int>(j % SS);
    mbar_expect_tx(&bars[s], len);
    bulk_load_g2s(r.data + s * PIECE, src, len, &bars[s]);
  };
  long long issued = 0;
  for (; issued < mine && issued < SS; ++issued) issue(issued);
  long long j = 0;
  for (; j < mine; ++j) {
    const int s = static_cast<int>(j % SS);
    if (!mbar_wait(&bars[s], static_cast<uint32_t>((j / SS) & 1), &abort_local, t.status, ST_TIMEOUT_FLAG, budget)) break;
    const uint8_t* src;
    uint8_t* dst;
    uint32_t len;
    piece(j, src, dst, len);
    bulk_store_s2g(dst, r.data + s * PIECE, len);
    bulk_commit_group();
    if (j >= 1 && issued < mine) {  // the stage of piece j-1 is free once its store has read it
      bulk_wait_group_read1();
      issue(issued);
      ++issued;
    }
  }
  if (j < mine) comm_drain(CommRing{r.data, bars, SS}, j, issued, t.status);
  bulk_wait_group0();
}

// Reduce-scatter: a stage holds one tile from each of the W ranks (this rank's own included), fetched by W bulk-async
// copies that one thread issues; all threads then add the tiles in rank order, scale, add the local shard and store.
__device__ __forceinline__ void comm_reduce_scatter_bulk(const CommTask& t, int cta, int nctas, uint8_t* smem, int smem_bytes,
                                                         int* smem_ok, float* red) {
  for (int p = 0; p < t.world; ++p)
    if (p != t.rank && !comm_wait_peer(t, p, smem_ok)) return;
  __syncthreads();  // everyone has read the last wait's verdict before the word is reused below
  CommRing r = comm_ring(smem, smem_bytes);
  const int W = t.world;
  const int S = r.stages;
  if (S < 2) {
    if (threadIdx.x == 0 && t.status != nullptr) atomicCAS(t.status, 0, (int)ST_BAD_ARGUMENT);
    return;
  }
  const int TB = (COMM_STAGE_BYTES / W) & ~15;  // bytes per rank per stage
  const long long budget = t.wait_cycles > 0 ? t.wait_cycles : OB_WAIT_BUDGET_CYCLES;
  const long long bytes = t.elems * 4;
  const long long total = (bytes + TB - 1) / TB;
  const long long mine = total > cta ? (total - cta + nctas - 1) / nctas : 0;
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) mbar_init(&r.bars[s], 1);
    *smem_ok = 0;  // doubles as the abort flag of the stage waits
    fence_barrier_init();
    fence_proxy_async();
  }
  __syncthreads();
  auto issue = [&](long long j) {
    const long long off = (cta + j * nctas) * static_cast<long long>(TB);
    const long long left = bytes - off;
    const uint32_t len = static_cast<uint32_t>(left < TB ? left : TB);
    const int s = static_cast<int>(j % S);
    mbar_expect_tx(&r.bars[s], len * W);
    for (int p = 0; p < W; ++p)
      bulk_load_g2s(r.data + s * COMM_STAGE_BYTES + p * TB, reinterpret_cast<const uint8_t*>(t.src[p]) + off, len, &r.bars[s]);
  };
  long long issued = 0;
  if (threadIdx.x == 0)
    for (; issued < mine && issued < S; ++issued) issue(issued);
  float ss = 0.f;
  long long j = 0;
  for (; j < mine; ++j) {
    const int s = static_cast<int>(j % S);
    const long long off = (cta + j * nctas) * static_cast<long long>(TB);
    const long long left = bytes - off;
    const int nvec = static_cast<int>((left < TB ? left : TB) >> 4);
    float4* dst = reinterpret_cast<float4*>(reinterpret_cast<uint8_t*>(t.dst) + off);
    float4 d[2];  // the local shard does not depend on the stage: fetch it while the stage is still arriving
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int i = threadIdx.x + u * blockDim.x;
      if (i < nvec) d[u] = dst[i];
    }
    const bool ok = mbar_wait(&r.bars[s], static_cast<uint32_t>((j / S) & 1), smem_ok, t.status, ST_TIMEOUT_FLAG, budget);
    if (!__syncthreads_and(ok ? 1 : 0)) break;
    const float4* st = reinterpret_cast<const float4*>(r.data + s * COMM_STAGE_BYTES);
    const int pitch = TB >> 4;
    auto finish = [&](int i, float4 o) {
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int p = 0; p < W; ++p) {
        const float4 v = st[p * pitch + i];
        acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
      }
      o.x += acc.x * t.scale; o.y += acc.y * t.scale; o.z += acc.z * t.scale; o.w += acc.w * t.scale;
      dst[i] = o;
      ss += o.x * o.x + o.y * o.y + o.z * o.z + o.w * o.w;
    };
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int i = threadIdx.x + u * blockDim.x;
      if (i < nvec) finish(i, d[u]);
    }
    for (int i = threadIdx.x + 2 * blockDim.x; i < nvec; i += blockDim.x) finish(i, dst[i]);
    __syncthreads();  // every thread has finished reading stage s
    if (threadIdx.x == 0 && issued < mine) {
      fence_proxy_async();
      issue(issued);
      ++issued;
    }
  }
  if (threadIdx.x == 0 && j < mine) comm_drain(r, j, issued, t.status);
  if (t.sumsq_partials != nullptr) {
    ss = block_sum(ss, red);
    if (threadIdx.x == 0) t.sumsq_partials[cta] += ss;
  }
}

// `smem` / `smem_bytes`: the launch's dynamic shared memory (used by the bulk-async variants only).
__device__ __forceinline__ void comm_run(const CommTask& t, int cta, int nctas, uint8_t* smem, int smem_bytes) {
  __shared__ int smem_ok;
  __shared__ float red[32];
  const bool bulk = (t.mode & COMM_MODE_BULK) != 0 && smem != nullptr;
  if (t.kind == COMM_ALL_GATHER) {
    if (bulk) comm_all_gather_bulk(t, cta, nctas, smem, smem_bytes);
    else comm_all_gather(t, cta, nctas, &smem_ok);
  } else if (t.kind == COMM_REDUCE_SCATTER) {
    if (bulk) comm_reduce_scatter_bulk(t, cta, nctas, smem, smem_bytes, &smem_ok, red);
    else comm_reduce_scatter(t, cta, nctas, &smem_ok, red);
  }
}

}  // namespace ob

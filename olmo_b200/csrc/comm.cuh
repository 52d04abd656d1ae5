// Peer-memory collectives as device functions executed by a *group* of threads, so that the same code runs
//  * as a stand-alone kernel (the group is the whole block),
//  * in dedicated "communication CTAs" of a GEMM launch (the first `comm_ctas` blocks of the grid do not compute), or
//  * in the spare warps of EVERY CTA of a GEMM launch (gemm.cu, gemm2.cu): a GEMM CTA needs six warps (TMA producer,
//    MMA issuer, four epilogue warps); a launch that carries a collective is started with sixteen, and warps 6..15 of
//    each CTA move that CTA's share of the collective while its tensor-core pipeline runs.  No SM is taken away from
//    the GEMM, and all 148 SMs together keep several megabytes of NVLink loads in flight.
//
// All remote accesses are plain 16-byte loads through peer-mapped pointers (NVLink 5 via NVSwitch).  Nothing here uses
// TMA or cluster multicast.  (Untiled bulk-async copies from peer memory into shared memory were measured as an
// alternative and sustained less per CTA than plain loads on this system, so they are not used.)  Waits on a peer's flag
// are bounded (common.cuh) and report through the status word.
#pragma once

#include "common.cuh"

namespace ob {

constexpr int COMM_MAX_WORLD = 8;

enum : int { COMM_NONE = 0, COMM_ALL_GATHER = 1, COMM_REDUCE_SCATTER = 2 };
enum : int { COMM_MODE_SELF = 2, COMM_MODE_STORE = 4 };

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
  float* sumsq_partials;          // reduce-scatter, optional: partial[c] += sum of squares of dst after part c's additions
  int* status;
  long long wait_cycles;          // budget of every flag wait in this task (0: library default)
  int mode;                       // bit 1 (COMM_MODE_SELF): an all-gather also copies this rank's own region;
                                  // bit 2 (COMM_MODE_STORE): a reduce-scatter overwrites dst instead of adding to it
  int reserved;
};

// The threads that execute a task together: `nthr` threads (a multiple of 32) numbered `tid`, synchronising on
// hardware barrier `bar` (barrier 0 belongs to __syncthreads of the whole block).
struct CommGroup {
  int tid;
  int nthr;
  int bar;
};

__device__ __forceinline__ void group_sync(const CommGroup& g) {
  asm volatile("bar.sync %0, %1;" ::"r"(g.bar), "r"(g.nthr) : "memory");
}

// Sum over the group; `scratch` holds 32 floats owned by the group.  Result valid in all threads.
__device__ __forceinline__ float group_sum(float v, float* scratch, const CommGroup& g) {
  const int lane = g.tid & 31, warp = g.tid >> 5, nwarps = g.nthr >> 5;
  v = warp_sum(v);
  group_sync(g);
  if (lane == 0) scratch[warp] = v;
  group_sync(g);
  float r = (lane < nwarps) ? scratch[lane] : 0.f;
  return warp_sum(r);
}

__device__ __forceinline__ uint4 ld_peer_16(const void* p) {
  uint4 v;
  asm volatile("ld.global.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p) : "memory");
  return v;
}

// Every thread of the group calls this; returns false if the wait ran out (the whole group agrees).
__device__ __forceinline__ bool comm_wait_peer(const CommTask& t, int p, int* smem_ok, const CommGroup& g) {
  if (t.wait_flags[p] == nullptr) return true;
  group_sync(g);
  if (g.tid == 0)
    *smem_ok = flag_wait_ge(t.wait_flags[p], t.wait_value, nullptr, t.status,
                            t.wait_cycles > 0 ? t.wait_cycles : OB_WAIT_BUDGET_CYCLES) ? 1 : 0;
  group_sync(g);
  return *smem_ok != 0;
}

// Copy every peer's region (and, with COMM_MODE_SELF, this rank's own) into dst.  This group is part `part` of `nparts`
// that share the task.  16-byte granularity: `elems` must be a multiple of 8 bf16 elements, all bases 16-byte aligned.
__device__ __forceinline__ void comm_all_gather(const CommTask& t, int part, int nparts, int* smem_ok, const CommGroup& g) {
  const long long vecs = t.elems >> 3;  // 16-byte vectors per peer
  constexpr int UNROLL = 8;
  const long long tile = static_cast<long long>(g.nthr) * UNROLL;  // vectors per group iteration
  for (int q = (t.mode & COMM_MODE_SELF) ? 0 : 1; q < t.world; ++q) {
    const int p = (t.rank + q) % t.world;  // start with the next rank so that peers are read evenly
    if (!comm_wait_peer(t, p, smem_ok, g)) return;
    const uint4* src = reinterpret_cast<const uint4*>(t.src[p]);
    uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<bf16*>(t.dst) + static_cast<long long>(p) * t.dst_peer_stride);
    for (long long base = static_cast<long long>(part) * tile; base < vecs; base += static_cast<long long>(nparts) * tile) {
      uint4 v[UNROLL];
#pragma unroll
      for (int u = 0; u < UNROLL; ++u) {
        const long long i = base + static_cast<long long>(u) * g.nthr + g.tid;
        if (i < vecs) v[u] = ld_peer_16(src + i);
      }
#pragma unroll
      for (int u = 0; u < UNROLL; ++u) {
        const long long i = base + static_cast<long long>(u) * g.nthr + g.tid;
        if (i < vecs) dst[i] = v[u];
      }
    }
  }
}

// dst[i] += scale * (src[0][i] + src[1][i] + ... + src[W-1][i]) over my slice, summed in rank order (deterministic).
// `elems` must be a multiple of 4 fp32 elements.  Each thread keeps 8 or more sixteen-byte loads in flight (U vectors
// from each of the W ranks).
template <int W, int U>
struct RsTile {
  uint4 v[W][U];
  float4 d[U];
};

template <int W, int U>
__device__ __forceinline__ void rs_load(const CommTask& t, RsTile<W, U>& r, long long base, long long vecs, const CommGroup& g) {
  const float4* dst = reinterpret_cast<const float4*>(t.dst);
#pragma unroll
  for (int u = 0; u < U; ++u) {
    const long long i = base + static_cast<long long>(u) * g.nthr + g.tid;
    if (i < vecs) {
#pragma unroll
      for (int p = 0; p < W; ++p) r.v[p][u] = ld_peer_16(reinterpret_cast<const uint4*>(t.src[p]) + i);
      r.d[u] = (t.mode & COMM_MODE_STORE) ? make_float4(0.f, 0.f, 0.f, 0.f) : dst[i];
    }
  }
}

template <int W, int U>
__device__ __forceinline__ float rs_finish(const CommTask& t, RsTile<W, U>& r, long long base, long long vecs, const CommGroup& g) {
  float4* dst = reinterpret_cast<float4*>(t.dst);
  float ss = 0.f;
#pragma unroll
  for (int u = 0; u < U; ++u) {
    const long long i = base + static_cast<long long>(u) * g.nthr + g.tid;
    if (i < vecs) {
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int p = 0; p < W; ++p) {
        acc.x += __uint_as_float(r.v[p][u].x);
        acc.y += __uint_as_float(r.v[p][u].y);
        acc.z += __uint_as_float(r.v[p][u].z);
        acc.w += __uint_as_float(r.v[p][u].w);
      }
      float4 d = r.d[u];
      d.x += acc.x * t.scale; d.y += acc.y * t.scale; d.z += acc.z * t.scale; d.w += acc.w * t.scale;
      dst[i] = d;
      ss += d.x * d.x + d.y * d.y + d.z * d.z + d.w * d.w;
    }
  }
  return ss;
}

template <int W, int U>
__device__ __forceinline__ float comm_rs_loop(const CommTask& t, int part, int nparts, const CommGroup& g) {
  const long long vecs = t.elems >> 2;
  const long long tile = static_cast<long long>(g.nthr) * U;
  const long long stride = static_cast<long long>(nparts) * tile;
  float ss = 0.f;
  for (long long base = static_cast<long long>(part) * tile; base < vecs; base += stride) {
    RsTile<W, U> r;
    rs_load<W, U>(t, r, base, vecs, g);
    ss += rs_finish<W, U>(t, r, base, vecs, g);
  }
  return ss;
}

__device__ __forceinline__ void comm_reduce_scatter(const CommTask& t, int part, int nparts, int* smem_ok, float* red,
                                                    const CommGroup& g) {
  for (int p = 0; p < t.world; ++p)
    if (p != t.rank && !comm_wait_peer(t, p, smem_ok, g)) return;
  float ss;
  switch (t.world) {
    case 1: ss = comm_rs_loop<1, 8>(t, part, nparts, g); break;
    case 2: ss = comm_rs_loop<2, 6>(t, part, nparts, g); break;
    case 3: ss = comm_rs_loop<3, 4>(t, part, nparts, g); break;
    case 4: ss = comm_rs_loop<4, 4>(t, part, nparts, g); break;
    case 5: ss = comm_rs_loop<5, 3>(t, part, nparts, g); break;
    case 6: ss = comm_rs_loop<6, 2>(t, part, nparts, g); break;
    case 7: ss = comm_rs_loop<7, 2>(t, part, nparts, g); break;
    default: ss = comm_rs_loop<8, 2>(t, part, nparts, g); break;
  }
  if (t.sumsq_partials != nullptr) {
    ss = group_sum(ss, red, g);
    if (g.tid == 0) t.sumsq_partials[part] += ss;
  }
}

// Shared-memory words a group needs; the caller provides them (static shared memory of the kernel).
struct CommScratch {
  int ok;
  float red[32];
};

__device__ __forceinline__ void comm_run(const CommTask& t, int part, int nparts, CommScratch* scratch, const CommGroup& g) {
  if (t.kind == COMM_ALL_GATHER) comm_all_gather(t, part, nparts, &scratch->ok, g);
  else if (t.kind == COMM_REDUCE_SCATTER) comm_reduce_scatter(t, part, nparts, &scratch->ok, scratch->red, g);
}

// Number of sum-of-squares partial slots a task may touch: one per part, and a launch has at most this many parts.
constexpr int COMM_MAX_PARTS = 256;

}  // namespace ob

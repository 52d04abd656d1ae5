// Peer-memory collectives as device functions, so that the same code runs either as a stand-alone kernel or as the
// "communication CTAs" of a GEMM launch (gemm.cu): the first `comm_ctas` blocks of the grid execute a CommTask while the
// remaining blocks compute tiles, which overlaps NVLink traffic with tensor-core work inside one kernel.
//
// All remote accesses are plain loads through peer-mapped pointers (NVLink 5 via NVSwitch).  Nothing here uses TMA or
// cluster multicast.  Waits on a peer's flag are bounded (common.cuh) and report through the status word.
#pragma once

#include "common.cuh"

namespace ob {

constexpr int COMM_MAX_WORLD = 8;

enum : int { COMM_NONE = 0, COMM_ALL_GATHER = 1, COMM_REDUCE_SCATTER = 2 };

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
  float* sumsq_partials;          // reduce-scatter, optional: partial[c] += sum of squares of what CTA c added
  int* status;
  long long wait_cycles;          // budget of every flag wait in this task (0: library default)
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
  for (int q = 1; q < t.world; ++q) {
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
      ss += acc.x * acc.x + acc.y * acc.y + acc.z * acc.z + acc.w * acc.w;
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

__device__ __forceinline__ void comm_run(const CommTask& t, int cta, int nctas) {
  __shared__ int smem_ok;
  __shared__ float red[32];
  if (t.kind == COMM_ALL_GATHER) comm_all_gather(t, cta, nctas, &smem_ok);
  else if (t.kind == COMM_REDUCE_SCATTER) comm_reduce_scatter(t, cta, nctas, &smem_ok, red);
}

}  // namespace ob

// Causal / full flash-attention forward for head dimension 128 on tcgen05 tensor cores.
//
// One CTA computes a 128-row query tile of one (batch, head) against its key/value tiles of 128 rows:
//   warps 0..7  softmax: thread (row r, half h) owns row r and 64 of the 128 columns of each score tile
//   warp 8      TMA producer (Q once; K and V double buffered; 128B-swizzled tiles of 2 x [128 rows x 64 elements])
//   warp 9      MMA issuer   S = Q Kt (tcgen05, both operands K-major)   and   Ot = P V (V is the MN-major operand)
// TMEM: two score accumulators (2 x 128 columns), so the tensor core works on Q Kt of tile j+1 while the softmax warps
// are busy with tile j, and one output accumulator (128 columns) into which every P V product accumulates.  The
// softmax reference maximum is only raised when a row's maximum grows by more than 2^8; in that (rare) case the warp
// rescales its rows of the output accumulator in TMEM.  This keeps the per-element instruction count of the softmax
// warps low enough (one FFMA, one EX2, one max, one add, half a convert) for the tensor core to be the limiter.
// P is handed to the tensor core through shared memory in the 128B-swizzled K-major layout.
//
// Layout of operands in global memory: (B, T, heads, 128) with arbitrary row pitch (views into fused QKV buffers are
// fine); grouped-query attention maps query head h to key/value head h / (H / Hkv).  T must be a multiple of 128.
// Outputs: O (B, T, H, 128) bf16 and the log-sum-exp (B, H, T) fp32 in natural-log units of the scaled scores.
#include <type_traits>

#include "common.cuh"
#include "api.h"

namespace ob {

int make_tensor_map_bf16_2d(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer, uint64_t ld,
                            uint32_t box_inner, uint32_t box_outer);
int make_tensor_map_f32_2d(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer, uint64_t ld,
                           uint32_t box_inner, uint32_t box_outer);

namespace {

constexpr int AT_THREADS = 320;
constexpr int AT_TILE_BYTES = 128 * 128 * 2;  // 32 KiB: one 128 x 128 bf16 tile = two 64-column halves
constexpr int AT_HALF_BYTES = 128 * 64 * 2;   // 16 KiB
constexpr int AT_SMEM_BWD = 1024 + 7 * AT_TILE_BYTES + 512;  // alignment slack + tiles (Q is double buffered) + barriers
constexpr int AT_SMEM = 1024 + 6 * AT_TILE_BYTES + 4096;  // alignment slack + tiles + barriers and row-statistic exchange (3.3 KiB)

// Two fp32 operations per instruction (packed 64-bit register pairs) and a three-input maximum.
__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void f2_unpack(uint64_t v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ float max3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// exp2 of two values on the FMA pipe (range reduction + cubic), relative error below 1e-4: enough for values that are
// rounded to bf16 next.  Takes work off the special-function unit, which is the busiest pipe of the softmax.
__device__ __forceinline__ void exp2_poly2(uint64_t x2, float& e0, float& e1) {
  float x0, x1;
  f2_unpack(x2, x0, x1);
  x0 = fmaxf(x0, -126.f);
  x1 = fmaxf(x1, -126.f);
  const uint64_t xc = f2_pack(x0, x1);
  const uint64_t magic = f2_pack(12582912.f, 12582912.f), neg_magic = f2_pack(-12582912.f, -12582912.f);
  const uint64_t t = f2_add(xc, magic);                      // low mantissa bits of t = round(x)
  const uint64_t r = f2_fma(f2_add(t, neg_magic), f2_pack(-1.f, -1.f), xc);  // x - round(x), in [-0.5, 0.5]
  uint64_t pl = f2_fma(r, f2_pack(0.055171654f, 0.055171654f), f2_pack(0.24261113f, 0.24261113f));
  pl = f2_fma(pl, r, f2_pack(0.69326097f, 0.69326097f));
  pl = f2_fma(pl, r, f2_pack(0.99992806f, 0.99992806f));
  float p0, p1, t0, t1;
  f2_unpack(pl, p0, p1);
  f2_unpack(t, t0, t1);
  e0 = __uint_as_float(__float_as_uint(p0) + (__float_as_uint(t0) << 23));
  e1 = __uint_as_float(__float_as_uint(p1) + (__float_as_uint(t1) << 23));
}

struct AttnParams {
  bf16* o;
  float* lse;
  int B, T, H, Hkv;
  long long o_stride_b, o_stride_t, o_stride_h;
  float scale_log2;  // softmax scale * log2(e)
  int causal;
  int* status;
  // Optional intra-document masking (implies causal): doc_start[b * T + t] is the position, inside its sequence, of the
  // first token of the document that token t belongs to; query t then attends to keys doc_start .. t only.
  const int* doc_start;
};

__global__ void __launch_bounds__(AT_THREADS, 1)
attn_fwd_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                const __grid_constant__ CUtensorMap tm_v, const AttnParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sK = sQ + AT_TILE_BYTES;       // 2 stages
  uint8_t* sV = sK + 2 * AT_TILE_BYTES;   // 2 stages
  uint8_t* sP = sV + 2 * AT_TILE_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sP + AT_TILE_BYTES);
  uint64_t* q_full = bars;          // 1
  uint64_t* k_full = bars + 1;      // 2
  uint64_t* k_empty = bars + 3;     // 2
  uint64_t* v_full = bars + 5;      // 2
  uint64_t* v_empty = bars + 7;     // 2
  uint64_t* s_full = bars + 9;      // 2
  uint64_t* s_empty = bars + 11;    // 2
  uint64_t* o_full = bars + 13;     // 1
  uint64_t* p_full = bars + 17;     // 1
  uint64_t* x_bar = bars + 18;      // 1: exchange of row statistics between the two column halves
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 19);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* smax = reinterpret_cast<float*>(tmem_slot + 4);  // [2 parities][2 halves][128]
  float* ssum = smax + 512;                               // [2 halves][128]

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int n_qt = p.T / 128;
  // heavy (late) query tiles first so that the tail of the grid is made of short CTAs
  const int qt = n_qt - 1 - static_cast<int>(blockIdx.x) / (p.B * p.H);
  const int bh = static_cast<int>(blockIdx.x) % (p.B * p.H);
  const int b = bh / p.H, h = bh % p.H;
  const int hk = h / (p.H / p.Hkv);
  const int row0 = b * p.T + qt * 128;  // first query row in the flattened (B*T) index space
  // key tiles j_lo .. j_lo + n_kv - 1 are visited; with document masking tiles that end before the document of the
  // tile's first query row starts hold nothing this tile may attend to (doc_start is non-decreasing along a sequence)
  const int j_lo = p.doc_start != nullptr ? p.doc_start[row0] >> 7 : 0;
  const int n_kv = (p.causal ? qt + 1 : n_qt) - j_lo;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
      mbar_init(&s_full[s], 1);
      mbar_init(&s_empty[s], 256);
    }
    mbar_init(o_full, 1);
    mbar_init(p_full, 256);
    mbar_init(x_bar, 256);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 9) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 8) {
    // ------------------------------------------------------------------------- TMA producer
    if (lane == 0) {
      prefetch_tensormap(&tm_q);
      prefetch_tensormap(&tm_k);
      prefetch_tensormap(&tm_v);
      mbar_expect_tx(q_full, AT_TILE_BYTES);
      tma_load_2d(sQ, &tm_q, q_full, h * 128, row0);
      tma_load_2d(sQ + AT_HALF_BYTES, &tm_q, q_full, h * 128 + 64, row0);
      for (int j = 0; j < n_kv; ++j) {
        const int s = j & 1;
        const uint32_t ph = (j >> 1) & 1;
        const int kv_row = b * p.T + (j_lo + j) * 128;
        if (!mbar_wait(&k_empty[s], ph ^ 1u, abort_flag, p.status, ST_TIMEOUT_PRODUCER)) break;
        mbar_expect_tx(&k_full[s], AT_TILE_BYTES);
        tma_load_2d(sK + s * AT_TILE_BYTES, &tm_k, &k_full[s], hk * 128, kv_row);
        tma_load_2d(sK + s * AT_TILE_BYTES + AT_HALF_BYTES, &tm_k, &k_full[s], hk * 128 + 64, kv_row);
        if (!mbar_wait(&v_empty[s], ph ^ 1u, abort_flag, p.status, ST_TIMEOUT_PRODUCER)) break;
        mbar_expect_tx(&v_full[s], AT_TILE_BYTES);
        tma_load_2d(sV + s * AT_TILE_BYTES, &tm_v, &v_full[s], hk * 128, kv_row);
        tma_load_2d(sV + s * AT_TILE_BYTES + AT_HALF_BYTES, &tm_v, &v_full[s], hk * 128 + 64, kv_row);
      }
      if (*abort_flag) {
        const long long t0 = clock64();
        while (clock64() - t0 < 2000000LL) {
        }
      }
    }
  } else if (warp == 9) {
    // --------------------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_qk = make_idesc_bf16(128, 128, 0, 0);
      constexpr uint32_t idesc_pv = make_idesc_bf16(128, 128, 0, 1);
      const uint32_t q_addr = smem_u32(sQ);
      const uint32_t p_addr = smem_u32(sP);
      bool ok = mbar_wait(q_full, 0, abort_flag, p.status, ST_TIMEOUT_MMA);

      auto issue_pv = [&](int i) -> bool {
        const int s = i & 1;
        const uint32_t ph = (i >> 1) & 1;
        if (!mbar_wait(&v_full[s], ph, abort_flag, p.status, ST_TIMEOUT_MMA)) return false;
        if (!mbar_wait(p_full, static_cast<uint32_t>(i & 1), abort_flag, p.status, ST_TIMEOUT_MMA)) return false;
        tc_fence_after();
        const uint32_t v_addr = smem_u32(sV + s * AT_TILE_BYTES);
        const uint32_t d_tmem = tmem_base + 256u;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          // A = P: K-major, 64-column halves;  B = V: MN-major, 16 kv rows per step = 2 KiB, 64-wide d halves 16 KiB apart
          const uint64_t a_desc = make_smem_desc_sw128(p_addr + (k >> 2) * AT_HALF_BYTES + (k & 3) * 32, 16, 1024);
          const uint64_t b_desc = make_smem_desc_sw128(v_addr + k * 2048, AT_HALF_BYTES, 1024);
          umma_f16_ss(d_tmem, a_desc, b_desc, idesc_pv, (i > 0 || k > 0) ? 1u : 0u);
        }
        umma_commit(o_full);
        umma_commit(&v_empty[s]);
        return true;
      };

      for (int j = 0; j < n_kv && ok; ++j) {
        const int s = j & 1;
        const uint32_t ph = (j >> 1) & 1;
        if (!mbar_wait(&k_full[s], ph, abort_flag, p.status, ST_TIMEOUT_MMA)) { ok = false; break; }
        if (!mbar_wait(&s_empty[s], ph ^ 1u, abort_flag, p.status, ST_TIMEOUT_MMA)) { ok = false; break; }
        tc_fence_after();
        const uint32_t k_addr = smem_u32(sK + s * AT_TILE_BYTES);
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(s) * 128u;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const uint64_t a_desc = make_smem_desc_sw128(q_addr + (k >> 2) * AT_HALF_BYTES + (k & 3) * 32, 16, 1024);
          const uint64_t b_desc = make_smem_desc_sw128(k_addr + (k >> 2) * AT_HALF_BYTES + (k & 3) * 32, 16, 1024);
          umma_f16_ss(d_tmem, a_desc, b_desc, idesc_qk, k > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[s]);
        umma_commit(&k_empty[s]);
        if (j > 0) ok = issue_pv(j - 1);
      }
      if (ok) issue_pv(n_kv - 1);
    }
  } else {
    // ------------------------------------------------------------------------------ softmax
    const int quarter = warp & 3;
    const int half = warp >> 2;
    const int row = quarter * 32 + lane;           // query row inside the tile == TMEM lane
    const uint32_t lane_addr = static_cast<uint32_t>(quarter * 32) << 16;
    const int col0 = half * 64;
    const uint32_t o_addr = tmem_base + lane_addr + 256u + static_cast<uint32_t>(col0);
    // reference maximum of the raw (unscaled) scores used in the exponent; a large finite start (not -inf) keeps rows
    // whose first visited tile is entirely masked free of inf - inf
    float m_ref = -1.0e30f;
    float l_run = 0.f;
    bool ok = true;
    const int my_doc_start = p.doc_start != nullptr ? p.doc_start[row0 + row] : 0;

    for (int j = 0; j < n_kv; ++j) {
      const int s = j & 1;
      if (!mbar_wait(&s_full[s], static_cast<uint32_t>((j >> 1) & 1), abort_flag, p.status, ST_TIMEOUT_EPILOGUE)) { ok = false; break; }
      tc_fence_after();
      __syncwarp();
      float sc[64];
      {
        const uint32_t t_addr = tmem_base + lane_addr + static_cast<uint32_t>(s) * 128u + static_cast<uint32_t>(col0);
        uint32_t r0[32], r1[32];
        tmem_ld_32x32b_x32(t_addr, r0);
        tmem_ld_32x32b_x32(t_addr + 32, r1);
        tmem_ld_wait();
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          sc[c] = __uint_as_float(r0[c]);
          sc[32 + c] = __uint_as_float(r1[c]);
        }
      }
      tc_fence_before();
      mbar_arrive(&s_empty[s]);
      if (p.causal && j_lo + j == qt) {
#pragma unroll
        for (int c = 0; c < 64; ++c)
          if (col0 + c > row) sc[c] = -INFINITY;
      }
      if ((j_lo + j) * 128 < my_doc_start) {  // this tile reaches back before the row's document
        const int first = my_doc_start - (j_lo + j) * 128 - col0;  // columns below `first` belong to earlier documents
#pragma unroll
        for (int c = 0; c < 64; ++c)
          if (c < first) sc[c] = -INFINITY;
      }
      float pm0 = fmaxf(sc[0], sc[1]), pm1 = fmaxf(sc[2], sc[3]);
#pragma unroll
      for (int c = 4; c < 64; c += 4) {
        pm0 = max3(pm0, sc[c], sc[c + 1]);
        pm1 = max3(pm1, sc[c + 2], sc[c + 3]);
      }
      float* mx = smax + (j & 1) * 256;
      mx[half * 128 + row] = fmaxf(pm0, pm1);
      mbar_arrive(x_bar);
      if (!mbar_wait(x_bar, static_cast<uint32_t>(j & 1), abort_flag, p.status, ST_TIMEOUT_EPILOGUE)) { ok = false; break; }
      const float m_row = fmaxf(mx[row], mx[128 + row]);
      // raise the reference only when the row maximum outgrows it by more than 2^8 in the exponent's units
      const bool raise = (m_row - m_ref) * p.scale_log2 > 8.0f;
      const float m_new = raise ? m_row : m_ref;
      const float alpha = raise ? exp2f((m_ref - m_new) * p.scale_log2) : 1.0f;
      const float neg_m = -m_new * p.scale_log2;
      uint32_t pk[32];
      const uint64_t scale2 = f2_pack(p.scale_log2, p.scale_log2), neg_m2 = f2_pack(neg_m, neg_m);
      uint64_t lsa = f2_pack(0.f, 0.f), lsb = lsa;
#pragma unroll
      for (int c = 0; c < 32; c += 2) {
        float a0, a1, b0, b1;
        f2_unpack(f2_fma(f2_pack(sc[2 * c], sc[2 * c + 1]), scale2, neg_m2), a0, a1);
        f2_unpack(f2_fma(f2_pack(sc[2 * c + 2], sc[2 * c + 3]), scale2, neg_m2), b0, b1);
        a0 = exp2f(a0); a1 = exp2f(a1);
        if ((c & 2) == 0) exp2_poly2(f2_pack(b0, b1), b0, b1);  // every fourth pair
        else { b0 = exp2f(b0); b1 = exp2f(b1); }
        pk[c] = pack_bf16x2(a0, a1);
        pk[c + 1] = pack_bf16x2(b0, b1);
        lsa = f2_add(lsa, f2_pack(a0, a1));
        lsb = f2_add(lsb, f2_pack(b0, b1));
      }
      float ls0, ls1, ls2, ls3;
      f2_unpack(lsa, ls0, ls1);
      f2_unpack(lsb, ls2, ls3);
      ls0 += ls2;
      ls1 += ls3;
      l_run = l_run * alpha + (ls0 + ls1);
      m_ref = m_new;
      if (j > 0) {
        // P V (j-1) must have completed: it was reading sP, and the accumulator may need rescaling
        if (!mbar_wait(o_full, static_cast<uint32_t>((j - 1) & 1), abort_flag, p.status, ST_TIMEOUT_EPILOGUE)) { ok = false; break; }
        tc_fence_after();
        if (__any_sync(0xffffffffu, raise)) {
#pragma unroll
          for (int cc = 0; cc < 4; ++cc) {
            uint32_t r[16];
            tmem_ld_32x32b_x16(o_addr + cc * 16, r);
            tmem_ld_wait();
#pragma unroll
            for (int c = 0; c < 16; ++c) r[c] = __float_as_uint(__uint_as_float(r[c]) * alpha);
            tmem_st_32x32b_x16(o_addr + cc * 16, r);
          }
          tmem_st_wait();
        }
      }
      // P tile -> shared memory, K-major with 128-byte swizzle: 16-byte chunk index XOR (row mod 8)
      uint8_t* prow = sP + half * AT_HALF_BYTES + (row >> 3) * 1024 + (row & 7) * 128;
#pragma unroll
      for (int ch = 0; ch < 8; ++ch) {
        uint4 v4 = make_uint4(pk[ch * 4 + 0], pk[ch * 4 + 1], pk[ch * 4 + 2], pk[ch * 4 + 3]);
        *reinterpret_cast<uint4*>(prow + ((ch ^ (row & 7)) << 4)) = v4;
      }
      tc_fence_before();
      fence_proxy_async();
      mbar_arrive(p_full);
    }
    if (ok) ok = mbar_wait(o_full, static_cast<uint32_t>((n_kv - 1) & 1), abort_flag, p.status, ST_TIMEOUT_EPILOGUE);
    ssum[half * 128 + row] = l_run;
    if (ok) {
      mbar_arrive(x_bar);
      ok = mbar_wait(x_bar, static_cast<uint32_t>(n_kv & 1), abort_flag, p.status, ST_TIMEOUT_EPILOGUE);
    }
    if (ok) {
      tc_fence_after();
      const float l_tot = ssum[row] + ssum[128 + row];
      const float inv = 1.f / l_tot;
      const long long t_idx = static_cast<long long>(qt) * 128 + row;
      bf16* orow = p.o + b * p.o_stride_b + t_idx * p.o_stride_t + h * p.o_stride_h + col0;
#pragma unroll
      for (int cc = 0; cc < 2; ++cc) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(o_addr + cc * 32, r);
        tmem_ld_wait();
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          uint4 o4;
          o4.x = pack_bf16x2(__uint_as_float(r[v * 8 + 0]) * inv, __uint_as_float(r[v * 8 + 1]) * inv);
          o4.y = pack_bf16x2(__uint_as_float(r[v * 8 + 2]) * inv, __uint_as_float(r[v * 8 + 3]) * inv);
          o4.z = pack_bf16x2(__uint_as_float(r[v * 8 + 4]) * inv, __uint_as_float(r[v * 8 + 5]) * inv);
          o4.w = pack_bf16x2(__uint_as_float(r[v * 8 + 6]) * inv, __uint_as_float(r[v * 8 + 7]) * inv);
          *reinterpret_cast<uint4*>(orow + cc * 32 + v * 8) = o4;
        }
      }
      if (half == 0)
        p.lse[(static_cast<long long>(b) * p.H + h) * p.T + t_idx] = (m_ref * p.scale_log2 + log2f(l_tot)) * 0.6931471805599453f;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
}

}  // namespace
}  // namespace ob

// q, k, v, o: (B, T, heads, 128) bf16 with element strides (batch, token, head); the last dimension is contiguous.
// The token stride is the row pitch; batch stride must equal T * token stride (rows of a batch are contiguous in the
// flattened B*T index space) and head stride must be 128.
extern "C" int ob_attention_fwd(const void* q, const void* k, const void* v, void* o, float* lse, int B, int T, int H, int Hkv,
                                int q_sb, int q_st, int q_sh, int k_sb, int k_st, int k_sh, int v_sb, int v_st, int v_sh,
                                int o_sb, int o_st, int o_sh, float scale, int causal, int* status, const int* doc_start,
                                cudaStream_t stream) {
  using namespace ob;
  if (B <= 0 || T <= 0) return 0;
  if (T % 128 != 0 || H % Hkv != 0) return -1;
  if (doc_start != nullptr && !causal) return -5;  // document masking is defined for causal attention only
  if (q_sh != 128 || k_sh != 128 || v_sh != 128) return -2;
  if (q_sb != T * q_st || k_sb != T * k_st || v_sb != T * v_st) return -3;
  if ((o_st % 8) != 0 || (o_sh % 8) != 0 || (reinterpret_cast<uintptr_t>(o) & 15) != 0) return -4;
  CUtensorMap tq, tk, tv;
  int rc = make_tensor_map_bf16_2d(&tq, q, (uint64_t)H * 128, (uint64_t)B * T, (uint64_t)q_st, 64, 128);
  if (rc != 0) return rc;
  rc = make_tensor_map_bf16_2d(&tk, k, (uint64_t)Hkv * 128, (uint64_t)B * T, (uint64_t)k_st, 64, 128);
  if (rc != 0) return rc;
  rc = make_tensor_map_bf16_2d(&tv, v, (uint64_t)Hkv * 128, (uint64_t)B * T, (uint64_t)v_st, 64, 128);
  if (rc != 0) return rc;
  static bool configured = false;
  if (!configured) {
    if (cudaFuncSetAttribute(attn_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, AT_SMEM) != cudaSuccess) return -10;
    configured = true;
  }
  AttnParams p;
  p.doc_start = doc_start;
  p.o = reinterpret_cast<bf16*>(o);
  p.lse = lse;
  p.B = B; p.T = T; p.H = H; p.Hkv = Hkv;
  p.o_stride_b = o_sb; p.o_stride_t = o_st; p.o_stride_h = o_sh;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.causal = causal;
  p.status = status;
  const int grid = B * H * (T / 128);
  attn_fwd_kernel<<<grid, AT_THREADS, AT_SMEM, stream>>>(tq, tk, tv, p);
  return cudaGetLastError() == cudaSuccess ? 0 : -11;
}

// =====================================================================================================================
// Backward.  One CTA owns a 128-row key/value tile of one (batch, kv head) and walks over the query tiles that attend
// to it (all query heads of the group).  Per query tile:
//     S  = Q Kt,  dP = dO Vt                         (tensor core -> TMEM)
//     P  = exp2(S * c - lse),  dS = P * (dP - delta)      (256 threads, bf16 to shared memory; the softmax scale is
//                                                          applied once, when dK and dQ are written out)
//     dV += Pt dO,  dK += dSt Q,  dQ = dS K          (tensor core; dV and dK accumulate in TMEM over the whole walk)
//     dQ -> fp32 global accumulator with vector reductions (other key tiles add to the same rows)
// `delta` = rowsum(dO * O) comes from a small pre-pass; a post-pass converts the dQ accumulator to bf16.
// The same shared-memory tiles serve as K-major and as MN-major operands (two descriptors over one swizzled tile).
// TMEM columns: [0,128) S then dQ, [128,256) dP, [256,384) dV, [384,512) dK.
// =====================================================================================================================
namespace ob {
namespace {

struct AttnBwdParams {
  const int* doc_start;  // optional intra-document masking, as in the forward kernel
  const float* lse;    // (B, H, T) natural log
  const float* delta;  // (B, H, T)
  float* dq_acc;       // (B, T, H, 128) fp32, zeroed
  bf16* dk;
  bf16* dv;
  long long dk_sb, dk_st, dk_sh, dv_sb, dv_st, dv_sh;
  int B, T, H, Hkv;
  float scale, scale_log2;
  int causal;
  int* status;
};

__device__ __forceinline__ void tmem_ld_32x32b_x8(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr)
               : "memory");
}

// 320 threads are ten warps, i.e. three on some of the four SM sub-partitions with 16,384 registers each, so a launch
// needs at most 170 registers per thread (allocated in steps of 8: 168).  Under that cap the kernel takes 138 registers
// and spills nothing; should a change push the count past the cap the compiler spills rather than failing the launch.
__global__ void __maxnreg__(168)
attn_bwd_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_do,
                const __grid_constant__ CUtensorMap tm_dq, const AttnBwdParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sK = smem;
  uint8_t* sV = sK + AT_TILE_BYTES;
  uint8_t* sQ = sV + AT_TILE_BYTES;
  uint8_t* sdO = sQ + AT_TILE_BYTES;
  uint8_t* sP = sdO + AT_TILE_BYTES;
  uint8_t* sdS = sP + AT_TILE_BYTES;
  uint8_t* sQ1 = sdS + AT_TILE_BYTES;  // second Q buffer: iteration it uses buffer it & 1
  uint64_t* bars = reinterpret_cast<uint64_t*>(sQ1 + AT_TILE_BYTES);
  // Pipeline of one key tile against its query tiles.  Q is double buffered and fetched one iteration ahead; dO is
  // refetched as soon as the dV product of the previous iteration has read it.  dQ is accumulated in the TMEM columns of
  // dP (free once P and dS are written), so S of the next iteration can be issued while the softmax warps still read dQ.
  uint64_t* kv_full = bars;        // K and V landed
  uint64_t* q_full = bars + 1;     // [2] Q of an iteration landed
  uint64_t* q_empty = bars + 3;    // [2] tensor core finished reading that Q buffer (S and dK)
  uint64_t* do_full = bars + 5;    // dO landed
  uint64_t* do_empty = bars + 6;   // tensor core finished reading dO (dP and dV)
  uint64_t* sdp_full = bars + 7;   // S and dP complete
  uint64_t* pds_full = bars + 8;   // P and dS written (256 arrivals)
  uint64_t* dq_full = bars + 9;    // dQ complete (and dV, dK updated)
  uint64_t* dq_read = bars + 10;   // dQ read out of TMEM (256 arrivals)
  // The dQ tile leaves through the P / dS buffers, which are idle between the last MMA of an iteration and the softmax
  // of the next one: column half h stages its columns [0,32) in its 16 KiB half of sP and [32,64) in its half of sdS,
  // i.e. exactly the bytes that the same 128 threads overwrite with P and dS later, so only they need to synchronise.
  uint64_t* stage_full = bars + 11;  // [2] a half's 128 threads have staged their dQ rows
  uint64_t* stage_free = bars + 13;  // [2] the reduce-add stores have finished reading that half's staging bytes
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 15);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int n_t = p.T / 128;
  const int jt = static_cast<int>(blockIdx.x) / (p.B * p.Hkv);  // kv tile; low tiles (most work when causal) first
  const int bh = static_cast<int>(blockIdx.x) % (p.B * p.Hkv);
  const int b = bh / p.Hkv, hk = bh % p.Hkv;
  const int group = p.H / p.Hkv;
  const int i0 = p.causal ? jt : 0;
  int per_head = n_t - i0;
  if (p.doc_start != nullptr) {
    // query tiles whose first row's document starts after this key tile ends cannot attend to it, nor can later ones
    per_head = 0;
    while (i0 + per_head < n_t && p.doc_start[b * p.T + (i0 + per_head) * 128] <= jt * 128 + 127) ++per_head;
  }
  const int n_it = per_head * group;
  const int kv_row = b * p.T + jt * 128;

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    mbar_init(do_full, 1);
    mbar_init(do_empty, 1);
    mbar_init(sdp_full, 1);
    mbar_init(pds_full, 256);
    mbar_init(dq_full, 1);
    mbar_init(dq_read, 256);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
      mbar_init(&stage_full[i], 128);
      mbar_init(&stage_free[i], 1);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 9) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 8) {
    if (lane == 0) {
      prefetch_tensormap(&tm_q);
      prefetch_tensormap(&tm_k);
      prefetch_tensormap(&tm_v);
      prefetch_tensormap(&tm_do);
      prefetch_tensormap(&tm_dq);
      mbar_expect_tx(kv_full, 2 * AT_TILE_BYTES);
      tma_load_2d(sK, &tm_k, kv_full, hk * 128, kv_row);
      tma_load_2d(sK + AT_HALF_BYTES, &tm_k, kv_full, hk * 128 + 64, kv_row);
      tma_load_2d(sV, &tm_v, kv_full, hk * 128, kv_row);
      tma_load_2d(sV + AT_HALF_BYTES, &tm_v, kv_full, hk * 128 + 64, kv_row);
      for (int it = 0; it < n_it; ++it) {
        const int h = hk * group + it / per_head;
        const int qrow = b * p.T + (i0 + it % per_head) * 128;
        const int qb = it & 1;
        uint8_t* q_dst = qb ? sQ1 : sQ;
        if (!mbar_wait(&q_empty[qb], static_cast<uint32_t>(((it >> 1) & 1) ^ 1), abort_flag, p.status, ST_TIMEOUT_PRODUCER)) break;
        mbar_expect_tx(&q_full[qb], AT_TILE_BYTES);
        tma_load_2d(q_dst, &tm_q, &q_full[qb], h * 128, qrow);
        tma_load_2d(q_dst + AT_HALF_BYTES, &tm_q, &q_full[qb], h * 128 + 64, qrow);
        if (!mbar_wait(do_empty, static_cast<uint32_t>((it & 1) ^ 1), abort_flag, p.status, ST_TIMEOUT_PRODUCER)) break;
        mbar_expect_tx(do_full, AT_TILE_BYTES);
        tma_load_2d(sdO, &tm_do, do_full, h * 128, qrow);
        tma_load_2d(sdO + AT_HALF_BYTES, &tm_do, do_full, h * 128 + 64, qrow);
      }
      if (*abort_flag) {
        const long long t0 = clock64();
        while (clock64() - t0 < 2000000LL) {
        }
      }
    }
  } else if (warp == 9) {
    if (lane == 0) {
      constexpr uint32_t idesc_kk = make_idesc_bf16(128, 128, 0, 0);  // A K-major, B K-major
      constexpr uint32_t idesc_km = make_idesc_bf16(128, 128, 0, 1);  // A K-major, B MN-major
      constexpr uint32_t idesc_mm = make_idesc_bf16(128, 128, 1, 1);  // both MN-major
      const uint32_t aK = smem_u32(sK), aV = smem_u32(sV), aO = smem_u32(sdO), aP = smem_u32(sP), aS = smem_u32(sdS);
      const uint32_t aQ0 = smem_u32(sQ), aQ1 = smem_u32(sQ1);
      const uint32_t tS = tmem_base, tdP = tmem_base + 128u, tdV = tmem_base + 256u, tdK = tmem_base + 384u;
      auto issue_s = [&](uint32_t aQ) {  // S = Q Kt
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const uint32_t off = (k >> 2) * AT_HALF_BYTES + (k & 3) * 32;
          umma_f16_ss(tS, make_smem_desc_sw128(aQ + off, 16, 1024), make_smem_desc_sw128(aK + off, 16, 1024), idesc_kk, k > 0 ? 1u : 0u);
        }
      };
      auto issue_dp = [&]() {  // dP = dO Vt
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const uint32_t off = (k >> 2) * AT_HALF_BYTES + (k & 3) * 32;
          umma_f16_ss(tdP, make_smem_desc_sw128(aO + off, 16, 1024), make_smem_desc_sw128(aV + off, 16, 1024), idesc_kk, k > 0 ? 1u : 0u);
        }
      };
      bool ok = mbar_wait(kv_full, 0, abort_flag, p.status, ST_TIMEOUT_MMA);
      if (ok && n_it > 0) {
        ok = mbar_wait(&q_full[0], 0, abort_flag, p.status, ST_TIMEOUT_MMA);
        if (ok) {
          tc_fence_after();
          issue_s(aQ0);
          ok = mbar_wait(do_full, 0, abort_flag, p.status, ST_TIMEOUT_MMA);
        }
        if (ok) {
          tc_fence_after();
          issue_dp();
          umma_commit(sdp_full);
        }
      }
      for (int it = 0; it < n_it && ok; ++it) {
        const uint32_t ph = static_cast<uint32_t>(it & 1);
        const uint32_t aQ = (it & 1) ? aQ1 : aQ0;
        if (!mbar_wait(pds_full, ph, abort_flag, p.status, ST_TIMEOUT_MMA)) break;
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < 8; ++k) {  // dV += Pt dO   (contraction over the 128 query rows, 16 per step)
          umma_f16_ss(tdV, make_smem_desc_sw128(aP + k * 2048, AT_HALF_BYTES, 1024), make_smem_desc_sw128(aO + k * 2048, AT_HALF_BYTES, 1024),
                      idesc_mm, (it > 0 || k > 0) ? 1u : 0u);
        }
        umma_commit(do_empty);  // dO of the next iteration may land while dK and dQ are computed
#pragma unroll
        for (int k = 0; k < 8; ++k) {  // dK += dSt Q
          umma_f16_ss(tdK, make_smem_desc_sw128(aS + k * 2048, AT_HALF_BYTES, 1024), make_smem_desc_sw128(aQ + k * 2048, AT_HALF_BYTES, 1024),
                      idesc_mm, (it > 0 || k > 0) ? 1u : 0u);
        }
#pragma unroll
        for (int k = 0; k < 8; ++k) {  // dQ = dS K    (contraction over the 128 key rows), into the columns dP has vacated
          umma_f16_ss(tdP, make_smem_desc_sw128(aS + (k >> 2) * AT_HALF_BYTES + (k & 3) * 32, 16, 1024),
                      make_smem_desc_sw128(aK + k * 2048, AT_HALF_BYTES, 1024), idesc_km, k > 0 ? 1u : 0u);
        }
        umma_commit(dq_full);
        umma_commit(&q_empty[it & 1]);
        if (it + 1 < n_it) {
          const int nb = (it + 1) & 1;
          if (!mbar_wait(&q_full[nb], static_cast<uint32_t>(((it + 1) >> 1) & 1), abort_flag, p.status, ST_TIMEOUT_MMA)) break;
          tc_fence_after();
          issue_s(nb ? aQ1 : aQ0);  // the softmax warps consumed S of this iteration before they published P and dS
          if (!mbar_wait(do_full, ph ^ 1u, abort_flag, p.status, ST_TIMEOUT_MMA)) break;
          if (!mbar_wait(dq_read, ph, abort_flag, p.status, ST_TIMEOUT_MMA)) break;  // dQ has left the dP columns
          tc_fence_after();
          issue_dp();
          umma_commit(sdp_full);
        }
      }
    }
  } else {
    const int quarter = warp & 3;
    const int half = warp >> 2;
    const int row = quarter * 32 + lane;
    const uint32_t lane_addr = static_cast<uint32_t>(quarter * 32) << 16;
    const int col0 = half * 64;
    bool ok = true;
    // row statistics of the next query tile are fetched one iteration ahead so that their latency is hidden
    auto stat_index = [&](int it_) -> long long {
      const int h_ = hk * group + it_ / per_head;
      const long long t_ = static_cast<long long>(i0 + it_ % per_head) * 128 + row;
      return (static_cast<long long>(b) * p.H + h_) * p.T + t_;
    };
    float lse_next = 0.f, dl_next = 0.f;
    int ds_next = 0;
    auto doc_index = [&](int it_) -> long long { return static_cast<long long>(b) * p.T + (i0 + it_ % per_head) * 128 + row; };
    if (n_it > 0) {
      lse_next = p.lse[stat_index(0)];
      dl_next = p.delta[stat_index(0)];
      if (p.doc_start != nullptr) ds_next = p.doc_start[doc_index(0)];
    }
    for (int it = 0; it < n_it; ++it) {
      const uint32_t ph = static_cast<uint32_t>(it & 1);
      const int h = hk * group + it / per_head;
      const int qi = i0 + it % per_head;
      const float lse2 = lse_next * 1.4426950408889634f;
      const float dl = dl_next;
      const int first_col = ds_next - jt * 128;  // key columns below this index lie before the row's document
      if (it + 1 < n_it) {
        lse_next = p.lse[stat_index(it + 1)];
        dl_next = p.delta[stat_index(it + 1)];
        if (p.doc_start != nullptr) ds_next = p.doc_start[doc_index(it + 1)];
      }
      if (!mbar_wait(sdp_full, ph, abort_flag, p.status, ST_TIMEOUT_EPILOGUE)) { ok = false; break; }
      tc_fence_after();
      __syncwarp();
      // the reduce-add stores of the previous iteration must have read their staging bytes before P / dS overwrite them
      if (it > 0) {
        if (quarter == 0 && lane == 0) {
          bulk_wait_group_read0();
          mbar_arrive(&stage_free[half]);
        }
        if (!mbar_wait(&stage_free[half], static_cast<uint32_t>((it - 1) & 1), abort_flag, p.status, ST_TIMEOUT_EPILOGUE)) { ok = false; break; }
      }
      // P and dS tiles -> shared memory, [query rows][key columns], 128-byte swizzle.  Eight columns (one 16-byte chunk
      // of each tile) at a time; the TMEM loads of the next eight are in flight while the current ones are processed.
      // Tiles that need no masking (all but the diagonal tile and those that reach back before a row's document) take
      // a copy of the loop without the per-element compares.
      uint8_t* prow = sP + half * AT_HALF_BYTES + (row >> 3) * 1024 + (row & 7) * 128;
      uint8_t* srow = sdS + half * AT_HALF_BYTES + (row >> 3) * 1024 + (row & 7) * 128;
      const bool diag = p.causal && qi == jt;
      auto pds_tile = [&](auto masked_tag) {
        constexpr bool MASKED = decltype(masked_tag)::value;
        const uint32_t ts = tmem_base + lane_addr + static_cast<uint32_t>(col0), tp = ts + 128u;
        const uint64_t scale2 = f2_pack(p.scale_log2, p.scale_log2);
        const uint64_t neg_lse2 = f2_pack(-lse2, -lse2);
        const uint64_t neg_dl2 = f2_pack(-dl, -dl);
        uint32_t rs[2][8], rp[2][8];
        tmem_ld_32x32b_x8(ts, rs[0]);
        tmem_ld_32x32b_x8(tp, rp[0]);
#pragma unroll
        for (int cc = 0; cc < 8; ++cc) {
          tmem_ld_wait();
          if (cc + 1 < 8) {
            tmem_ld_32x32b_x8(ts + static_cast<uint32_t>((cc + 1) * 8), rs[(cc + 1) & 1]);
            tmem_ld_32x32b_x8(tp + static_cast<uint32_t>((cc + 1) * 8), rp[(cc + 1) & 1]);
          }
          uint32_t pk[4], dsk[4];
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            const uint64_t s2 = f2_pack(__uint_as_float(rs[cc & 1][2 * c]), __uint_as_float(rs[cc & 1][2 * c + 1]));
            const uint64_t dp2 = f2_pack(__uint_as_float(rp[cc & 1][2 * c]), __uint_as_float(rp[cc & 1][2 * c + 1]));
            float a0, a1;
            f2_unpack(f2_fma(s2, scale2, neg_lse2), a0, a1);
            float p0 = exp2f(a0), p1 = exp2f(a1);
            if (MASKED) {
              const int col = col0 + cc * 8 + 2 * c;
              if ((diag && col > row) || col < first_col) p0 = 0.f;
              if ((diag && col + 1 > row) || col + 1 < first_col) p1 = 0.f;
            }
            float d0, d1;
            f2_unpack(f2_mul(f2_pack(p0, p1), f2_add(dp2, neg_dl2)), d0, d1);
            pk[c] = pack_bf16x2(p0, p1);
            dsk[c] = pack_bf16x2(d0, d1);
          }
          const int o = (cc ^ (row & 7)) << 4;
          *reinterpret_cast<uint4*>(prow + o) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
          *reinterpret_cast<uint4*>(srow + o) = make_uint4(dsk[0], dsk[1], dsk[2], dsk[3]);
        }
      };
      if (diag || __any_sync(0xffffffffu, first_col > col0)) pds_tile(std::true_type{});
      else pds_tile(std::false_type{});
      tc_fence_before();
      fence_proxy_async();
      mbar_arrive(pds_full);
      // dQ tile: add this key tile's contribution to the fp32 accumulator.  The tile leaves through shared memory and
      // a TMA reduce-add store (two rounds of 32 columns per half), which keeps the additions off the load/store units.
      if (!mbar_wait(dq_full, ph, abort_flag, p.status, ST_TIMEOUT_EPILOGUE)) { ok = false; break; }
      tc_fence_after();
      __syncwarp();
      uint32_t r0[32], r1[32];
      tmem_ld_32x32b_x32(tmem_base + lane_addr + 128u + static_cast<uint32_t>(col0), r0);
      tmem_ld_32x32b_x32(tmem_base + lane_addr + 128u + static_cast<uint32_t>(col0 + 32), r1);
      tmem_ld_wait();
      tc_fence_before();
      mbar_arrive(dq_read);  // the columns may be overwritten by the next dP
      uint8_t* stage0 = sP + half * AT_HALF_BYTES;   // fp32 [128 rows][32 columns], 128-byte swizzle: columns col0 .. col0+31
      uint8_t* stage1 = sdS + half * AT_HALF_BYTES;  // columns col0+32 .. col0+63
#pragma unroll
      for (int ch = 0; ch < 8; ++ch) {
        const int o = row * 128 + ((ch ^ (row & 7)) << 4);
        *reinterpret_cast<uint4*>(stage0 + o) = make_uint4(r0[ch * 4 + 0], r0[ch * 4 + 1], r0[ch * 4 + 2], r0[ch * 4 + 3]);
        *reinterpret_cast<uint4*>(stage1 + o) = make_uint4(r1[ch * 4 + 0], r1[ch * 4 + 1], r1[ch * 4 + 2], r1[ch * 4 + 3]);
      }
      fence_proxy_async();
      mbar_arrive(&stage_full[half]);
      if (quarter == 0 && lane == 0) {
        if (!mbar_wait(&stage_full[half], ph, abort_flag, p.status, ST_TIMEOUT_EPILOGUE)) { ok = false; break; }
        tma_reduce_add_2d(&tm_dq, stage0, h * 128 + col0, b * p.T + qi * 128);
        tma_reduce_add_2d(&tm_dq, stage1, h * 128 + col0 + 32, b * p.T + qi * 128);
        bulk_commit_group();
      }
    }
    if (quarter == 0 && lane == 0) bulk_wait_group0();  // every reduce-add of this thread has been performed
    if (ok && n_it > 0) {
      // dV and dK are complete once the last dq_full has fired (same commit covers all earlier MMAs)
      const long long t_idx = static_cast<long long>(jt) * 128 + row;
      bf16* dv_row = p.dv + b * p.dv_sb + t_idx * p.dv_st + hk * p.dv_sh + col0;
      bf16* dk_row = p.dk + b * p.dk_sb + t_idx * p.dk_st + hk * p.dk_sh + col0;
#pragma unroll
      for (int which = 0; which < 2; ++which) {
        bf16* out = which == 0 ? dv_row : dk_row;
        const uint32_t t_addr = tmem_base + lane_addr + (which == 0 ? 256u : 384u) + static_cast<uint32_t>(col0);
#pragma unroll
        for (int cc = 0; cc < 2; ++cc) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(t_addr + cc * 32, r);
          tmem_ld_wait();
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            uint4 o4;
            const float f = which == 0 ? 1.0f : p.scale;  // dS was kept unscaled: dK = scale * dSt Q
            o4.x = pack_bf16x2(__uint_as_float(r[v * 8 + 0]) * f, __uint_as_float(r[v * 8 + 1]) * f);
            o4.y = pack_bf16x2(__uint_as_float(r[v * 8 + 2]) * f, __uint_as_float(r[v * 8 + 3]) * f);
            o4.z = pack_bf16x2(__uint_as_float(r[v * 8 + 4]) * f, __uint_as_float(r[v * 8 + 5]) * f);
            o4.w = pack_bf16x2(__uint_as_float(r[v * 8 + 6]) * f, __uint_as_float(r[v * 8 + 7]) * f);
            *reinterpret_cast<uint4*>(out + cc * 32 + v * 8) = o4;
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
}

// delta[b, h, t] = sum_d dO * O ; one warp per (b, t, h) row of 128 elements
__global__ void attn_bwd_delta_kernel(const bf16* __restrict__ dO, const bf16* __restrict__ O, float* __restrict__ delta, int B, int T,
                                      int H, long long do_sb, long long do_st, long long do_sh, long long o_sb, long long o_st,
                                      long long o_sh) {
  const long long w = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const long long total = static_cast<long long>(B) * T * H;
  if (w >= total) return;
  const int h = static_cast<int>(w % H);
  const long long bt = w / H;
  const int t = static_cast<int>(bt % T);
  const int b = static_cast<int>(bt / T);
  const uint2 a = *reinterpret_cast<const uint2*>(dO + b * do_sb + t * do_st + h * do_sh + lane * 4);
  const uint2 c = *reinterpret_cast<const uint2*>(O + b * o_sb + t * o_st + h * o_sh + lane * 4);
  const float2 a0 = unpack_bf16x2(a.x), a1 = unpack_bf16x2(a.y), c0 = unpack_bf16x2(c.x), c1 = unpack_bf16x2(c.y);
  float s = a0.x * c0.x + a0.y * c0.y + a1.x * c1.x + a1.y * c1.y;
  s = warp_sum(s);
  if (lane == 0) delta[(static_cast<long long>(b) * H + h) * T + t] = s;
}

// dq (bf16, strided) = scale * dq_acc (fp32, contiguous (B, T, H, 128))
__global__ void attn_bwd_dq_convert_kernel(const float* __restrict__ acc, bf16* __restrict__ dq, int B, int T, int H, long long sb,
                                           long long st, long long sh, float scale) {
  const long long v = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;  // one thread per 8 elements
  const long long total = static_cast<long long>(B) * T * H * 16;
  if (v >= total) return;
  const int c = static_cast<int>(v % 16);
  const long long bth = v / 16;
  const int h = static_cast<int>(bth % H);
  const long long bt = bth / H;
  const int t = static_cast<int>(bt % T);
  const int b = static_cast<int>(bt / T);
  const float4 x = *reinterpret_cast<const float4*>(acc + bth * 128 + c * 8);
  const float4 y = *reinterpret_cast<const float4*>(acc + bth * 128 + c * 8 + 4);
  uint4 o;
  o.x = pack_bf16x2(x.x * scale, x.y * scale);
  o.y = pack_bf16x2(x.z * scale, x.w * scale);
  o.z = pack_bf16x2(y.x * scale, y.y * scale);
  o.w = pack_bf16x2(y.z * scale, y.w * scale);
  *reinterpret_cast<uint4*>(dq + b * sb + t * st + h * sh + c * 8) = o;
}

}  // namespace
}  // namespace ob

// Scratch supplied by the caller: `delta` (B*H*T floats) and `dq_acc` (B*T*H*128 floats; zeroed here).
extern "C" int ob_attention_bwd(const void* dout, const void* q, const void* k, const void* v, const void* o, const float* lse,
                                void* dq, void* dk, void* dv, float* delta, float* dq_acc, int B, int T, int H, int Hkv,
                                int do_sb, int do_st, int do_sh, int q_sb, int q_st, int q_sh, int k_sb, int k_st, int k_sh,
                                int v_sb, int v_st, int v_sh, int o_sb, int o_st, int o_sh, int dq_sb, int dq_st, int dq_sh,
                                int dk_sb, int dk_st, int dk_sh, int dv_sb, int dv_st, int dv_sh, float scale, int causal,
                                int* status, const int* doc_start, cudaStream_t stream) {
  using namespace ob;
  if (B <= 0 || T <= 0) return 0;
  if (T % 128 != 0 || H % Hkv != 0) return -1;
  if (doc_start != nullptr && !causal) return -5;
  if (q_sh != 128 || k_sh != 128 || v_sh != 128 || do_sh != 128) return -2;
  if (q_sb != T * q_st || k_sb != T * k_st || v_sb != T * v_st || do_sb != T * do_st) return -3;
  if ((dq_st % 8) || (dk_st % 8) || (dv_st % 8) || (dq_sh % 8) || (dk_sh % 8) || (dv_sh % 8)) return -4;
  CUtensorMap tq, tk, tv, tdo;
  int rc = make_tensor_map_bf16_2d(&tq, q, (uint64_t)H * 128, (uint64_t)B * T, (uint64_t)q_st, 64, 128);
  if (rc == 0) rc = make_tensor_map_bf16_2d(&tk, k, (uint64_t)Hkv * 128, (uint64_t)B * T, (uint64_t)k_st, 64, 128);
  if (rc == 0) rc = make_tensor_map_bf16_2d(&tv, v, (uint64_t)Hkv * 128, (uint64_t)B * T, (uint64_t)v_st, 64, 128);
  if (rc == 0) rc = make_tensor_map_bf16_2d(&tdo, dout, (uint64_t)H * 128, (uint64_t)B * T, (uint64_t)do_st, 64, 128);
  CUtensorMap tdq;
  if (rc == 0) rc = make_tensor_map_f32_2d(&tdq, dq_acc, (uint64_t)H * 128, (uint64_t)B * T, (uint64_t)H * 128, 32, 128);
  if (rc != 0) return rc;
  static bool configured = false;
  if (!configured) {
    if (cudaFuncSetAttribute(attn_bwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, AT_SMEM_BWD) != cudaSuccess) return -10;
    configured = true;
  }
  const long long rows = static_cast<long long>(B) * T * H;
  if (cudaMemsetAsync(dq_acc, 0, static_cast<size_t>(rows) * 128 * sizeof(float), stream) != cudaSuccess) return -12;
  attn_bwd_delta_kernel<<<static_cast<unsigned>((rows * 32 + 255) / 256), 256, 0, stream>>>(
      (const bf16*)dout, (const bf16*)o, delta, B, T, H, do_sb, do_st, do_sh, o_sb, o_st, o_sh);
  AttnBwdParams p;
  p.doc_start = doc_start;
  p.lse = lse; p.delta = delta; p.dq_acc = dq_acc;
  p.dk = (bf16*)dk; p.dv = (bf16*)dv;
  p.dk_sb = dk_sb; p.dk_st = dk_st; p.dk_sh = dk_sh; p.dv_sb = dv_sb; p.dv_st = dv_st; p.dv_sh = dv_sh;
  p.B = B; p.T = T; p.H = H; p.Hkv = Hkv;
  p.scale = scale; p.scale_log2 = scale * 1.4426950408889634f;
  p.causal = causal; p.status = status;
  attn_bwd_kernel<<<B * Hkv * (T / 128), AT_THREADS, AT_SMEM_BWD, stream>>>(tq, tk, tv, tdo, tdq, p);
  attn_bwd_dq_convert_kernel<<<static_cast<unsigned>((rows * 16 + 255) / 256), 256, 0, stream>>>(dq_acc, (bf16*)dq, B, T, H, dq_sb,
                                                                                               dq_st, dq_sh, scale);
  return cudaGetLastError() == cudaSuccess ? 0 : -11;
}

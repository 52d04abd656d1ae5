// CPU reference for 4-bit weight / fp32 activation linear layers: the oracle for the GPU kernels in w4a16.cu and the
// fallback on machines without a GPU.  Same storage layout as the GPU side:
//   qweight [N, K/8] int32 (entry i of a word in bits 4i..4i+3), scales [N, K/G] float, zeros [N, K/G] uint8,
//   optional perm [K] (activation order): column j of the stored matrix multiplies x[:, perm[j]].
// Plain C++17, no intrinsics; rows are processed in parallel with std::thread.
// (Takes the place of the AVX kernel in the reference's vendored AutoGPTQ, autogptq_extension/qigen.)
#include <algorithm>
#include <cstdint>
#include <thread>
#include <vector>

namespace {

inline void dequant_row(const int32_t* qrow, const float* srow, const uint8_t* zrow, int K, int group, float* out) {
  for (int w = 0; w < K / 8; ++w) {
    const uint32_t word = static_cast<uint32_t>(qrow[w]);
    const int g = (w * 8) / group;
    const float s = srow[g], z = static_cast<float>(zrow[g]);
    for (int i = 0; i < 8; ++i) out[w * 8 + i] = (static_cast<float>((word >> (4 * i)) & 0xF) - z) * s;
  }
}

template <typename F>
void parallel_rows(int n, int threads, F fn) {
  threads = std::max(1, std::min(threads, n));
  if (threads == 1) {
    fn(0, n);
    return;
  }
  std::vector<std::thread> pool;
  const int per = (n + threads - 1) / threads;
  for (int t = 0; t < threads; ++t) {
    const int lo = t * per, hi = std::min(n, lo + per);
    if (lo < hi) pool.emplace_back(fn, lo, hi);
  }
  for (auto& th : pool) th.join();
}

}  // namespace

extern "C" {

// out[N, K] (row-major float) = reconstructed weights, in stored (permuted) column order.
int ob_cpu_w4a16_dequant(const int32_t* qweight, const float* scales, const uint8_t* zeros, float* out, int N, int K, int group, int threads) {
  if (K % 8 != 0 || group % 8 != 0 || K % group != 0) return -1;
  const int groups = K / group;
  parallel_rows(N, threads, [&](int lo, int hi) {
    for (int n = lo; n < hi; ++n)
      dequant_row(qweight + static_cast<size_t>(n) * (K / 8), scales + static_cast<size_t>(n) * groups, zeros + static_cast<size_t>(n) * groups, K,
                  group, out + static_cast<size_t>(n) * K);
  });
  return 0;
}

// y[M, N] = x[M, K] · Wᵀ with W reconstructed on the fly; perm may be null.
int ob_cpu_w4a16_matmul(const float* x, const int32_t* qweight, const float* scales, const uint8_t* zeros, const int32_t* perm, float* y, int M,
                        int N, int K, int group, int threads) {
  if (K % 8 != 0 || group % 8 != 0 || K % group != 0) return -1;
  const int groups = K / group;
  std::vector<float> xp;
  const float* xin = x;
  if (perm != nullptr) {
    xp.resize(static_cast<size_t>(M) * K);
    for (int m = 0; m < M; ++m)
      for (int j = 0; j < K; ++j) xp[static_cast<size_t>(m) * K + j] = x[static_cast<size_t>(m) * K + perm[j]];
    xin = xp.data();
  }
  parallel_rows(N, threads, [&](int lo, int hi) {
    std::vector<float> w(K);
    for (int n = lo; n < hi; ++n) {
      dequant_row(qweight + static_cast<size_t>(n) * (K / 8), scales + static_cast<size_t>(n) * groups, zeros + static_cast<size_t>(n) * groups, K,
                  group, w.data());
      for (int m = 0; m < M; ++m) {
        const float* xr = xin + static_cast<size_t>(m) * K;
        double acc = 0.0;
        for (int k = 0; k < K; ++k) acc += static_cast<double>(w[k]) * xr[k];
        y[static_cast<size_t>(m) * N + n] = static_cast<float>(acc);
      }
    }
  });
  return 0;
}

}  // extern "C"

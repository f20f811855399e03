// CPU baseline kernels (TEST INFRASTRUCTURE ONLY: timed by bench.py as the
// reported CPU baseline, never a parity reference and never the product).
//
// fp32 y = gelu_tanh(x w + b) over all host cores: the reference's Family A
// path is f32 in / f32 out (tests/test_family_a.py:52-67) and its CPU GEMM is
// a row-band OpenMP executor; this is a register-blocked restatement of the
// same arithmetic (fp32 fma accumulate, GELU-tanh constants from
// src/fusion_emitter_common.cpp:86-108).
#include "oracle.h"

#include <algorithm>
#include <cmath>
#include <vector>

#ifdef _OPENMP
#include <omp.h>
#endif

namespace {

typedef float v8 __attribute__((vector_size(32)));

inline float gelu_f(float x) {
  return 0.5f * x * (1.0f + std::tanh(0.7978845608f * (x + 0.044715f * x * x * x)));
}

// acc[4 rows][16 cols] += x[4 rows][k0:k1] * w[k0:k1][16 cols]
inline void micro_4x16(const float *x, int64_t ldx, const float *w, int64_t ldw,
                       int64_t k0, int64_t k1, v8 acc[4][2]) {
  for (int64_t h = k0; h < k1; ++h) {
    v8 w0, w1;
    __builtin_memcpy(&w0, w + h * ldw, 32);
    __builtin_memcpy(&w1, w + h * ldw + 8, 32);
    for (int r = 0; r < 4; ++r) {
      const float s = x[r * ldx + h];
      const v8 sv = {s, s, s, s, s, s, s, s};
      acc[r][0] += sv * w0;
      acc[r][1] += sv * w1;
    }
  }
}

}  // namespace

extern "C" void orc_baseline_gemm_bias_gelu_f32_full(const float *x, const float *w,
                                                      const float *b, float *y,
                                                      int64_t m, int64_t k, int64_t n,
                                                      int threads) {
  // Tiles of 4 rows x 256 columns with k blocked by 256 so a w panel stays in
  // L2; every thread owns whole output tiles.
  const int64_t MB = 4, NB = 256, KB = 256;
  const int64_t mt = (m + MB - 1) / MB, nt = (n + NB - 1) / NB;
  if (threads < 1) threads = 1;
#pragma omp parallel for collapse(2) schedule(static) num_threads(threads)
  for (int64_t jt = 0; jt < nt; ++jt)
    for (int64_t it = 0; it < mt; ++it) {
      const int64_t i0 = it * MB, j0 = jt * NB;
      const int64_t rows = std::min(MB, m - i0), cols = std::min(NB, n - j0);
      float out[4][256];
      for (int r = 0; r < 4; ++r)
        for (int c = 0; c < 256; ++c) out[r][c] = 0.0f;
      if (rows == 4 && cols % 16 == 0) {
        for (int64_t c = 0; c < cols; c += 16) {
          v8 acc[4][2] = {};
          for (int64_t kk = 0; kk < k; kk += KB)
            micro_4x16(x + i0 * k, k, w + j0 + c, n, kk, std::min(k, kk + KB), acc);
          for (int r = 0; r < 4; ++r) {
            __builtin_memcpy(&out[r][c], &acc[r][0], 32);
            __builtin_memcpy(&out[r][c + 8], &acc[r][1], 32);
          }
        }
      } else {
        for (int64_t r = 0; r < rows; ++r)
          for (int64_t c = 0; c < cols; ++c) {
            float acc = 0.0f;
            for (int64_t h = 0; h < k; ++h) acc = std::fma(x[(i0 + r) * k + h], w[h * n + j0 + c], acc);
            out[r][c] = acc;
          }
      }
      for (int64_t r = 0; r < rows; ++r)
        for (int64_t c = 0; c < cols; ++c)
          y[(i0 + r) * n + j0 + c] = gelu_f(out[r][c] + b[j0 + c]);
    }
}

extern "C" void orc_baseline_gemm_bias_gelu_f32(const uint16_t *x, const uint16_t *w,
                                                const uint16_t *b, float *y, int64_t m,
                                                int64_t k, int64_t n, int threads) {
  std::vector<float> xf(static_cast<size_t>(m * k)), wf(static_cast<size_t>(k * n)),
      bf(static_cast<size_t>(n));
  orc_bf16_to_f32(x, xf.data(), m * k);
  orc_bf16_to_f32(w, wf.data(), k * n);
  orc_bf16_to_f32(b, bf.data(), n);
  orc_baseline_gemm_bias_gelu_f32_full(xf.data(), wf.data(), bf.data(), y, m, k, n, threads);
}

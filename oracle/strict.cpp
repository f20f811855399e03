// Strict f32 restatement (TEST INFRASTRUCTURE ONLY: the checker, never the
// product). Compiled with -ffp-contract=off and without -ffast-math so that
// every multiply and every add rounds to binary32 on its own, exactly as the
// reference's strict leaf does.
//
// Semantics restated from:
//   compiler/lib/runtime/closed_host_v1.cpp:401-415   (strictGemm: sum = 0.0F;
//       sum = sum + a*b in increasing k)
//   compiler/lib/mlir/MatcoreCpuFusedGemmCandidate.h:19-31 and
//   compiler/lib/mlir/MatcoreCpuFusedGemmCandidate.cpp:114-133 (fused pair:
//       E filled with +0, row panels of min(4,M), panel C = +0 fill then
//       producer matmul, consumer matmul accumulates into E; C is binary32)
//   compiler/tests/generated_cpu_fused_pair/execution_test.cpp:37-40
//       (volatile product / sum restatement used as the test oracle)
#include "oracle.h"

#include <algorithm>
#include <cstring>
#include <vector>

#ifdef _OPENMP
#include <omp.h>
#endif

namespace {

// acc[j] = sum_h a_row[h] * b[h, j] for j in [0, n): each output is reduced in
// increasing h from a +0 seed with a separate binary32 multiply and add. The
// loop order (h outer, j inner) only changes which outputs are in flight at
// once, never the order of any single output's reduction, so the compiler may
// vectorise across j without changing a bit. -ffp-contract=off forbids FMA
// and SSE/AVX arithmetic on x86-64 has no excess precision.
inline void strict_row(const float *a_row, const float *b, float *acc,
                       int64_t k, int64_t n, int64_t ldb) {
  for (int64_t j = 0; j < n; ++j) acc[j] = 0.0F;
  for (int64_t h = 0; h < k; ++h) {
    const float s = a_row[h];
    const float *brow = b + h * ldb;
    for (int64_t j = 0; j < n; ++j) {
      const float product = s * brow[j];
      acc[j] = acc[j] + product;
    }
  }
}

void pair_rows(const float *a, const float *b, const float *d, float *e,
               int64_t r0, int64_t r1, int64_t k, int64_t n, int64_t p,
               std::vector<float> &panel) {
  // Row panels of up to 4 rows, as the bufferized leaf does. The panel is a
  // private binary32 buffer: C is rounded before the consumer GEMM reads it.
  for (int64_t i = r0; i < r1; i += 4) {
    const int64_t rows = std::min<int64_t>(4, r1 - i);
    for (int64_t r = 0; r < rows; ++r)
      strict_row(a + (i + r) * k, b, panel.data() + r * n, k, n, n);
    for (int64_t r = 0; r < rows; ++r)
      strict_row(panel.data() + r * n, d, e + (i + r) * p, n, p, p);
  }
}

}  // namespace

extern "C" {

void orc_strict_gemm_f32(const float *a, const float *b, float *c, int64_t m,
                         int64_t k, int64_t n) {
  for (int64_t i = 0; i < m; ++i) strict_row(a + i * k, b, c + i * n, k, n, n);
}

void orc_strict_fused_pair_f32(const float *a, const float *b, const float *d,
                               float *e, int64_t m, int64_t k, int64_t n,
                               int64_t p) {
  if (m <= 0 || p <= 0) return;
  // E starts as +0 (linalg.fill). With N == 0 the consumer reduction is empty
  // and E stays +0; with K == 0 the producer panel is +0 and the consumer still
  // multiplies it by D, so Inf/NaN in D propagate.
  for (int64_t x = 0; x < m * p; ++x) e[x] = 0.0F;
  if (n <= 0) return;
  std::vector<float> panel(static_cast<size_t>(std::min<int64_t>(4, m) * n));
  pair_rows(a, b, d, e, 0, m, k, n, p, panel);
}

void orc_strict_fused_pair_f32_mt(const float *a, const float *b,
                                  const float *d, float *e, int64_t m,
                                  int64_t k, int64_t n, int64_t p,
                                  int threads) {
  if (m <= 0 || p <= 0) return;
  for (int64_t x = 0; x < m * p; ++x) e[x] = 0.0F;
  if (n <= 0) return;
  if (threads < 1) threads = 1;
  const int64_t panels = (m + 3) / 4;
#pragma omp parallel num_threads(threads)
  {
    std::vector<float> panel(static_cast<size_t>(4 * n));
#pragma omp for schedule(static)
    for (int64_t t = 0; t < panels; ++t) {
      const int64_t r0 = t * 4, r1 = std::min<int64_t>(m, r0 + 4);
      pair_rows(a, b, d, e, r0, r1, k, n, p, panel);
    }
  }
}

}  // extern "C"

// Typed and fp64 restatements (TEST INFRASTRUCTURE ONLY: the checker, never
// the product). Each function cites the reference source it restates.
#include "oracle.h"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <vector>

#ifdef _OPENMP
#include <omp.h>
#endif

namespace {

inline uint32_t bits_of(float x) {
  uint32_t u;
  std::memcpy(&u, &x, 4);
  return u;
}
inline float float_of(uint32_t u) {
  float x;
  std::memcpy(&x, &u, 4);
  return x;
}

// compiler/lib/runtime/cpu_numeric_reference.cpp:134-147: NaN keeps its sign
// and becomes the quiet payload 0x7fc0; everything else rounds to nearest,
// ties to even, on the upper 16 bits (overflow carries into Inf naturally).
inline uint16_t bf16_from(float x) {
  const uint32_t u = bits_of(x);
  if ((u & 0x7fffffffu) > 0x7f800000u)
    return static_cast<uint16_t>(((u >> 16) & 0x8000u) | 0x7fc0u);
  const uint32_t lsb = (u >> 16) & 1u;
  return static_cast<uint16_t>((u + 0x7fffu + lsb) >> 16);
}
inline float bf16_to(uint16_t h) { return float_of(static_cast<uint32_t>(h) << 16); }

inline double gelu_tanh(double x) {
  // src/fusion_emitter_common.cpp:86-108: 0.5*x*(1+tanh(0.7978845608*(x+0.044715*x^3)))
  return 0.5 * x * (1.0 + std::tanh(0.7978845608 * (x + 0.044715 * x * x * x)));
}

inline double activate(double v, int act) {
  switch (act) {
    case ORC_ACT_RELU: return v > 0.0 ? v : 0.0;        // arith.maximumf(v, 0)
    case ORC_ACT_GELU_TANH: return gelu_tanh(v);
    case ORC_ACT_EXP: return std::exp(v);               // math.exp
    case ORC_ACT_SIGMOID: return 1.0 / (1.0 + std::exp(-v));
    case ORC_ACT_TANH: return std::tanh(v);
    default: return v;
  }
}

// ---- OCP 8-bit floating point (OFP8) formats -------------------------------
// E4M3 ("fn"): bias 7, 3 mantissa bits, no infinities, NaN only at S.1111.111,
// largest finite 448. E5M2: bias 15, 2 mantissa bits, IEEE-style Inf/NaN,
// largest finite 57344.
struct Fp8Format {
  int mbits, bias;
  float max_finite;
  uint8_t nan_code;
};
inline Fp8Format fmt_of(int fmt) {
  return fmt == ORC_FP8_E5M2 ? Fp8Format{2, 15, 57344.0f, 0x7f}
                             : Fp8Format{3, 7, 448.0f, 0x7f};
}

uint8_t fp8_encode_one(float x, const Fp8Format &f) {
  const uint32_t u = bits_of(x);
  const uint8_t sign = static_cast<uint8_t>((u >> 24) & 0x80u);
  if (std::isnan(x)) return static_cast<uint8_t>(sign | f.nan_code);
  float a = std::fabs(x);
  if (a == 0.0f) return sign;
  if (a > f.max_finite) a = f.max_finite;  // saturate (Inf included)
  const int emin = 1 - f.bias;
  int e = std::ilogb(a);
  const int eq = std::max(e, emin);
  // The quantum at this binade; dividing by a power of two is exact, and
  // nearbyint rounds to nearest-even under the default rounding mode.
  const float quantum = std::ldexp(1.0f, eq - f.mbits);
  float r = std::nearbyint(a / quantum) * quantum;
  if (r > f.max_finite) r = f.max_finite;
  if (r == 0.0f) return sign;
  e = std::ilogb(r);
  uint32_t expfield, mant;
  if (e < emin) {  // subnormal
    expfield = 0;
    mant = static_cast<uint32_t>(std::ldexp(r, f.mbits - emin));
  } else {
    expfield = static_cast<uint32_t>(e + f.bias);
    mant = static_cast<uint32_t>(std::ldexp(r, f.mbits - e)) - (1u << f.mbits);
  }
  return static_cast<uint8_t>(sign | (expfield << f.mbits) | mant);
}

float fp8_decode_one(uint8_t q, int fmt) {
  const Fp8Format f = fmt_of(fmt);
  const float sign = (q & 0x80) ? -1.0f : 1.0f;
  const uint32_t expfield = (q & 0x7f) >> f.mbits;
  const uint32_t mant = q & ((1u << f.mbits) - 1u);
  if (fmt == ORC_FP8_E5M2 && expfield == 31) {
    if (mant == 0) return sign * INFINITY;
    return NAN;
  }
  if (fmt == ORC_FP8_E4M3 && (q & 0x7f) == 0x7f) return NAN;
  if (expfield == 0) return sign * std::ldexp(static_cast<float>(mant), 1 - f.bias - f.mbits);
  return sign * std::ldexp(1.0f + std::ldexp(static_cast<float>(mant), -f.mbits),
                           static_cast<int>(expfield) - f.bias);
}

}  // namespace

extern "C" {

void orc_bf16_from_f32(const float *x, uint16_t *y, int64_t count) {
  for (int64_t i = 0; i < count; ++i) y[i] = bf16_from(x[i]);
}
void orc_bf16_to_f32(const uint16_t *x, float *y, int64_t count) {
  for (int64_t i = 0; i < count; ++i) y[i] = bf16_to(x[i]);
}

void orc_gemm_bf16_f32_fma(const uint16_t *a, const uint16_t *b, float *c,
                           int64_t m, int64_t k, int64_t n) {
  for (int64_t i = 0; i < m; ++i)
    for (int64_t j = 0; j < n; ++j) {
      float acc = 0.0f;
      for (int64_t h = 0; h < k; ++h)
        acc = std::fmaf(bf16_to(a[i * k + h]), bf16_to(b[h * n + j]), acc);
      c[i * n + j] = acc;
    }
}

void orc_gemm_i8_i32(const int8_t *a, const int8_t *b, int32_t *c, int64_t m,
                     int64_t k, int64_t n) {
  for (int64_t i = 0; i < m; ++i)
    for (int64_t j = 0; j < n; ++j) {
      uint32_t acc = 0;
      for (int64_t h = 0; h < k; ++h)
        acc += static_cast<uint32_t>(static_cast<int32_t>(a[i * k + h]) *
                                     static_cast<int32_t>(b[h * n + j]));
      int32_t out;
      std::memcpy(&out, &acc, 4);
      c[i * n + j] = out;
    }
}

// Quantized int8 matmul with zero points, as the legacy path lowers it
// (src/mlir_engine.cpp:944-958, linalg.quantized_matmul):
// C[i,j] = sum_h (sext(A[i,h]) - za) * (sext(B[h,j]) - zb) in wrapping int32
// arithmetic; the per-tensor zero point, else the kernel's global one. The
// reference's plan test expects exactly (A - zp) @ (B - zp)
// (tests/test_plan_quantization.py:22-25).
void orc_gemm_i8_i32_zp(const int8_t *a, const int8_t *b, int32_t *c, int64_t m, int64_t k,
                        int64_t n, int32_t za, int32_t zb) {
  const uint32_t uza = static_cast<uint32_t>(za), uzb = static_cast<uint32_t>(zb);
  for (int64_t i = 0; i < m; ++i)
    for (int64_t j = 0; j < n; ++j) {
      uint32_t acc = 0;
      for (int64_t h = 0; h < k; ++h) {
        const uint32_t x = static_cast<uint32_t>(static_cast<int32_t>(a[i * k + h])) - uza;
        const uint32_t y = static_cast<uint32_t>(static_cast<int32_t>(b[h * n + j])) - uzb;
        acc += x * y;
      }
      int32_t out;
      std::memcpy(&out, &acc, 4);
      c[i * n + j] = out;
    }
}

void orc_gemm_epilogue_f64(const float *x, const float *w, const float *bias,
                           int bias_mode, int bias_op, int act, double *y,
                           int64_t m, int64_t k, int64_t n,
                           const int64_t *rows, int64_t nrows) {
  const int64_t count = rows ? nrows : m;
#pragma omp parallel for schedule(dynamic, 1)
  for (int64_t t = 0; t < count; ++t) {
    const int64_t i = rows ? rows[t] : t;
    std::vector<double> acc(static_cast<size_t>(n), 0.0);
    for (int64_t h = 0; h < k; ++h) {
      const double s = x[i * k + h];
      const float *wr = w + h * n;
      for (int64_t j = 0; j < n; ++j) acc[j] += s * static_cast<double>(wr[j]);
    }
    for (int64_t j = 0; j < n; ++j) {
      double v = acc[j];
      if (bias_mode != ORC_BIAS_NONE) {
        const double bv = bias_mode == ORC_BIAS_ROW ? bias[j] : bias[i * n + j];
        v = bias_op == ORC_BIAS_RSUB ? bv - v : v + bv;
      }
      y[t * n + j] = activate(v, act);
    }
  }
}

void orc_msm_f64(const float *q, const float *k, const float *v, double *o,
                 int64_t m, int64_t n, int64_t dqk, int64_t dv, double scale) {
#pragma omp parallel for schedule(dynamic, 4)
  for (int64_t i = 0; i < m; ++i) {
    std::vector<double> s(static_cast<size_t>(n));
    double mx = -INFINITY;
    for (int64_t j = 0; j < n; ++j) {
      double acc = 0.0;
      for (int64_t h = 0; h < dqk; ++h)
        acc += static_cast<double>(q[i * dqk + h]) * static_cast<double>(k[j * dqk + h]);
      s[j] = acc * scale;
      mx = std::max(mx, s[j]);
    }
    double l = 0.0;
    for (int64_t j = 0; j < n; ++j) {
      s[j] = std::exp(s[j] - mx);
      l += s[j];
    }
    for (int64_t c = 0; c < dv; ++c) o[i * dv + c] = 0.0;
    for (int64_t j = 0; j < n; ++j) {
      const double pj = s[j] / l;
      for (int64_t c = 0; c < dv; ++c) o[i * dv + c] += pj * static_cast<double>(v[j * dv + c]);
    }
  }
}

void orc_fp8_encode(const float *x, uint8_t *q, int64_t count, int fmt) {
  const Fp8Format f = fmt_of(fmt);
  for (int64_t i = 0; i < count; ++i) q[i] = fp8_encode_one(x[i], f);
}
void orc_fp8_decode(const uint8_t *q, float *x, int64_t count, int fmt) {
  for (int64_t i = 0; i < count; ++i) x[i] = fp8_decode_one(q[i], fmt);
}

void orc_fp8_quantize_blockwise(const float *x, int64_t rows, int64_t cols,
                                int64_t block, int fmt, uint8_t *q,
                                float *scales) {
  const Fp8Format f = fmt_of(fmt);
  const int64_t rb = (rows + block - 1) / block, cb = (cols + block - 1) / block;
#pragma omp parallel for collapse(2) schedule(static)
  for (int64_t bi = 0; bi < rb; ++bi)
    for (int64_t bj = 0; bj < cb; ++bj) {
      const int64_t r0 = bi * block, r1 = std::min(rows, r0 + block);
      const int64_t c0 = bj * block, c1 = std::min(cols, c0 + block);
      float amax = 0.0f;
      for (int64_t r = r0; r < r1; ++r)
        for (int64_t c = c0; c < c1; ++c) amax = std::max(amax, std::fabs(x[r * cols + c]));
      const float s = amax > 0.0f ? amax / f.max_finite : 1.0f;
      scales[bi * cb + bj] = s;
      for (int64_t r = r0; r < r1; ++r)
        for (int64_t c = c0; c < c1; ++c) q[r * cols + c] = fp8_encode_one(x[r * cols + c] / s, f);
    }
}

void orc_gemm_fp8_blockscaled_f64(const uint8_t *a, int a_fmt,
                                  const float *sa, const uint8_t *bt, int b_fmt,
                                  const float *sbt, double *c, int64_t m,
                                  int64_t k, int64_t n, int64_t block,
                                  const int64_t *rows, int64_t nrows) {
  const int64_t kb = (k + block - 1) / block;
  float lut_a[256], lut_b[256];
  for (int i = 0; i < 256; ++i) {
    lut_a[i] = fp8_decode_one(static_cast<uint8_t>(i), a_fmt);
    lut_b[i] = fp8_decode_one(static_cast<uint8_t>(i), b_fmt);
  }
  const int64_t count = rows ? nrows : m;
#pragma omp parallel for schedule(dynamic, 1)
  for (int64_t t = 0; t < count; ++t) {
    const int64_t i = rows ? rows[t] : t;
    std::vector<double> arow(static_cast<size_t>(k));
    for (int64_t h = 0; h < k; ++h)
      arow[h] = static_cast<double>(lut_a[a[i * k + h]]) *
                static_cast<double>(sa[(i / block) * kb + h / block]);
    for (int64_t j = 0; j < n; ++j) {
      double acc = 0.0;
      const uint8_t *brow = bt + j * k;
      const float *srow = sbt + (j / block) * kb;
      for (int64_t h = 0; h < k; ++h)
        acc += arow[h] * static_cast<double>(lut_b[brow[h]]) * static_cast<double>(srow[h / block]);
      c[t * n + j] = acc;
    }
  }
}

int orc_max_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

}  // extern "C"

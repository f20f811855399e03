/*
 * CPU oracle for the MatcoreDSL data-parallel hot path.
 *
 * TEST INFRASTRUCTURE ONLY. This library is the checker that the CUDA path is
 * compared against; it is never linked into, loaded by, or called from the
 * product library (libmcb). Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline / --impl reference legs of bench.py may load it.
 *
 * Every function restates the reference's arithmetic in plain C++ and cites
 * the reference source it follows (paths are relative to the MatcoreDSL
 * repository root).
 *
 * Parity anchors:
 *   - strict f32 GEMM / fused pair: pinned against the known answers of
 *     compiler/examples/experimental/two_gemm.mdsl:24-43 and the discriminator
 *     cases of compiler/tests/generated_cpu_fused_pair/execution_test.cpp:100-135.
 *   - bf16 conversion, bf16 GEMM, int8 GEMM: pinned bit-for-bit against the
 *     reference's own compiler/lib/runtime/cpu_numeric_reference.cpp, compiled
 *     from its source into oracle/_ref by the `ref` target of oracle/Makefile.
 *   - GELU-tanh epilogue and matmul-softmax-matmul: pinned against golden
 *     vectors produced by the reference's own numpy test oracles
 *     (tests/test_family_a.py:63, tests/test_family_c.py:27-37) via
 *     tests/golden/make_golden.py.
 *   - FP8 block-scaled GEMM and the attention-residual block: the reference
 *     has no arithmetic for these (src/lowering_pipeline.cpp:2531-2572 throws;
 *     the block is composed), so they are "parity unpinned" against the
 *     reference and restated from the OCP FP8 format definition and the
 *     BASELINE configuration text.
 */
#ifndef MCB_ORACLE_H
#define MCB_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- strict f32 (bit-exact) --------------------------------------------- */
/* C[m,n] = A[m,k] * B[k,n]; separate multiply then add, increasing k, +0 seed.
 * compiler/lib/runtime/closed_host_v1.cpp:401-415 */
void orc_strict_gemm_f32(const float *a, const float *b, float *c, int64_t m,
                         int64_t k, int64_t n);
/* E[m,p] = (A[m,k]*B[k,n]) * D[n,p] with C rounded to f32 between the GEMMs.
 * compiler/lib/mlir/MatcoreCpuFusedGemmCandidate.h:19-31 and the bufferized
 * leaf in compiler/lib/mlir/MatcoreCpuFusedGemmCandidate.cpp:114-133
 * (row panels of min(4,M); panel order does not change any result bit). */
void orc_strict_fused_pair_f32(const float *a, const float *b, const float *d,
                               float *e, int64_t m, int64_t k, int64_t n,
                               int64_t p);
/* Same arithmetic, rows split over `threads` OpenMP threads (bit-identical). */
void orc_strict_fused_pair_f32_mt(const float *a, const float *b,
                                  const float *d, float *e, int64_t m,
                                  int64_t k, int64_t n, int64_t p,
                                  int threads);

/* ---- bf16 / int8 typed references --------------------------------------- */
/* RNE, NaN -> quiet 0x7fc0 with sign kept.
 * compiler/lib/runtime/cpu_numeric_reference.cpp:134-147 */
void orc_bf16_from_f32(const float *x, uint16_t *y, int64_t count);
void orc_bf16_to_f32(const uint16_t *x, float *y, int64_t count);
/* bf16 x bf16 -> f32, one fma per k in increasing order.
 * compiler/lib/runtime/cpu_numeric_reference.cpp:108-127 */
void orc_gemm_bf16_f32_fma(const uint16_t *a, const uint16_t *b, float *c,
                           int64_t m, int64_t k, int64_t n);
/* i8 x i8 -> i32 modulo 2^32.
 * compiler/lib/runtime/cpu_numeric_reference.cpp:185-209 */
void orc_gemm_i8_i32(const int8_t *a, const int8_t *b, int32_t *c, int64_t m,
                     int64_t k, int64_t n);
/* Quantized i8 x i8 -> i32 with zero points: sum (A - za)(B - zb), wrapping.
 * src/mlir_engine.cpp:944-958 (linalg.quantized_matmul) */
void orc_gemm_i8_i32_zp(const int8_t *a, const int8_t *b, int32_t *c, int64_t m,
                        int64_t k, int64_t n, int32_t za, int32_t zb);

/* ---- Family A: GEMM + epilogue (fp64) ----------------------------------- */
enum {
  ORC_ACT_NONE = 0,
  ORC_ACT_RELU = 1,
  ORC_ACT_GELU_TANH = 2,
  ORC_ACT_EXP = 3,
  ORC_ACT_SIGMOID = 4,
  ORC_ACT_TANH = 5
};
enum { ORC_BIAS_NONE = 0, ORC_BIAS_ROW = 1, ORC_BIAS_FULL = 2 };
enum { ORC_BIAS_ADD = 0, ORC_BIAS_RSUB = 1 };
/* y = act(acc (+|r-) bias) for the listed rows, fp64 throughout, inputs given
 * as f32 (bf16 callers widen first). GELU is the tanh form with 0.5, 0.044715
 * and 0.7978845608 (src/fusion_emitter_common.cpp:86-108); unary kinds follow
 * src/fusion_emitter_common.cpp:51-85. rows==NULL means all m rows. */
void orc_gemm_epilogue_f64(const float *x, const float *w, const float *bias,
                           int bias_mode, int bias_op, int act, double *y,
                           int64_t m, int64_t k, int64_t n,
                           const int64_t *rows, int64_t nrows);

/* ---- Family C: matmul-softmax-matmul (fp64) ----------------------------- */
/* O[m,dv] = softmax(scale * Q[m,dqk] K[n,dqk]^T) V[n,dv]; max-shifted softmax
 * in float64 as in tests/test_family_c.py:27-37. */
void orc_msm_f64(const float *q, const float *k, const float *v, double *o,
                 int64_t m, int64_t n, int64_t dqk, int64_t dv, double scale);

/* ---- FP8 (OCP 8-bit floating point formats) ------------------------------ */
enum { ORC_FP8_E4M3 = 0, ORC_FP8_E5M2 = 1 };
/* Saturating round-to-nearest-even encode (NaN -> NaN pattern). */
void orc_fp8_encode(const float *x, uint8_t *q, int64_t count, int fmt);
void orc_fp8_decode(const uint8_t *q, float *x, int64_t count, int fmt);
/* Per-(block x block) absmax scaling: s = absmax / fmt_max (s = 1 when the
 * block is all zero), q = sat_RNE(x / s) with an f32 division.
 * scales is [ceil(rows/block), ceil(cols/block)] row-major. */
void orc_fp8_quantize_blockwise(const float *x, int64_t rows, int64_t cols,
                                int64_t block, int fmt, uint8_t *q,
                                float *scales);
/* C[r,:] = sum_k (sa*A)[r,k] (sb*B)[k,:] in fp64 for the listed rows. A is
 * [m,k] row-major fp8 codes with scales sa [ceil(m/block), ceil(k/block)];
 * B is supplied K-major, i.e. as Bt [n,k] row-major with scales
 * sbt [ceil(n/block), ceil(k/block)] (the layout FP8 tensor-core GEMMs take). */
void orc_gemm_fp8_blockscaled_f64(const uint8_t *a, int a_fmt,
                                  const float *sa, const uint8_t *bt, int b_fmt,
                                  const float *sbt, double *c, int64_t m,
                                  int64_t k, int64_t n, int64_t block,
                                  const int64_t *rows, int64_t nrows);

/* ---- fast CPU baselines (reported only, never a parity reference) ------- */
/* fp32 OpenMP y = gelu_tanh(x w + b) over rows [0,m); bf16 inputs widened. */
void orc_baseline_gemm_bias_gelu_f32(const uint16_t *x, const uint16_t *w,
                                     const uint16_t *b, float *y, int64_t m,
                                     int64_t k, int64_t n, int threads);

/* Same with f32 inputs already widened (the timed CPU baseline). */
void orc_baseline_gemm_bias_gelu_f32_full(const float *x, const float *w,
                                          const float *b, float *y, int64_t m,
                                          int64_t k, int64_t n, int threads);

int orc_max_threads(void);

#ifdef __cplusplus
}
#endif
#endif

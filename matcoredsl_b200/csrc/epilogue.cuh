// Element-wise epilogue math shared by the GEMM kernels (Family A semantics,
// src/fusion_emitter_common.cpp:51-108): optional bias (row broadcast or full
// boundary, added or reverse-subtracted), then one activation.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "common.cuh"
#include "internal.h"

namespace mcb {

constexpr float kGeluC0 = 0.7978845608f;  // sqrt(2/pi) as written in the reference
constexpr float kGeluC1 = 0.044715f;

// `fast` selects the hardware tanh approximation (used when the result is
// rounded to bf16 anyway); otherwise CUDA's accurate tanhf.
template <bool fast>
__device__ __forceinline__ float apply_act(float v, int act) {
  switch (act) {
    case 1: return fmaxf(v, 0.0f);
    case 2: {
      const float u = kGeluC0 * (v + kGeluC1 * v * v * v);
      const float t = fast ? tanh_fast(u) : tanhf(u);
      return 0.5f * v * (1.0f + t);
    }
    case 3: return fast ? __expf(v) : expf(v);
    case 4: return 1.0f / (1.0f + (fast ? __expf(-v) : expf(-v)));
    case 5: return fast ? tanh_fast(v) : tanhf(v);
    default: return v;
  }
}

__device__ __forceinline__ float load_bias(const Epilogue &e, int64_t row, int64_t col) {
  const int64_t idx = e.bias_mode == 1 ? col : row * e.ld_bias + col;
  if (e.bias_bf16)
    return __bfloat162float(reinterpret_cast<const __nv_bfloat16 *>(e.bias)[idx]);
  if (e.bias_f16) return __half2float(reinterpret_cast<const __half *>(e.bias)[idx]);
  return reinterpret_cast<const float *>(e.bias)[idx];
}

// ---- general epilogue chain (src/fusion_emitter_common.cpp:38-160) ----------
// Unary kinds (MCB_EW_*): 1 relu, 2 exp, 3 log, 4 tanh, 5 sqrt, 6 neg, 7 abs,
// 8 sin, 9 cos, 10 rsqrt, 11 sigmoid, 12 gelu (tanh form); binary: 32 add,
// 33 sub, 34 mul, 35 div, 36 min, 37 max. relu, min and max follow
// arith.maximumf / minimumf: a NaN operand gives NaN, and -0 < +0.
__device__ __forceinline__ float ew_maximum(float a, float b) {
  if (a != a || b != b) return __int_as_float(0x7fc00000);
  if (a == b) return signbit(a) ? b : a;
  return a > b ? a : b;
}
__device__ __forceinline__ float ew_minimum(float a, float b) {
  if (a != a || b != b) return __int_as_float(0x7fc00000);
  if (a == b) return signbit(a) ? a : b;
  return a < b ? a : b;
}
__device__ __forceinline__ float ew_unary(int kind, float v) {
  switch (kind) {
    case 1: return ew_maximum(v, 0.0f);
    case 2: return expf(v);
    case 3: return logf(v);
    case 4: return tanhf(v);
    case 5: return sqrtf(v);
    case 6: return -v;
    case 7: return fabsf(v);
    case 8: return sinf(v);
    case 9: return cosf(v);
    case 10: return rsqrtf(v);
    case 11: return 1.0f / (1.0f + expf(-v));
    case 12: return 0.5f * v * (1.0f + tanhf(kGeluC0 * (v + kGeluC1 * v * v * v)));
    default: return v;
  }
}
__device__ __forceinline__ float ew_binary(int kind, float a, float b) {
  switch (kind) {
    case 32: return a + b;
    case 33: return a - b;
    case 34: return a * b;
    case 35: return a / b;
    case 36: return ew_minimum(a, b);
    case 37: return ew_maximum(a, b);
    default: return a;
  }
}
__device__ __forceinline__ float load_boundary(const Epilogue &e, int b, int64_t row,
                                               int64_t col) {
  const int64_t idx = row * e.ld_bnd[b] + col;
  if (e.bnd_dt[b] == 3)
    return __bfloat162float(reinterpret_cast<const __nv_bfloat16 *>(e.bnd[b])[idx]);
  if (e.bnd_dt[b] == 6) return __half2float(reinterpret_cast<const __half *>(e.bnd[b])[idx]);
  return reinterpret_cast<const float *>(e.bnd[b])[idx];
}
// One element through the chain (row < M and col < N: the caller checks).
__device__ __forceinline__ float apply_chain(const Epilogue &e, float v, int64_t row,
                                             int64_t col) {
#pragma unroll 1
  for (int o = 0; o < e.n_ops; ++o) {
    const int kind = e.op_kind[o];
    if (kind < 32) {
      v = ew_unary(kind, v);
    } else {
      const float bv = load_boundary(e, e.op_bnd[o], row, col);
      v = e.op_pos[o] == 0 ? ew_binary(kind, v, bv) : ew_binary(kind, bv, v);
    }
  }
  return v;
}

// The chain over one row's 32-column chunk v (columns col0.., row < M). The
// switch is taken once per op and every loop over v is fully unrolled, so v
// stays in registers.
template <typename F>
__device__ __forceinline__ void map32(float (&v)[32], F f) {
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = f(v[i]);
}
template <typename F>
__device__ __forceinline__ void zip32(const Epilogue &e, int b, bool value_left, float (&v)[32],
                                      int64_t row, int64_t col0, int64_t n, F f) {
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    if (col0 + i < n) {
      const float bv = load_boundary(e, b, row, col0 + i);
      v[i] = value_left ? f(v[i], bv) : f(bv, v[i]);
    }
  }
}
__device__ __forceinline__ void epilogue_chain_chunk(const Epilogue &e, float (&v)[32], int64_t row,
                                                  int64_t col0, int64_t n) {
#pragma unroll 1
  for (int o = 0; o < e.n_ops; ++o) {
    const int kind = e.op_kind[o];
    const int b = e.op_bnd[o];
    const bool vl = e.op_pos[o] == 0;
    switch (kind) {
      case 1: map32(v, [](float x) { return ew_maximum(x, 0.0f); }); break;
      case 2: map32(v, [](float x) { return expf(x); }); break;
      case 3: map32(v, [](float x) { return logf(x); }); break;
      case 4: map32(v, [](float x) { return tanhf(x); }); break;
      case 5: map32(v, [](float x) { return sqrtf(x); }); break;
      case 6: map32(v, [](float x) { return -x; }); break;
      case 7: map32(v, [](float x) { return fabsf(x); }); break;
      case 8: map32(v, [](float x) { return sinf(x); }); break;
      case 9: map32(v, [](float x) { return cosf(x); }); break;
      case 10: map32(v, [](float x) { return rsqrtf(x); }); break;
      case 11: map32(v, [](float x) { return ew_unary(11, x); }); break;
      case 12: map32(v, [](float x) { return ew_unary(12, x); }); break;
      case 32: zip32(e, b, vl, v, row, col0, n, [](float x, float y) { return x + y; }); break;
      case 33: zip32(e, b, vl, v, row, col0, n, [](float x, float y) { return x - y; }); break;
      case 34: zip32(e, b, vl, v, row, col0, n, [](float x, float y) { return x * y; }); break;
      case 35: zip32(e, b, vl, v, row, col0, n, [](float x, float y) { return x / y; }); break;
      case 36: zip32(e, b, vl, v, row, col0, n, ew_minimum); break;
      case 37: zip32(e, b, vl, v, row, col0, n, ew_maximum); break;
      default: break;
    }
  }
}

template <bool fast>
__device__ __forceinline__ float apply_epilogue(const Epilogue &e, float acc, int64_t row,
                                                int64_t col) {
  if (e.n_ops > 0) return apply_chain(e, acc, row, col);
  float v = acc;
  if (e.bias_mode != 0) {
    const float b = load_bias(e, row, col);
    v = e.bias_op == 1 ? b - v : v + b;
  }
  return apply_act<fast>(v, e.act);
}

}  // namespace mcb

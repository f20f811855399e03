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

template <bool fast>
__device__ __forceinline__ float apply_epilogue(const Epilogue &e, float acc, int64_t row,
                                                int64_t col) {
  float v = acc;
  if (e.bias_mode != 0) {
    const float b = load_bias(e, row, col);
    v = e.bias_op == 1 ? b - v : v + b;
  }
  return apply_act<fast>(v, e.act);
}

}  // namespace mcb

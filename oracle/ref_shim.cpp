// C entry points over the reference's own compiler/lib/runtime/
// cpu_numeric_reference.cpp, compiled from its source where it lies (see
// oracle/Makefile, target `ref`). TEST INFRASTRUCTURE ONLY: used to pin the
// oracle's bf16 conversion and typed GEMMs bit-for-bit against the reference.
#include "cpu_numeric_reference.h"

#include <cstdint>

namespace rt = matcore::mdslc::runtime;

extern "C" {

void ref_bf16_from_f32(const float *x, std::uint16_t *y, std::int64_t count) {
  for (std::int64_t i = 0; i < count; ++i) y[i] = rt::bfloat16_from_float_v1(x[i]).bits;
}

void ref_bf16_to_f32(const std::uint16_t *x, float *y, std::int64_t count) {
  for (std::int64_t i = 0; i < count; ++i) y[i] = rt::bfloat16_to_float_v1(rt::BFloat16V1{x[i]});
}

int ref_gemm_bf16_f32(const std::uint16_t *a, const std::uint16_t *b, float *c,
                      std::int64_t m, std::int64_t k, std::int64_t n) {
  rt::CpuTypedGemmShapeV1 shape;
  shape.m = m;
  shape.n = n;
  shape.k = k;
  return static_cast<int>(rt::cpu_reference_gemm_bf16_storage_f32_v1(shape, a, b, c));
}

int ref_gemm_i8_i32(const std::int8_t *a, const std::int8_t *b, std::int32_t *c,
                    std::int64_t m, std::int64_t k, std::int64_t n) {
  rt::CpuTypedGemmShapeV1 shape;
  shape.m = m;
  shape.n = n;
  shape.k = k;
  return static_cast<int>(rt::cpu_reference_gemm_i8_i32_v1(shape, a, b, c));
}

}  // extern "C"

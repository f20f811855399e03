// Residual add + RMSNorm (unit gain) for the attention-residual block region:
//   y[r, :] = s / sqrt(mean(s^2) + eps),  s = x[r, :] + proj[r, :]
// One CTA of 256 threads per row; each thread keeps its slice of s in
// registers (up to 32 elements, i.e. rows of <= 8192), the sum of squares is
// reduced with warp shuffles and shared memory, then the row is written once.
// HBM-bound: it reads x and proj once and writes y once (3 x rows x cols x 2 B).
#include <cuda_bf16.h>

#include "common.cuh"
#include "internal.h"

namespace mcb {
namespace {

constexpr int THREADS = 256;
constexpr int MAX_PER_THREAD = 32;

__global__ void __launch_bounds__(THREADS) residual_rmsnorm_kernel(
    const __nv_bfloat16 *__restrict__ x, const __nv_bfloat16 *__restrict__ proj,
    __nv_bfloat16 *__restrict__ y, int64_t cols, float eps, int aligned16) {
  __shared__ float red[THREADS / 32];
  const int64_t row = blockIdx.x;
  const __nv_bfloat16 *xr = x + row * cols;
  const __nv_bfloat16 *pr = proj + row * cols;
  __nv_bfloat16 *yr = y + row * cols;
  float s[MAX_PER_THREAD];
  float ss = 0.0f;
  const bool vec = aligned16 && (cols % (8 * THREADS) == 0);
  if (vec) {
    // 8 bf16 (16 bytes) per load, contiguous chunks per thread.
    const int per = static_cast<int>(cols / (8 * THREADS));
#pragma unroll
    for (int v = 0; v < MAX_PER_THREAD / 8; ++v) {
      if (v >= per) break;
      const int64_t off = (static_cast<int64_t>(v) * THREADS + threadIdx.x) * 8;
      const uint4 a = *reinterpret_cast<const uint4 *>(xr + off);
      const uint4 b = *reinterpret_cast<const uint4 *>(pr + off);
      const uint32_t aw[4] = {a.x, a.y, a.z, a.w}, bw[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        const float s0 = __uint_as_float(aw[h] << 16) + __uint_as_float(bw[h] << 16);
        const float s1 = __uint_as_float(aw[h] & 0xffff0000u) + __uint_as_float(bw[h] & 0xffff0000u);
        s[v * 8 + h * 2] = s0;
        s[v * 8 + h * 2 + 1] = s1;
        ss = fmaf(s0, s0, fmaf(s1, s1, ss));
      }
    }
  } else {
    for (int i = 0; i < MAX_PER_THREAD; ++i) {
      const int64_t c = static_cast<int64_t>(i) * THREADS + threadIdx.x;
      if (c >= cols) break;
      const float v = __bfloat162float(xr[c]) + __bfloat162float(pr[c]);
      s[i] = v;
      ss = fmaf(v, v, ss);
    }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.0f;
#pragma unroll
  for (int w = 0; w < THREADS / 32; ++w) tot += red[w];
  const float inv = rsqrtf(tot / static_cast<float>(cols) + eps);
  if (vec) {
    const int per = static_cast<int>(cols / (8 * THREADS));
#pragma unroll
    for (int v = 0; v < MAX_PER_THREAD / 8; ++v) {
      if (v >= per) break;
      const int64_t off = (static_cast<int64_t>(v) * THREADS + threadIdx.x) * 8;
      uint4 o;
      o.x = pack_bf16x2(s[v * 8 + 0] * inv, s[v * 8 + 1] * inv);
      o.y = pack_bf16x2(s[v * 8 + 2] * inv, s[v * 8 + 3] * inv);
      o.z = pack_bf16x2(s[v * 8 + 4] * inv, s[v * 8 + 5] * inv);
      o.w = pack_bf16x2(s[v * 8 + 6] * inv, s[v * 8 + 7] * inv);
      *reinterpret_cast<uint4 *>(yr + off) = o;
    }
  } else {
    for (int i = 0; i < MAX_PER_THREAD; ++i) {
      const int64_t c = static_cast<int64_t>(i) * THREADS + threadIdx.x;
      if (c >= cols) break;
      yr[c] = __float2bfloat16_rn(s[i] * inv);
    }
  }
}

}  // namespace

cudaError_t launch_residual_rmsnorm(const void *x, const void *attn_proj, void *y, int64_t rows,
                                    int64_t cols, float eps, cudaStream_t stream,
                                    LaunchInfo *info) {
  if (rows == 0 || cols == 0) return cudaSuccess;
  if (cols > static_cast<int64_t>(THREADS) * MAX_PER_THREAD) return cudaErrorNotSupported;
  if (rows > 0x7fffffff) return cudaErrorInvalidConfiguration;
  residual_rmsnorm_kernel<<<static_cast<unsigned>(rows), THREADS, 0, stream>>>(
      static_cast<const __nv_bfloat16 *>(x), static_cast<const __nv_bfloat16 *>(attn_proj),
      static_cast<__nv_bfloat16 *>(y), cols, eps,
      ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(attn_proj) |
        reinterpret_cast<uintptr_t>(y)) & 15u) == 0);
  if (info) {
    info->launches += 1;
    info->set_route("attn_block_region");
  }
  return cudaGetLastError();
}

}  // namespace mcb

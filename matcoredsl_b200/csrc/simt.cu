// CUDA-core kernels for the shapes and dtypes the tensor-core kernels do not
// take: f32 Family A GEMM + epilogue (the reference's Family A tests are f32,
// tests/test_family_a.py), odd alignments, and the general rank-2 MSM with
// arbitrary Dqk/Dv (Family C, tests/test_family_c.py). These are still the
// GPU path -- there is no CPU fallback anywhere in the library.
#include <cuda_bf16.h>

#include "common.cuh"
#include "epilogue.cuh"
#include "internal.h"

namespace mcb {
namespace {

__device__ __forceinline__ float load_elem(const void *p, int dtype, int64_t idx) {
  if (dtype == 3) return __bfloat162float(reinterpret_cast<const __nv_bfloat16 *>(p)[idx]);
  return reinterpret_cast<const float *>(p)[idx];
}
__device__ __forceinline__ void store_elem(void *p, int dtype, int64_t idx, float v) {
  if (dtype == 3)
    reinterpret_cast<__nv_bfloat16 *>(p)[idx] = __float2bfloat16_rn(v);
  else
    reinterpret_cast<float *>(p)[idx] = v;
}

// 64x64 output tile per CTA, 256 threads, 4x4 outputs per thread, K in steps
// of 16 staged through shared memory; f32 FMA accumulation.
constexpr int TM = 64, TN = 64, TK = 16;

__global__ void __launch_bounds__(256) gemm_simt_kernel(const void *x, int x_dtype, const void *w,
                                                        int w_dtype, void *y, int y_dtype,
                                                        int64_t m, int64_t n, int64_t k,
                                                        int64_t ld_x, int64_t ld_w, int64_t ld_y,
                                                        int w_transposed, Epilogue epi) {
  __shared__ float xs[TK][TM + 4];
  __shared__ float ws[TK][TN + 4];
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
  const int64_t m0 = static_cast<int64_t>(blockIdx.y) * TM;
  const int64_t n0 = static_cast<int64_t>(blockIdx.x) * TN;
  float acc[4][4] = {};
  for (int64_t k0 = 0; k0 < k; k0 += TK) {
    for (int i = threadIdx.x; i < TM * TK; i += 256) {
      const int r = i / TK, c = i % TK;
      const int64_t gr = m0 + r, gc = k0 + c;
      xs[c][r] = (gr < m && gc < k) ? load_elem(x, x_dtype, gr * ld_x + gc) : 0.0f;
    }
    for (int i = threadIdx.x; i < TN * TK; i += 256) {
      int r, c;  // r: k index, c: n index
      if (w_transposed) {
        c = i / TK;
        r = i % TK;
      } else {
        r = i / TN;
        c = i % TN;
      }
      const int64_t gk = k0 + r, gn = n0 + c;
      float v = 0.0f;
      if (gk < k && gn < n)
        v = load_elem(w, w_dtype, w_transposed ? gn * ld_w + gk : gk * ld_w + gn);
      ws[r][c] = v;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < TK; ++kk) {
      float xv[4], wv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) xv[i] = xs[kk][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) wv[j] = ws[kk][tx * 4 + j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(xv[i], wv[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t row = m0 + ty * 4 + i;
    if (row >= m) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int64_t col = n0 + tx * 4 + j;
      if (col >= n) continue;
      store_elem(y, y_dtype, row * ld_y + col, apply_epilogue<false>(epi, acc[i][j], row, col));
    }
  }
}

// One warp per query row, keys streamed in chunks of 32 (one key per lane for
// the score), online softmax with warp-shuffle max/sum, the output row held
// as Dv/32 accumulators per lane. Dqk, Dv <= 256.
constexpr int MSM_WARPS = 4;
constexpr int MSM_DMAX = 256;

__global__ void __launch_bounds__(MSM_WARPS * 32) msm_simt_kernel(const void *q, const void *k,
                                                                  const void *v, void *o,
                                                                  int dtype, MsmShape s,
                                                                  float scale) {
  __shared__ float qs[MSM_WARPS][MSM_DMAX];
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int64_t bh = blockIdx.y;
  const int64_t b = bh / s.heads, h = bh % s.heads;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * MSM_WARPS + warp;
  if (row >= s.m) return;
  const int64_t qoff = b * s.q_s[0] + h * s.q_s[1] + row * s.q_s[2];
  const int64_t koff = b * s.k_s[0] + h * s.k_s[1];
  const int64_t voff = b * s.v_s[0] + h * s.v_s[1];
  const int64_t ooff = b * s.o_s[0] + h * s.o_s[1] + row * s.o_s[2];
  for (int64_t c = lane; c < s.dqk; c += 32) qs[warp][c] = load_elem(q, dtype, qoff + c);
  __syncwarp();
  float m_run = -INFINITY, l_run = 0.0f;
  float acc[MSM_DMAX / 32];
#pragma unroll
  for (int i = 0; i < MSM_DMAX / 32; ++i) acc[i] = 0.0f;
  for (int64_t j0 = 0; j0 < s.n; j0 += 32) {
    const int64_t j = j0 + lane;
    float sc = -INFINITY;
    if (j < s.n) {
      float d = 0.0f;
      for (int64_t c = 0; c < s.dqk; ++c)
        d = fmaf(qs[warp][c], load_elem(k, dtype, koff + j * s.k_s[2] + c), d);
      sc = d * scale;
    }
    float cmax = sc;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) cmax = fmaxf(cmax, __shfl_xor_sync(0xffffffffu, cmax, off));
    const float m_new = fmaxf(m_run, cmax);
    const float corr = expf(m_run - m_new);  // 0 on the first chunk (m_run = -inf)
    const float pj = (j < s.n) ? expf(sc - m_new) : 0.0f;
    float psum = pj;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) psum += __shfl_xor_sync(0xffffffffu, psum, off);
    l_run = l_run * corr + psum;
#pragma unroll
    for (int i = 0; i < MSM_DMAX / 32; ++i) acc[i] *= corr;
    const int cnt = static_cast<int>(s.n - j0 < 32 ? s.n - j0 : 32);
    for (int t = 0; t < cnt; ++t) {
      const float pt = __shfl_sync(0xffffffffu, pj, t);
      const int64_t vrow = voff + (j0 + t) * s.v_s[2];
#pragma unroll
      for (int i = 0; i < MSM_DMAX / 32; ++i) {
        const int64_t c = lane + i * 32;
        if (c < s.dv) acc[i] = fmaf(pt, load_elem(v, dtype, vrow + c), acc[i]);
      }
    }
    m_run = m_new;
  }
  const float inv = 1.0f / l_run;
#pragma unroll
  for (int i = 0; i < MSM_DMAX / 32; ++i) {
    const int64_t c = lane + i * 32;
    if (c < s.dv) store_elem(o, dtype, ooff + c, acc[i] * inv);
  }
}

}  // namespace

cudaError_t launch_gemm_simt(const void *x, int x_dtype, const void *w, int w_dtype, void *y,
                             int y_dtype, int64_t m, int64_t n, int64_t k, int64_t ld_x,
                             int64_t ld_w, int64_t ld_y, int w_transposed, const Epilogue &epi,
                             cudaStream_t stream, LaunchInfo *info) {
  if (m == 0 || n == 0) return cudaSuccess;
  dim3 grid(static_cast<unsigned>((n + TN - 1) / TN), static_cast<unsigned>((m + TM - 1) / TM));
  if (grid.y > 65535u) return cudaErrorInvalidConfiguration;
  gemm_simt_kernel<<<grid, 256, 0, stream>>>(x, x_dtype, w, w_dtype, y, y_dtype, m, n, k, ld_x,
                                             ld_w, ld_y, w_transposed, epi);
  if (info) {
    info->launches = 1;
    info->tile_m = TM;
    info->tile_n = TN;
    info->tile_k = TK;
    info->ctas = static_cast<int>(grid.x * grid.y);
    info->set_route("simt_f32_gemm_epilogue");
  }
  return cudaGetLastError();
}

cudaError_t launch_msm_simt(const void *q, const void *k, const void *v, void *o, int dtype,
                            const MsmShape &s, float scale, cudaStream_t stream,
                            LaunchInfo *info) {
  if (s.m == 0 || s.dv == 0 || s.batch * s.heads == 0) return cudaSuccess;
  if (s.dqk > MSM_DMAX || s.dv > MSM_DMAX) return cudaErrorInvalidValue;
  dim3 grid(static_cast<unsigned>((s.m + MSM_WARPS - 1) / MSM_WARPS),
            static_cast<unsigned>(s.batch * s.heads));
  if (grid.y > 65535u) return cudaErrorInvalidConfiguration;
  msm_simt_kernel<<<grid, MSM_WARPS * 32, 0, stream>>>(q, k, v, o, dtype, s, scale);
  if (info) {
    info->launches = 1;
    info->tile_m = MSM_WARPS;
    info->tile_n = 32;
    info->ctas = static_cast<int>(grid.x * grid.y);
    info->set_route("simt_online_softmax_msm");
  }
  return cudaGetLastError();
}

}  // namespace mcb

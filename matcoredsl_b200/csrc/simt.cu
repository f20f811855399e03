// CUDA-core kernels for the shapes and dtypes the tensor-core kernels do not
// take: f32 Family A GEMM + epilogue (the reference's Family A tests are f32,
// tests/test_family_a.py), odd alignments, and the general rank-2 MSM with
// arbitrary Dqk/Dv (Family C, tests/test_family_c.py). These are still the
// GPU path -- there is no CPU fallback anywhere in the library.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "common.cuh"
#include "epilogue.cuh"
#include "internal.h"

namespace mcb {
namespace {

__device__ __forceinline__ float load_elem(const void *p, int dtype, int64_t idx) {
  if (dtype == 3) return __bfloat162float(reinterpret_cast<const __nv_bfloat16 *>(p)[idx]);
  if (dtype == 6) return __half2float(reinterpret_cast<const __half *>(p)[idx]);
  return reinterpret_cast<const float *>(p)[idx];
}
__device__ __forceinline__ void store_elem(void *p, int dtype, int64_t idx, float v) {
  if (dtype == 3)
    reinterpret_cast<__nv_bfloat16 *>(p)[idx] = __float2bfloat16_rn(v);
  else if (dtype == 6)
    reinterpret_cast<__half *>(p)[idx] = __float2half_rn(v);
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

// Large f32 GEMM + epilogue (f32 X [M,K], f32 W [K,N], 16-byte aligned rows):
// 256 threads own a 128x128 tile, each thread 8x8 accumulators (rows 4ty..
// and 64+4ty.., columns 4tx.. and 64+4tx..); 16-deep k-slices of X (stored
// transposed, [k][row]) and W ([k][col]) are double-buffered in shared memory
// with the next slice fetched into registers (two 16-byte loads per thread
// per operand) while the current one is consumed; four 16-byte shared loads
// per 64 FMAs. The epilogue (bias, activation, f32 or bf16 store) is the one
// the generic kernel above applies.
constexpr int FBM = 128, FBN = 128, FBK = 16, FPAD = 4;

__global__ void __launch_bounds__(256, 2) gemm_f32_big_kernel(const float *__restrict__ x,
                                                           const float *__restrict__ w, void *y,
                                                           int y_dtype, int64_t m, int64_t n,
                                                           int64_t k, int64_t ld_x, int64_t ld_w,
                                                           int64_t ld_y, Epilogue epi) {
  __shared__ __align__(16) float xs[2][FBK][FBM + FPAD];
  __shared__ __align__(16) float ws[2][FBK][FBN + FPAD];
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const int64_t row0 = static_cast<int64_t>(blockIdx.y) * FBM;
  const int64_t col0 = static_cast<int64_t>(blockIdx.x) * FBN;
  // Staging roles per slice: X rows (tid & 127) at k-quads (tid >> 7) and
  // (tid >> 7) + 2; W k-rows (tid >> 5) and 8 + (tid >> 5) at column quad tid & 31.
  const int xr = tid & 127, xq = (tid >> 7) * 4;
  const int wk = tid >> 5, wc = (tid & 31) * 4;
  float4 rx[2], rw[2];
  auto fetch = [&](int64_t sl) {
    const int64_t h0 = sl * FBK;
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int64_t gr = row0 + xr, gk = h0 + xq + i * 8;
      rx[i] = (gr < m && gk < k) ? *reinterpret_cast<const float4 *>(x + gr * ld_x + gk)
                                 : make_float4(0.f, 0.f, 0.f, 0.f);
      const int64_t wk_g = h0 + wk + i * 8, gc = col0 + wc;
      rw[i] = (wk_g < k && gc < n) ? *reinterpret_cast<const float4 *>(w + wk_g * ld_w + gc)
                                   : make_float4(0.f, 0.f, 0.f, 0.f);
    }
  };
  auto stage = [&](int buf) {
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int kq = xq + i * 8;
      xs[buf][kq][xr] = rx[i].x;
      xs[buf][kq + 1][xr] = rx[i].y;
      xs[buf][kq + 2][xr] = rx[i].z;
      xs[buf][kq + 3][xr] = rx[i].w;
      *reinterpret_cast<float4 *>(&ws[buf][wk + i * 8][wc]) = rw[i];
    }
  };
  float acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.0f;
  const int64_t nslices = (k + FBK - 1) / FBK;
  if (nslices > 0) {
    fetch(0);
    stage(0);
  }
  __syncthreads();
  for (int64_t sl = 0; sl < nslices; ++sl) {
    const int buf = static_cast<int>(sl & 1);
    if (sl + 1 < nslices) fetch(sl + 1);
#pragma unroll
    for (int kk = 0; kk < FBK; ++kk) {
      const float4 a0 = *reinterpret_cast<const float4 *>(&xs[buf][kk][ty * 4]);
      const float4 a1 = *reinterpret_cast<const float4 *>(&xs[buf][kk][64 + ty * 4]);
      const float4 b0 = *reinterpret_cast<const float4 *>(&ws[buf][kk][tx * 4]);
      const float4 b1 = *reinterpret_cast<const float4 *>(&ws[buf][kk][64 + tx * 4]);
      const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
      const float bv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
    }
    if (sl + 1 < nslices) stage(buf ^ 1);
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int64_t row = row0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + (i - 4));
    if (row >= m) continue;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int64_t col = col0 + (j < 4 ? tx * 4 + j : 64 + tx * 4 + (j - 4));
      if (col < n)
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

// Tiled CUDA-core MSM for Dqk = Dv = D in {32, 64, 128}: a 256-thread CTA
// owns 64 query rows of one (batch, head) and walks the keys in tiles of 64.
// Thread (ty, tx) computes the 4 x 4 scores of rows 4ty.. and keys 4tx.. from
// Q^T and K^T staged in shared memory (two 16-byte loads per 16 FMAs), keeps
// the online-softmax state of its 4 rows (the 16 threads of a half warp share
// a row block and combine their max and sum with shuffles), writes its P
// block to shared memory and accumulates O[4 rows][D/16 columns] += P V.
// f32 arithmetic for f32 and bf16 inputs; rows past M and keys past N are
// zero-filled when staged, and scores of keys past N are masked.
constexpr int SQ = 64, SK = 64, SPAD = 4;

template <int D>
constexpr size_t msm_tiled_smem_bytes() {
  return sizeof(float) * (static_cast<size_t>(D) * (SQ + SPAD) + D * (SK + SPAD) +
                          SK * (D + SPAD) + SQ * (SK + SPAD));
}

template <int D>
__global__ void __launch_bounds__(256) msm_simt_tiled_kernel(const void *q, const void *k,
                                                             const void *v, void *o, int dtype,
                                                             MsmShape s, float c2) {
  extern __shared__ float4 smem_f4[];
  float *qt = reinterpret_cast<float *>(smem_f4);  // [D][SQ + SPAD]  Q^T
  float *kt = qt + D * (SQ + SPAD);                // [D][SK + SPAD]  K^T
  float *vs = kt + D * (SK + SPAD);                // [SK][D + SPAD]  V
  float *ps = vs + SK * (D + SPAD);                // [SQ][SK + SPAD] P
  constexpr int DC = D / 16;                       // output columns per thread
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const int64_t bh = blockIdx.y, b = bh / s.heads, h = bh % s.heads;
  const int64_t q0 = static_cast<int64_t>(blockIdx.x) * SQ;
  const int64_t qoff = b * s.q_s[0] + h * s.q_s[1], koff = b * s.k_s[0] + h * s.k_s[1];
  const int64_t voff = b * s.v_s[0] + h * s.v_s[1], ooff = b * s.o_s[0] + h * s.o_s[1];
  for (int i = tid; i < SQ * D; i += 256) {
    const int r = i / D, d = i - r * D;
    const int64_t row = q0 + r;
    qt[d * (SQ + SPAD) + r] = row < s.m ? load_elem(q, dtype, qoff + row * s.q_s[2] + d) : 0.0f;
  }
  float m_r[4], l_r[4], acc[4][DC];
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    m_r[r] = -INFINITY;
    l_r[r] = 0.0f;
#pragma unroll
    for (int cc = 0; cc < DC; ++cc) acc[r][cc] = 0.0f;
  }
  const int64_t ntiles = (s.n + SK - 1) / SK;
  for (int64_t t = 0; t < ntiles; ++t) {
    const int64_t k0 = t * SK;
    __syncthreads();  // every read of the previous tile's K^T, V and P is done
    for (int i = tid; i < SK * D; i += 256) {
      const int key = i / D, d = i - key * D;
      const int64_t j = k0 + key;
      const bool in = j < s.n;
      kt[d * (SK + SPAD) + key] = in ? load_elem(k, dtype, koff + j * s.k_s[2] + d) : 0.0f;
      vs[key * (D + SPAD) + d] = in ? load_elem(v, dtype, voff + j * s.v_s[2] + d) : 0.0f;
    }
    __syncthreads();
    float sc[4][4];
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
      for (int cc = 0; cc < 4; ++cc) sc[r][cc] = 0.0f;
#pragma unroll 8
    for (int d = 0; d < D; ++d) {
      const float4 a = *reinterpret_cast<const float4 *>(&qt[d * (SQ + SPAD) + ty * 4]);
      const float4 kk = *reinterpret_cast<const float4 *>(&kt[d * (SK + SPAD) + tx * 4]);
      const float av[4] = {a.x, a.y, a.z, a.w}, kv[4] = {kk.x, kk.y, kk.z, kk.w};
#pragma unroll
      for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) sc[r][cc] = fmaf(av[r], kv[cc], sc[r][cc]);
    }
    // Online softmax of the 4 rows (log2 domain: c2 = scale * log2(e)).
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      float x[4], mx = -INFINITY;
#pragma unroll
      for (int cc = 0; cc < 4; ++cc) {
        x[cc] = k0 + tx * 4 + cc < s.n ? sc[r][cc] * c2 : -INFINITY;
        mx = fmaxf(mx, x[cc]);
      }
#pragma unroll
      for (int off = 8; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
      const float m_new = fmaxf(m_r[r], mx);
      const float alpha = exp2f(m_r[r] - m_new);  // 0 on the first tile (m_r = -inf)
      float pv[4], sum = 0.0f;
#pragma unroll
      for (int cc = 0; cc < 4; ++cc) {
        pv[cc] = exp2f(x[cc] - m_new);
        sum += pv[cc];
      }
#pragma unroll
      for (int off = 8; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
      l_r[r] = fmaf(l_r[r], alpha, sum);
      m_r[r] = m_new;
#pragma unroll
      for (int cc = 0; cc < DC; ++cc) acc[r][cc] *= alpha;
      *reinterpret_cast<float4 *>(&ps[(ty * 4 + r) * (SK + SPAD) + tx * 4]) =
          make_float4(pv[0], pv[1], pv[2], pv[3]);
    }
    __syncthreads();
#pragma unroll 4
    for (int j = 0; j < SK; ++j) {
      float pr[4];
#pragma unroll
      for (int r = 0; r < 4; ++r) pr[r] = ps[(ty * 4 + r) * (SK + SPAD) + j];
      float vv[DC];
      const float *vrow = &vs[j * (D + SPAD) + tx * DC];
      if constexpr (DC % 4 == 0) {
#pragma unroll
        for (int cc = 0; cc < DC; cc += 4) {
          const float4 t4 = *reinterpret_cast<const float4 *>(vrow + cc);
          vv[cc] = t4.x;
          vv[cc + 1] = t4.y;
          vv[cc + 2] = t4.z;
          vv[cc + 3] = t4.w;
        }
      } else {
#pragma unroll
        for (int cc = 0; cc < DC; ++cc) vv[cc] = vrow[cc];
      }
#pragma unroll
      for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int cc = 0; cc < DC; ++cc) acc[r][cc] = fmaf(pr[r], vv[cc], acc[r][cc]);
    }
  }
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int64_t row = q0 + ty * 4 + r;
    if (row >= s.m) continue;
    const float inv = 1.0f / l_r[r];
#pragma unroll
    for (int cc = 0; cc < DC; ++cc)
      store_elem(o, dtype, ooff + row * s.o_s[2] + tx * DC + cc, acc[r][cc] * inv);
  }
}

template <int D>
cudaError_t launch_msm_tiled(const void *q, const void *k, const void *v, void *o, int dtype,
                             const MsmShape &s, float scale, cudaStream_t stream) {
  constexpr size_t smem = msm_tiled_smem_bytes<D>();
  cudaError_t e = cudaFuncSetAttribute(msm_simt_tiled_kernel<D>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  const dim3 grid(static_cast<unsigned>((s.m + SQ - 1) / SQ), static_cast<unsigned>(s.batch * s.heads));
  msm_simt_tiled_kernel<D><<<grid, 256, smem, stream>>>(q, k, v, o, dtype, s,
                                                        scale * 1.4426950408889634f);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_gemm_simt(const void *x, int x_dtype, const void *w, int w_dtype, void *y,
                             int y_dtype, int64_t m, int64_t n, int64_t k, int64_t ld_x,
                             int64_t ld_w, int64_t ld_y, int w_transposed, const Epilogue &epi,
                             cudaStream_t stream, LaunchInfo *info) {
  if (m == 0 || n == 0) return cudaSuccess;
  // f32 operands with 16-byte aligned rows and at least one wave of 128x128
  // tiles take the large-tile kernel.
  const int64_t big_tiles = ((m + FBM - 1) / FBM) * ((n + FBN - 1) / FBN);
  constexpr int kF32 = 1;  // mcb_dtype code of f32 (bf16 is 3, as load_elem reads them)
  const bool big = x_dtype == kF32 && w_dtype == kF32 && !w_transposed &&
                   k % 4 == 0 && n % 4 == 0 && ld_x % 4 == 0 && ld_w % 4 == 0 &&
                   ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w)) & 15u) == 0 &&
                   big_tiles >= 148 && (m + FBM - 1) / FBM <= 65535;
  if (big) {
    const dim3 grid(static_cast<unsigned>((n + FBN - 1) / FBN), static_cast<unsigned>((m + FBM - 1) / FBM));
    gemm_f32_big_kernel<<<grid, 256, 0, stream>>>(static_cast<const float *>(x),
                                                  static_cast<const float *>(w), y, y_dtype, m, n,
                                                  k, ld_x, ld_w, ld_y, epi);
    if (info) {
      info->launches = 1;
      info->tile_m = FBM;
      info->tile_n = FBN;
      info->tile_k = FBK;
      info->ctas = static_cast<int>(grid.x * grid.y);
      info->set_route("simt_f32_gemm_epilogue");
    }
    return cudaGetLastError();
  }
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
  if (s.n > 0 && s.batch * s.heads <= 65535 && s.dqk == s.dv &&
      (s.dqk == 32 || s.dqk == 64 || s.dqk == 128)) {
    // 64 x 64 score tiles with 4 x 4 per thread.
    const cudaError_t e = s.dqk == 32   ? launch_msm_tiled<32>(q, k, v, o, dtype, s, scale, stream)
                          : s.dqk == 64 ? launch_msm_tiled<64>(q, k, v, o, dtype, s, scale, stream)
                                        : launch_msm_tiled<128>(q, k, v, o, dtype, s, scale, stream);
    if (info) {
      info->launches = 1;
      info->tile_m = SQ;
      info->tile_n = SK;
      info->tile_k = static_cast<int>(s.dqk);
      info->ctas = static_cast<int>(((s.m + SQ - 1) / SQ) * s.batch * s.heads);
      info->set_route("simt_tiled_online_softmax_msm");
    }
    return e;
  }
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


namespace {
// Family B chain on CUDA cores for small problems, with the intermediate
// kept in shared memory in f32 (the reference's Family B intermediate,
// src/fusion_emitter_family_b.cpp:231-383): one CTA per CHAIN_RB rows of A
// computes glue(A B) for its rows into shared memory, then E = C W.
constexpr int CHAIN_RB = 16;
__global__ void __launch_bounds__(256) chain_simt_kernel(const void *a, const void *b,
                                                         const void *w, void *e, int dt,
                                                         int e_dt, int64_t m, int64_t k,
                                                         int64_t n1, int64_t n2, int64_t lda,
                                                         int64_t ldb, int64_t ldw, int64_t lde,
                                                         Epilogue glue) {
  extern __shared__ float c_sm[];  // [CHAIN_RB][n1]
  const int64_t r0 = static_cast<int64_t>(blockIdx.x) * CHAIN_RB;
  const int64_t rows = m - r0 < CHAIN_RB ? m - r0 : CHAIN_RB;
  for (int64_t i = threadIdx.x; i < rows * n1; i += blockDim.x) {
    const int64_t r = i / n1, c = i % n1;
    float acc = 0.0f;
    for (int64_t kk = 0; kk < k; ++kk)
      acc = fmaf(load_elem(a, dt, (r0 + r) * lda + kk), load_elem(b, dt, kk * ldb + c), acc);
    c_sm[r * n1 + c] = apply_epilogue<false>(glue, acc, r0 + r, c);
  }
  __syncthreads();
  for (int64_t i = threadIdx.x; i < rows * n2; i += blockDim.x) {
    const int64_t r = i / n2, c = i % n2;
    float acc = 0.0f;
    for (int64_t j = 0; j < n1; ++j) acc = fmaf(c_sm[r * n1 + j], load_elem(w, dt, j * ldw + c), acc);
    store_elem(e, e_dt, (r0 + r) * lde + c, acc);
  }
}
}  // namespace

cudaError_t launch_chain_simt_small(const void *a, const void *b, const void *w, void *e, int dt,
                                    int e_dt, int64_t m, int64_t k, int64_t n1, int64_t n2,
                                    int64_t lda, int64_t ldb, int64_t ldw, int64_t lde,
                                    const Epilogue &glue, cudaStream_t stream, LaunchInfo *info) {
  if (m == 0 || n2 == 0) return cudaSuccess;
  const size_t smem = static_cast<size_t>(CHAIN_RB) * static_cast<size_t>(n1) * sizeof(float);
  if (n1 <= 0 || smem > 96 * 1024 || glue.n_ops != 0) return cudaErrorNotSupported;
  cudaError_t err = cudaFuncSetAttribute(chain_simt_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
  if (err != cudaSuccess) return err;
  const int64_t blocks = (m + CHAIN_RB - 1) / CHAIN_RB;
  if (blocks > 0x7fffffff) return cudaErrorNotSupported;
  chain_simt_kernel<<<static_cast<unsigned>(blocks), 256, smem, stream>>>(
      a, b, w, e, dt, e_dt, m, k, n1, n2, lda, ldb, ldw, lde, glue);
  if (info) {
    info->launches = 1;
    info->tile_m = CHAIN_RB;
    info->tile_n = static_cast<int>(n2);
    info->ctas = static_cast<int>(blocks);
    info->set_route("simt_chain_fused");
  }
  return cudaGetLastError();
}

}  // namespace mcb

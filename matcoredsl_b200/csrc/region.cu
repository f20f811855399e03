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

// kTwo: the projection is the sum of two bf16 partials (proj + proj2), added
// in that order after x (the head-sharded block's own and received halves).
template <bool kTwo>
__global__ void __launch_bounds__(THREADS) residual_rmsnorm_kernel(
    const __nv_bfloat16 *__restrict__ x, const __nv_bfloat16 *__restrict__ proj,
    const __nv_bfloat16 *__restrict__ proj2, __nv_bfloat16 *__restrict__ y, int64_t cols,
    float eps, int aligned16) {
  __shared__ float red[THREADS / 32];
  const int64_t row = blockIdx.x;
  const __nv_bfloat16 *xr = x + row * cols;
  const __nv_bfloat16 *pr = proj + row * cols;
  const __nv_bfloat16 *qr = kTwo ? proj2 + row * cols : nullptr;
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
      uint4 c = make_uint4(0u, 0u, 0u, 0u);
      if constexpr (kTwo) c = *reinterpret_cast<const uint4 *>(qr + off);
      const uint32_t cw4[4] = {c.x, c.y, c.z, c.w};
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        float s0 = __uint_as_float(aw[h] << 16) + __uint_as_float(bw[h] << 16);
        float s1 = __uint_as_float(aw[h] & 0xffff0000u) + __uint_as_float(bw[h] & 0xffff0000u);
        if constexpr (kTwo) {
          s0 += __uint_as_float(cw4[h] << 16);
          s1 += __uint_as_float(cw4[h] & 0xffff0000u);
        }
        s[v * 8 + h * 2] = s0;
        s[v * 8 + h * 2 + 1] = s1;
        ss = fmaf(s0, s0, fmaf(s1, s1, ss));
      }
    }
  } else {
    for (int i = 0; i < MAX_PER_THREAD; ++i) {
      const int64_t c = static_cast<int64_t>(i) * THREADS + threadIdx.x;
      if (c >= cols) break;
      float v = __bfloat162float(xr[c]) + __bfloat162float(pr[c]);
      if constexpr (kTwo) v += __bfloat162float(qr[c]);
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

// ---- block_attn_res (the reference's region op) -------------------------------------
// Depth attention over packed block history, f32 (src/region_emitter_block_
// attn_res.cpp): for every (b, t) row, sources = blocks[0..block_count) plus
// the partial; score_s = <x_s / rms(x_s), q>; w = softmax_s(score); out =
// sum_s w_s x_s. General kernel (any D, any alignment): one CTA of 128
// threads per row. Pass 1 reads every source
// row once (sum of squares and dot with q per thread, warp-shuffle then
// shared-memory reduction); pass 2 re-reads the rows (L1/L2-resident) for the
// weighted sum. HBM-bound: algorithmic bytes = (S + 1) * B*T*D*4 + D*4.
constexpr int BAR_THREADS = 128;
constexpr int BAR_MAX_SOURCES = 33;

__global__ void __launch_bounds__(BAR_THREADS) block_attn_res_kernel(
    const float *__restrict__ blocks, const float *__restrict__ partial,
    const float *__restrict__ query, float *__restrict__ out, int64_t rows, int64_t d,
    int64_t block_stride, int nsrc, int has_partial, int block_count, float eps, int vec4) {
  __shared__ float red[BAR_THREADS / 32][BAR_MAX_SOURCES][2];
  __shared__ float weight[BAR_MAX_SOURCES];
  const int64_t row = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  auto src = [&](int s) -> const float * {
    return s < block_count ? blocks + s * block_stride + row * d : partial + row * d;
  };
  for (int s = 0; s < nsrc; ++s) {
    const float *x = src(s);
    float ss = 0.0f, dot = 0.0f;
    if (vec4) {
      for (int64_t i = threadIdx.x * 4; i < d; i += BAR_THREADS * 4) {
        const float4 v = *reinterpret_cast<const float4 *>(x + i);
        const float4 q = *reinterpret_cast<const float4 *>(query + i);
        ss = fmaf(v.x, v.x, fmaf(v.y, v.y, fmaf(v.z, v.z, fmaf(v.w, v.w, ss))));
        dot = fmaf(v.x, q.x, fmaf(v.y, q.y, fmaf(v.z, q.z, fmaf(v.w, q.w, dot))));
      }
    } else {
      for (int64_t i = threadIdx.x; i < d; i += BAR_THREADS) {
        ss = fmaf(x[i], x[i], ss);
        dot = fmaf(x[i], query[i], dot);
      }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      ss += __shfl_xor_sync(0xffffffffu, ss, off);
      dot += __shfl_xor_sync(0xffffffffu, dot, off);
    }
    if (lane == 0) {
      red[warp][s][0] = ss;
      red[warp][s][1] = dot;
    }
  }
  __syncthreads();
  if (threadIdx.x < 32) {
    // Softmax over the sources, one lane per source (a 33rd in a second round).
    float score[2] = {-INFINITY, -INFINITY};
    for (int r = 0; r < 2; ++r) {
      const int s = lane + 32 * r;
      if (s < nsrc) {
        float ss = 0.0f, dot = 0.0f;
        for (int w = 0; w < BAR_THREADS / 32; ++w) {
          ss += red[w][s][0];
          dot += red[w][s][1];
        }
        score[r] = dot / sqrtf(ss / static_cast<float>(d) + eps);
      }
    }
    float mx = fmaxf(score[0], score[1]);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
    float e[2], sum = 0.0f;
    for (int r = 0; r < 2; ++r) {
      e[r] = (lane + 32 * r < nsrc) ? expf(score[r] - mx) : 0.0f;
      sum += e[r];
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
    for (int r = 0; r < 2; ++r)
      if (lane + 32 * r < nsrc) weight[lane + 32 * r] = e[r] / sum;
  }
  __syncthreads();
  float *o = out + row * d;
  if (vec4) {
    for (int64_t i = threadIdx.x * 4; i < d; i += BAR_THREADS * 4) {
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int s = 0; s < nsrc; ++s) {
        const float w = weight[s];
        const float4 v = *reinterpret_cast<const float4 *>(src(s) + i);
        acc.x = fmaf(w, v.x, acc.x);
        acc.y = fmaf(w, v.y, acc.y);
        acc.z = fmaf(w, v.z, acc.z);
        acc.w = fmaf(w, v.w, acc.w);
      }
      *reinterpret_cast<float4 *>(o + i) = acc;
    }
  } else {
    for (int64_t i = threadIdx.x; i < d; i += BAR_THREADS) {
      float acc = 0.0f;
      for (int s = 0; s < nsrc; ++s) acc = fmaf(weight[s], src(s)[i], acc);
      o[i] = acc;
    }
  }
  (void)has_partial;
}

// Row-group kernel for D = 32 * VPL4 (16-byte aligned rows): 8 lanes own one
// (b, t) row, so one warp instruction serves 4 rows and a 256-thread CTA 32
// rows. Single pass with an online softmax: every source row is read once
// (each lane VPL4 float4, loads running up to four sources ahead), its sum of squares
// and dot with q are reduced over the 8 lanes with three xor-shuffles, and the
// score is folded into a running max m, running sum l and running weighted sum
// acc (rescaled by exp(m_old - m_new)). HBM sees one read of the sources and
// one write of out. The score uses rsqrtf and the weights __expf (a few ulp,
// far inside the reference's 1e-4 tolerance).
constexpr int BARG_ROWS = 32;  // rows per CTA (8 lanes each)

// Streaming read of one source chunk: read-only path, no L1 allocation, and
// a 256-byte L2 prefetch size, so each DRAM access brings in two 128-byte
// lines of the same source row (the 8 lanes of a row read 512 contiguous
// bytes over four loads). With 17 interleaved source streams this cut the
// [16,8,2048,128] launch from 34.3 to 30.2 us back to back, and from 43.0 to
// 36.9 us right after a 256 MiB write has filled L2 with dirty lines; a cold,
// isolated launch (caches invalidated) is unchanged at 32.2 us.
__device__ __forceinline__ float4 ldg_stream256(const float4 *p) {
  float4 v;
  asm("ld.global.nc.L1::no_allocate.L2::256B.v4.f32 {%0, %1, %2, %3}, [%4];"
      : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
      : "l"(p));
  return v;
}

template <int VPL4>
__global__ void __launch_bounds__(256) block_attn_res_rows_kernel(
    const float *__restrict__ blocks, const float *__restrict__ partial,
    const float *__restrict__ query, float *__restrict__ out, int64_t rows,
    int64_t block_stride, int nsrc, int block_count, float eps) {
  constexpr int D = 32 * VPL4;
  const int lr = threadIdx.x >> 3;        // row within the CTA
  const int gl = threadIdx.x & 7;         // lane within the row group
  const int64_t row = static_cast<int64_t>(blockIdx.x) * BARG_ROWS + lr;
  const bool live = row < rows;
  const int64_t rrow = live ? row : 0;    // dead rows read row 0 and store nothing
  float4 q[VPL4];
#pragma unroll
  for (int j = 0; j < VPL4; ++j) q[j] = *reinterpret_cast<const float4 *>(query + (j * 8 + gl) * 4);
  auto src = [&](int s) -> const float4 * {
    const float *base = s < block_count ? blocks + s * block_stride + rrow * D : partial + rrow * D;
    return reinterpret_cast<const float4 *>(base);
  };
  const float inv_d = 1.0f / static_cast<float>(D);
  // Ring of PF source rows in registers: slot f holds source s0 + f and is
  // refilled with source s0 + f + PF as soon as it has been consumed.
  constexpr int PF = VPL4 <= 4 ? 4 : 2;
  float4 buf[PF][VPL4];
#pragma unroll
  for (int f = 0; f < PF; ++f)
    if (f < nsrc) {
#pragma unroll
      for (int j = 0; j < VPL4; ++j) buf[f][j] = ldg_stream256(src(f) + j * 8 + gl);
    }
  float m = -INFINITY, l = 0.0f;
  float4 acc[VPL4];
#pragma unroll
  for (int j = 0; j < VPL4; ++j) acc[j] = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int s0 = 0; s0 < nsrc; s0 += PF) {
#pragma unroll
    for (int f = 0; f < PF; ++f) {
      const int s = s0 + f;
      if (s < nsrc) {
        float4 v[VPL4];
#pragma unroll
        for (int j = 0; j < VPL4; ++j) v[j] = buf[f][j];
        if (s + PF < nsrc) {
          const float4 *xn = src(s + PF);
#pragma unroll
          for (int j = 0; j < VPL4; ++j) buf[f][j] = ldg_stream256(xn + j * 8 + gl);
        }
        float ss = 0.0f, dot = 0.0f;
#pragma unroll
        for (int j = 0; j < VPL4; ++j) {
          ss = fmaf(v[j].x, v[j].x, fmaf(v[j].y, v[j].y, fmaf(v[j].z, v[j].z, fmaf(v[j].w, v[j].w, ss))));
          dot = fmaf(v[j].x, q[j].x, fmaf(v[j].y, q[j].y, fmaf(v[j].z, q[j].z, fmaf(v[j].w, q[j].w, dot))));
        }
#pragma unroll
        for (int off = 4; off > 0; off >>= 1) {
          ss += __shfl_xor_sync(0xffffffffu, ss, off);
          dot += __shfl_xor_sync(0xffffffffu, dot, off);
        }
        const float sc = dot * rsqrtf(fmaf(ss, inv_d, eps));
        const float m_new = fmaxf(m, sc);
        const float r = __expf(m - m_new);  // 0 for the first source (m = -inf)
        const float p = __expf(sc - m_new);
        l = fmaf(l, r, p);
#pragma unroll
        for (int j = 0; j < VPL4; ++j) {
          acc[j].x = fmaf(p, v[j].x, acc[j].x * r);
          acc[j].y = fmaf(p, v[j].y, acc[j].y * r);
          acc[j].z = fmaf(p, v[j].z, acc[j].z * r);
          acc[j].w = fmaf(p, v[j].w, acc[j].w * r);
        }
        m = m_new;
      }
    }
  }
  if (live) {
    const float inv = 1.0f / l;
    float4 *o = reinterpret_cast<float4 *>(out + row * D);
#pragma unroll
    for (int j = 0; j < VPL4; ++j)
      o[j * 8 + gl] = make_float4(acc[j].x * inv, acc[j].y * inv, acc[j].z * inv, acc[j].w * inv);
  }
}

__global__ void zero_f32_kernel(float *__restrict__ y, int64_t n) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    y[i] = 0.0f;
}

}  // namespace

cudaError_t launch_block_attn_res(const float *blocks, const float *partial, const float *query,
                                  float *out, int64_t rows, int64_t d, int64_t block_stride,
                                  int block_count, int has_partial, float eps, int sms,
                                  cudaStream_t stream, LaunchInfo *info) {
  if (rows == 0 || d == 0) return cudaSuccess;
  const int nsrc = block_count + (has_partial ? 1 : 0);
  if (nsrc > BAR_MAX_SOURCES || rows > 0x7fffffff) return cudaErrorInvalidValue;
  if (info) info->launches = 1;
  if (nsrc == 0) {  // no sources: zeros (the reference returns zeros_like(partial))
    zero_f32_kernel<<<sms * 4, 256, 0, stream>>>(out, rows * d);
    if (info) info->set_route("block_attn_res_zero");
    return cudaGetLastError();
  }
  const bool vec4 = d % 4 == 0 && block_stride % 4 == 0 &&
                    ((reinterpret_cast<uintptr_t>(blocks) | reinterpret_cast<uintptr_t>(partial) |
                      reinterpret_cast<uintptr_t>(query) | reinterpret_cast<uintptr_t>(out)) &
                     15u) == 0;
  const int64_t groups = (rows + BARG_ROWS - 1) / BARG_ROWS;
  if (vec4 && (d == 32 || d == 64 || d == 128 || d == 256) && groups <= 0x7fffffff) {
    const unsigned grid = static_cast<unsigned>(groups);
    switch (d) {
      case 32:
        block_attn_res_rows_kernel<1><<<grid, 256, 0, stream>>>(blocks, partial, query, out, rows,
                                                               block_stride, nsrc, block_count, eps);
        break;
      case 64:
        block_attn_res_rows_kernel<2><<<grid, 256, 0, stream>>>(blocks, partial, query, out, rows,
                                                               block_stride, nsrc, block_count, eps);
        break;
      case 128:
        block_attn_res_rows_kernel<4><<<grid, 256, 0, stream>>>(blocks, partial, query, out, rows,
                                                               block_stride, nsrc, block_count, eps);
        break;
      default:
        block_attn_res_rows_kernel<8><<<grid, 256, 0, stream>>>(blocks, partial, query, out, rows,
                                                               block_stride, nsrc, block_count, eps);
        break;
    }
    if (info) {
      info->tile_m = BARG_ROWS;
      info->tile_n = static_cast<int>(d);
      info->ctas = static_cast<int>(grid);
      info->set_route("block_attn_res");
    }
    return cudaGetLastError();
  }
  block_attn_res_kernel<<<static_cast<unsigned>(rows), BAR_THREADS, 0, stream>>>(
      blocks, partial, query, out, rows, d, block_stride, nsrc, has_partial, block_count, eps,
      vec4 ? 1 : 0);
  if (info) {
    info->tile_m = 1;
    info->tile_n = BAR_THREADS;
    info->ctas = static_cast<int>(rows);
    info->set_route("block_attn_res");
  }
  return cudaGetLastError();
}

cudaError_t launch_residual_rmsnorm(const void *x, const void *attn_proj, void *y, int64_t rows,
                                    int64_t cols, float eps, cudaStream_t stream,
                                    LaunchInfo *info, const void *attn_proj2) {
  if (rows == 0 || cols == 0) return cudaSuccess;
  if (cols > static_cast<int64_t>(THREADS) * MAX_PER_THREAD) return cudaErrorNotSupported;
  if (rows > 0x7fffffff) return cudaErrorInvalidConfiguration;
  const bool aligned = ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(attn_proj) |
                         reinterpret_cast<uintptr_t>(attn_proj2) | reinterpret_cast<uintptr_t>(y)) &
                        15u) == 0;
  if (attn_proj2)
    residual_rmsnorm_kernel<true><<<static_cast<unsigned>(rows), THREADS, 0, stream>>>(
        static_cast<const __nv_bfloat16 *>(x), static_cast<const __nv_bfloat16 *>(attn_proj),
        static_cast<const __nv_bfloat16 *>(attn_proj2), static_cast<__nv_bfloat16 *>(y), cols,
        eps, aligned);
  else
    residual_rmsnorm_kernel<false><<<static_cast<unsigned>(rows), THREADS, 0, stream>>>(
        static_cast<const __nv_bfloat16 *>(x), static_cast<const __nv_bfloat16 *>(attn_proj),
        nullptr, static_cast<__nv_bfloat16 *>(y), cols, eps, aligned);
  if (info) {
    info->launches += 1;
    info->set_route("attn_block_region");
  }
  return cudaGetLastError();
}

}  // namespace mcb

// FP8 block-scaled GEMM and blockwise quantiser (e4m3 / e5m2, OCP formats).
//
//   C[m,n] = sum_kb sa[m/128, kb] * sbt[n/128, kb] * sum_{k in kb} A[m,k] Bt[n,k]
//
// A [M,K] and Bt [N,K] hold fp8 codes, K-major; sa / sbt hold one fp32 scale
// per 128x128 block. This is the arithmetic the reference's FP8 "WGMMA"
// preflight (src/lowering_pipeline.cpp:2531-2572) describes but never
// implements; the fp32 scales are arbitrary (absmax/448), so the hardware
// UE8M0 block-scale MMA cannot represent them and the scaling is done on
// CUDA cores ("promotion").
//
// GEMM kernel (persistent, one CTA per SM, 320 threads):
//   warp 0      TMA producer, 4-stage ring of 128x128 A and 256x128 Bt tiles
//               (one 128-deep K block per stage, 48 KiB, 128-byte swizzle).
//   warp 1      allocates 512 TMEM columns = two 128x256 f32 partial buffers;
//               one thread issues 4 tcgen05.mma.kind::f8f6f4 (K=32 each) per
//               K block into a fresh partial, committing `pfull[buf]`.
//   warps 2-9   promotion: warp w reads TMEM lane quarter w%4 and 128-column
//               half (w-2)/4 of the partial (16 columns per tcgen05.ld),
//               multiplies by sa*sbt of that K block and accumulates into 128
//               f32 registers per thread; after the last K block it rounds to
//               bf16/f32 and stores. Two warps per lane quarter overlap their
//               TMEM-load latencies, and two partial buffers let the MMA of
//               block kb+1 overlap the promotion of block kb.
// Tiles are rasterised in groups of 16 M-tiles so the CTAs running at once
// share A and Bt panels through L2 (config 4's operands are 2x L2).
//
// Roofline (config 4, 16384^3): 2*M*N*K = 8.796 TFLOP against the FP8 dense
// tensor peak (2x the bf16 peak).
#include <cuda_bf16.h>
#include <cuda_fp8.h>

#include "common.cuh"
#include "internal.h"

namespace mcb {
namespace {

constexpr int BM = 128, BN = 256, BKB = 128;  // K block == scale block
constexpr int STAGES = 4;
constexpr int A_BYTES = BM * BKB;    // 16 KiB
constexpr int B_BYTES = BN * BKB;    // 32 KiB
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int PROMO_WARPS = 8;                      // 2 per TMEM lane quarter
constexpr int COLS_PER_WARP = BN * 4 / PROMO_WARPS;  // 128
constexpr int THREADS = 64 + 32 * PROMO_WARPS;       // producer, MMA, promotion
constexpr int GROUP_M = 16;

struct Params {
  int64_t m, n, k, ld_c;
  int m_tiles, n_tiles, num_tiles, num_kb;
  int64_t sa_ld, sb_ld;  // scales per row of the scale grids (= ceil(K/128))
  const float *sa, *sbt;
  void *c;
  int c_bf16;
  uint32_t idesc;
  uint32_t *status;
};

__device__ __forceinline__ void tile_coords(const Params &p, int tile, int &mt, int &nt) {
  const int per_group = GROUP_M * p.n_tiles;
  const int g = tile / per_group;
  const int r = tile - g * per_group;
  const int rows = min(GROUP_M, p.m_tiles - g * GROUP_M);
  mt = g * GROUP_M + r % rows;
  nt = r / rows;
}

__global__ void __launch_bounds__(THREADS, 1)
    gemm_fp8_kernel(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tb,
                    const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t *sa_tiles = smem;
  uint8_t *sb_tiles = smem + STAGES * A_BYTES;
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + STAGES * STAGE_BYTES);
  uint64_t *full = bars, *empty = bars + STAGES;
  uint64_t *pfull = bars + 2 * STAGES, *pempty = pfull + 2;
  uint64_t *drain = pempty + 2;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&pfull[b], 1);
      mbar_init(&pempty[b], PROMO_WARPS);  // one elected arrival per promotion warp
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&ta);
    tma_prefetch_desc(&tb);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x) {
        int mt, nt;
        tile_coords(p, tile, mt, nt);
        for (int kb = 0; kb < p.num_kb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, p.status, kErrTimeoutEmpty))
            goto producer_done;
          mbar_arrive_expect_tx(&full[stage], STAGE_BYTES);
          tma_load_2d(sa_tiles + stage * A_BYTES, &ta, &full[stage], kb * BKB, mt * BM);
          tma_load_2d(sb_tiles + stage * B_BYTES, &tb, &full[stage], kb * BKB, nt * BN);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    producer_done:;
    }
  } else if (warp == 1) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0, kc = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x) {
        for (int kb = 0; kb < p.num_kb; ++kb, ++kc) {
          const int buf = kc & 1;
          if (!(ok = mbar_wait(&pempty[buf], ((kc >> 1) & 1) ^ 1, abort_flag, p.status,
                               kErrTimeoutAccum)))
            break;
          if (!(ok = mbar_wait(&full[stage], phase, abort_flag, p.status, kErrTimeoutFull))) break;
          tc_fence_after();
          const uint32_t a_addr = smem_u32(sa_tiles + stage * A_BYTES);
          const uint32_t b_addr = smem_u32(sb_tiles + stage * B_BYTES);
#pragma unroll
          for (int kk = 0; kk < BKB / 32; ++kk)
            mma_f8_ss(tmem + buf * BN, make_sdesc_sw128(a_addr + kk * 32, 16, 1024),
                      make_sdesc_sw128(b_addr + kk * 32, 16, 1024), p.idesc, kk ? 1u : 0u);
          mma_commit(&empty[stage]);
          mma_commit(&pfull[buf]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      mma_commit(drain);
      if (!mbar_wait(drain, 0, nullptr, p.status, kErrTimeoutDrain)) *abort_flag = 1;
    }
  } else {
    // Promotion warps 2..(2+PROMO_WARPS): warp w reads TMEM lane quarter w%4
    // and the 64-column group (w-2)/4 of the 256-column partial; four warps
    // share each lane quarter so their TMEM-load latencies overlap.
    const int q = warp & 3;
    const int grp = (warp - 2) >> 2;
    const uint32_t lane_base =
        tmem + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(grp * COLS_PER_WARP);
    uint32_t kc = 0;
    for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x) {
      int mt, nt;
      tile_coords(p, tile, mt, nt);
      const int64_t row = static_cast<int64_t>(mt) * BM + q * 32 + lane;
      const int64_t col0 = static_cast<int64_t>(nt) * BN + grp * COLS_PER_WARP;
      const int sa_row = mt;                                       // M block (BM == block)
      const int sb_row = nt * 2 + (grp * COLS_PER_WARP) / 128;     // N block of these columns
      const bool cols_live = col0 < p.n;
      uint64_t acc2[COLS_PER_WARP / 2];  // f32 accumulator pairs (packed f32x2 FMAs)
#pragma unroll
      for (int i = 0; i < COLS_PER_WARP / 2; ++i) acc2[i] = 0;
      bool ok = true;
      for (int kb = 0; kb < p.num_kb; ++kb, ++kc) {
        const int buf = kc & 1;
        const float s = __ldg(p.sa + sa_row * p.sa_ld + kb) *
                        (cols_live ? __ldg(p.sbt + sb_row * p.sb_ld + kb) : 0.0f);
        if (!(ok = mbar_wait_warp(&pfull[buf], (kc >> 1) & 1, abort_flag, p.status,
                                  kErrTimeoutAccum)))
          break;
        tc_fence_after();
        const uint64_t s2 = f2_pack(s, s);
#pragma unroll
        for (int c = 0; c < COLS_PER_WARP / 16; ++c) {
          uint32_t r[16];  // 16-column loads: the 128 accumulators + 16 stay in registers
          tmem_ld16_sync(lane_base + buf * BN + c * 16, r);
#pragma unroll
          for (int i = 0; i < 8; ++i)
            acc2[c * 8 + i] = f2_fma(s2, f2_pack(__uint_as_float(r[2 * i]), __uint_as_float(r[2 * i + 1])),
                                     acc2[c * 8 + i]);
        }
        // One arrival per warp, after every lane's loads have completed
        // (per-thread arrivals: config 4 1690 instead of 1955 TFLOP/s).
        tc_fence_before();
        mbar_arrive_warp(&pempty[buf]);
      }
      if (!ok) break;
      float acc[COLS_PER_WARP];
#pragma unroll
      for (int i = 0; i < COLS_PER_WARP / 2; ++i) f2_unpack(acc2[i], acc[2 * i], acc[2 * i + 1]);
      if (row < p.m && cols_live) {
        const bool full_cols = col0 + COLS_PER_WARP <= p.n;
        if (p.c_bf16) {
          __nv_bfloat16 *crow = reinterpret_cast<__nv_bfloat16 *>(p.c) + row * p.ld_c + col0;
          if (full_cols) {
#pragma unroll
            for (int v = 0; v < COLS_PER_WARP / 8; ++v) {
              uint4 w;
              w.x = pack_bf16x2(acc[v * 8 + 0], acc[v * 8 + 1]);
              w.y = pack_bf16x2(acc[v * 8 + 2], acc[v * 8 + 3]);
              w.z = pack_bf16x2(acc[v * 8 + 4], acc[v * 8 + 5]);
              w.w = pack_bf16x2(acc[v * 8 + 6], acc[v * 8 + 7]);
              reinterpret_cast<uint4 *>(crow)[v] = w;
            }
          } else {
#pragma unroll
            for (int i = 0; i < COLS_PER_WARP; ++i)
              if (col0 + i < p.n) crow[i] = __float2bfloat16_rn(acc[i]);
          }
        } else {
          float *crow = reinterpret_cast<float *>(p.c) + row * p.ld_c + col0;
          if (full_cols) {
#pragma unroll
            for (int v = 0; v < COLS_PER_WARP / 4; ++v)
              reinterpret_cast<float4 *>(crow)[v] =
                  make_float4(acc[v * 4], acc[v * 4 + 1], acc[v * 4 + 2], acc[v * 4 + 3]);
          } else {
#pragma unroll
            for (int i = 0; i < COLS_PER_WARP; ++i)
              if (col0 + i < p.n) crow[i] = acc[i];
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ---- blockwise quantiser -------------------------------------------------------
// One CTA (256 threads) per block x block tile: absmax reduction, then
// q = cvt.satfinite.rn(x / s) with an IEEE division, as the oracle specifies.
template <typename T>
__device__ __forceinline__ float to_f(T v);
template <>
__device__ __forceinline__ float to_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}

template <typename T>
__global__ void __launch_bounds__(256) quantize_kernel(const T *__restrict__ x, uint8_t *__restrict__ q,
                                                       float *__restrict__ scales, int64_t rows,
                                                       int64_t cols, int64_t ld_x, int64_t block,
                                                       int e5m2) {
  __shared__ float red[8];
  const int64_t r0 = static_cast<int64_t>(blockIdx.y) * block;
  const int64_t c0 = static_cast<int64_t>(blockIdx.x) * block;
  const int64_t r1 = min(rows, r0 + block), c1 = min(cols, c0 + block);
  const int64_t w = c1 - c0, count = (r1 - r0) * w;
  float amax = 0.0f;
  for (int64_t i = threadIdx.x; i < count; i += blockDim.x) {
    const float v = to_f(x[(r0 + i / w) * ld_x + c0 + i % w]);
    amax = fmaxf(amax, fabsf(v));
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < 8 ? red[threadIdx.x] : 0.0f;
#pragma unroll
    for (int off = 4; off > 0; off >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, off));
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  const float fmax = e5m2 ? 57344.0f : 448.0f;
  const float s = red[0] > 0.0f ? __fdiv_rn(red[0], fmax) : 1.0f;
  if (threadIdx.x == 0) scales[blockIdx.y * gridDim.x + blockIdx.x] = s;
  for (int64_t i = threadIdx.x; i < count; i += blockDim.x) {
    const int64_t r = r0 + i / w, c = c0 + i % w;
    const float v = __fdiv_rn(to_f(x[r * ld_x + c]), s);
    q[r * cols + c] = static_cast<uint8_t>(
        __nv_cvt_float_to_fp8(v, __NV_SATFINITE, e5m2 ? __NV_E5M2 : __NV_E4M3));
  }
}

// ---- CUDA-core FP8 GEMM for shapes the TMA path cannot take ----------------------
__device__ __forceinline__ float fp8_to_f(uint8_t v, int e5m2) {
  __half_raw h = __nv_cvt_fp8_to_halfraw(static_cast<__nv_fp8_storage_t>(v),
                                         e5m2 ? __NV_E5M2 : __NV_E4M3);
  return __half2float(__half(h));
}

__global__ void __launch_bounds__(256) gemm_fp8_simt_kernel(
    const uint8_t *__restrict__ a, int a_e5m2, const float *__restrict__ sa,
    const uint8_t *__restrict__ bt, int b_e5m2, const float *__restrict__ sbt, void *c, int c_bf16,
    int64_t m, int64_t n, int64_t k, int64_t block) {
  const int64_t row = blockIdx.y;
  const int64_t col = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (row >= m || col >= n) return;
  const int64_t kbs = (k + block - 1) / block;
  float acc = 0.0f;
  for (int64_t kb = 0; kb < kbs; ++kb) {
    float part = 0.0f;
    const int64_t k1 = min(k, (kb + 1) * block);
    for (int64_t h = kb * block; h < k1; ++h)
      part = fmaf(fp8_to_f(a[row * k + h], a_e5m2), fp8_to_f(bt[col * k + h], b_e5m2), part);
    acc = fmaf(sa[(row / block) * kbs + kb] * sbt[(col / block) * kbs + kb], part, acc);
  }
  if (c_bf16)
    reinterpret_cast<__nv_bfloat16 *>(c)[row * n + col] = __float2bfloat16_rn(acc);
  else
    reinterpret_cast<float *>(c)[row * n + col] = acc;
}

}  // namespace

cudaError_t launch_fp8_quantize(const void *x, int x_dtype, uint8_t *q, float *scales,
                                int64_t rows, int64_t cols, int64_t ld_x, int64_t block,
                                int fmt_e5m2, cudaStream_t stream, LaunchInfo *info) {
  if (rows == 0 || cols == 0) return cudaSuccess;
  dim3 grid(static_cast<unsigned>((cols + block - 1) / block),
            static_cast<unsigned>((rows + block - 1) / block));
  if (grid.y > 65535u) return cudaErrorInvalidConfiguration;
  if (x_dtype == 3)
    quantize_kernel<__nv_bfloat16><<<grid, 256, 0, stream>>>(
        static_cast<const __nv_bfloat16 *>(x), q, scales, rows, cols, ld_x, block, fmt_e5m2);
  else
    quantize_kernel<float><<<grid, 256, 0, stream>>>(static_cast<const float *>(x), q, scales,
                                                     rows, cols, ld_x, block, fmt_e5m2);
  if (info) {
    info->launches = 1;
    info->tile_m = info->tile_n = static_cast<int>(block);
    info->ctas = static_cast<int>(grid.x * grid.y);
    info->set_route("fp8_blockwise_quantize");
  }
  return cudaGetLastError();
}

cudaError_t launch_gemm_fp8_tc(const uint8_t *a, int a_e5m2, const float *sa, const uint8_t *bt,
                               int b_e5m2, const float *sbt, void *c, int c_bf16, int64_t m,
                               int64_t n, int64_t k, int64_t block, uint32_t *status, int sms,
                               cudaStream_t stream, LaunchInfo *info) {
  if (m == 0 || n == 0) return cudaSuccess;
  if (block != BKB || k % 16 != 0 || k == 0) return cudaErrorNotSupported;
  CUtensorMap ta, tb;
  if (!encode_tmap_2d(&ta, CU_TENSOR_MAP_DATA_TYPE_UINT8, a, k, m, k, BKB, BM,
                      CU_TENSOR_MAP_SWIZZLE_128B) ||
      !encode_tmap_2d(&tb, CU_TENSOR_MAP_DATA_TYPE_UINT8, bt, k, n, k, BKB, BN,
                      CU_TENSOR_MAP_SWIZZLE_128B))
    return cudaErrorNotSupported;
  Params p;
  p.m = m;
  p.n = n;
  p.k = k;
  p.ld_c = n;
  p.m_tiles = static_cast<int>((m + BM - 1) / BM);
  p.n_tiles = static_cast<int>((n + BN - 1) / BN);
  const int64_t tiles = static_cast<int64_t>(p.m_tiles) * p.n_tiles;
  if (tiles > 0x7fffffff) return cudaErrorNotSupported;
  p.num_tiles = static_cast<int>(tiles);
  p.num_kb = static_cast<int>((k + BKB - 1) / BKB);
  p.sa_ld = p.num_kb;
  p.sb_ld = p.num_kb;
  p.sa = sa;
  p.sbt = sbt;
  p.c = c;
  p.c_bf16 = c_bf16;
  p.idesc = make_idesc(a_e5m2 ? 1u : 0u, b_e5m2 ? 1u : 0u, 0, 0, BM, BN);
  p.status = status;
  const size_t smem = static_cast<size_t>(STAGES) * STAGE_BYTES + 256 + 1024;
  cudaError_t e = cudaFuncSetAttribute(gemm_fp8_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  const int grid = static_cast<int>(tiles < sms ? tiles : sms);
  gemm_fp8_kernel<<<grid, THREADS, smem, stream>>>(ta, tb, p);
  if (info) {
    info->launches = 1;
    info->tile_m = BM;
    info->tile_n = BN;
    info->tile_k = BKB;
    info->stages = STAGES;
    info->ctas = grid;
    info->set_route("tcgen05_fp8_blockscaled_gemm");
  }
  return cudaGetLastError();
}

cudaError_t launch_gemm_fp8_simt(const uint8_t *a, int a_e5m2, const float *sa,
                                 const uint8_t *bt, int b_e5m2, const float *sbt, void *c,
                                 int c_bf16, int64_t m, int64_t n, int64_t k, int64_t block,
                                 cudaStream_t stream, LaunchInfo *info) {
  if (m == 0 || n == 0) return cudaSuccess;
  if (m > 65535) return cudaErrorInvalidConfiguration;
  dim3 grid(static_cast<unsigned>((n + 255) / 256), static_cast<unsigned>(m));
  gemm_fp8_simt_kernel<<<grid, 256, 0, stream>>>(a, a_e5m2, sa, bt, b_e5m2, sbt, c, c_bf16, m, n,
                                                 k, block);
  if (info) {
    info->launches = 1;
    info->tile_m = 1;
    info->tile_n = 256;
    info->ctas = static_cast<int>(grid.x * grid.y);
    info->set_route("simt_fp8_blockscaled_gemm");
  }
  return cudaGetLastError();
}

}  // namespace mcb

// Typed isolated GEMMs, bit-exact with the reference's typed CPU references
// (compiler/lib/runtime/cpu_numeric_reference.cpp):
//
//   int8 x int8 -> int32, accumulated modulo 2^32 (:185-209). Integer
//     products and sums are exact, so the tensor-core kernel (tcgen05.mma
//     kind::i8, int32 accumulator in TMEM, no saturation) gives the same bits
//     as the CPU loop whatever the summation order.
//   bf16 x bf16 -> f32 with one fused multiply-add per k in increasing order
//     (:108-127). Rounding depends on the order, so this one runs on CUDA
//     cores with fmaf in exactly that order.
//
// int8 kernel layout: A [M,K] K-major. B [K,N] is consumed MN-major straight
// from memory when its rows are 16-byte aligned (tcgen05 takes MN-major 8-bit
// operands); otherwise it is first transposed into a K-major scratch
// Bt [N,K] by a small kernel. Two persistent, warp-specialised kernels:
//
//   gemm_i8_pair_kernel (M >= 256): clusters of two CTAs on two SMs compute
//     256x256 tiles with tcgen05.mma.cta_group::2.kind::i8 (M=256, N=256,
//     K=32). CTA r stages rows [128r, 128r+128) of the A tile and columns
//     [128r, 128r+128) of the B tile, so each SM moves 32 KiB per 128-deep
//     K block (half the B bytes of a single-SM 128x256 tile) through a
//     6-stage TMA ring; its TMEM holds its 128 rows of two 256-column int32
//     accumulators. The leader CTA issues every MMA; eight epilogue warps per
//     CTA (two per TMEM lane quarter) store int32 rows.
//   gemm_i8_kernel (M < 256): one CTA per SM, 128x256 tiles, cta_group::1,
//     4-stage ring, four epilogue warps.
//
// Zero points (the legacy quantized_i8 matmul, src/mlir_engine.cpp:944-958:
// C = sum_k (A - za)(B - zb) in wrapping int32): in Z/2^32 the sum expands to
// A.B + K*za*zb - zb*rowsum(A) - za*colsum(B), so the tensor cores still
// multiply the raw codes and the epilogue adds one per-row and one
// per-column term (sums from a short pre-pass over A and B).
#include <cuda_bf16.h>

#include <atomic>
#include <cstdlib>

#include "common.cuh"
#include "internal.h"

namespace mcb {
namespace {

constexpr int BM = 128, BN = 256, BK = 128, STAGES = 4;  // BK in bytes == elements
constexpr int A_BYTES = BM * BK, B_BYTES = BN * BK, STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int THREADS = 192;
constexpr int MN_CHUNK = 128;                // B columns per 128-byte swizzle row
constexpr int MN_CHUNK_BYTES = MN_CHUNK * BK;  // one MN-major box: 128 columns x BK rows
constexpr size_t SMEM_BYTES = static_cast<size_t>(STAGES) * STAGE_BYTES + 256 + 1024;

constexpr int P_B_COLS = BN / 2;  // B columns staged per CTA of a pair
constexpr int P_A_BYTES = BM * BK, P_B_BYTES = P_B_COLS * BK;
constexpr int P_STAGE_BYTES = P_A_BYTES + P_B_BYTES;  // 32 KiB
constexpr int P_STAGES = 6;
constexpr int P_THREADS = 320;
constexpr size_t P_SMEM_BYTES = static_cast<size_t>(P_STAGES) * P_STAGE_BYTES + 256 + 1024;

// kind::i8 instruction descriptor: D s32 (format 2), A and B signed 8-bit
// (format 1), A K-major, B K-major or MN-major.
__host__ __device__ constexpr uint32_t idesc_i8(uint32_t b_mn, uint32_t m, uint32_t n) {
  return (2u << 4) | (1u << 7) | (1u << 10) | (b_mn << 16) | ((n >> 3) << 17) | ((m >> 4) << 24);
}

__device__ __forceinline__ void mma_i8_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                          uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void mma_i8_ss_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                               uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// B operand descriptor for the kk-th 32-deep K step of a stage. K-major Bt:
// K advances 32 bytes inside each 128-byte row. MN-major B: 128-column chunks
// LBO = MN_CHUNK_BYTES apart, 8-row K groups SBO = 1 KiB apart, and K
// advances by 32 rows = 4 KiB.
__device__ __forceinline__ uint64_t b_desc_i8(uint32_t b_addr, int kk, int b_mn) {
  return b_mn ? make_sdesc_sw128(b_addr + kk * 32 * 128, MN_CHUNK_BYTES, 1024)
              : make_sdesc_sw128(b_addr + kk * 32, 16, 1024);
}

struct Params {
  int64_t m, n, ld_c;
  int n_tiles, num_tiles, num_kb;
  int b_mn;
  int zp;                   // zero-point correction on
  uint32_t za, zb, kzz;     // zero points and K*za*zb, modulo 2^32
  const int32_t *row_sum;   // sum_k A[m,k] (null when zb == 0)
  const int32_t *col_sum;   // sum_k B[k,n] (null when za == 0)
  int32_t *c;
  uint32_t *status;
};

// Adds K*za*zb - zb*row_sum[row] - za*col_sum[col] to one 32-column chunk
// (uint32 arithmetic: the wrapping int32 result of the reference).
__device__ __forceinline__ void zero_point_chunk(const Params &p, uint32_t (&r)[32], int64_t row,
                                                 int64_t col0) {
  const uint32_t rc = p.kzz - (p.row_sum ? p.zb * static_cast<uint32_t>(p.row_sum[row]) : 0u);
  if (!p.col_sum) {
#pragma unroll
    for (int i = 0; i < 32; ++i) r[i] += rc;
  } else if (col0 + 32 <= p.n) {
    // Every lane of the warp reads the same 128 bytes (a broadcast).
    const int4 *cs = reinterpret_cast<const int4 *>(p.col_sum + col0);
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const int4 v = cs[q];
      r[q * 4 + 0] += rc - p.za * static_cast<uint32_t>(v.x);
      r[q * 4 + 1] += rc - p.za * static_cast<uint32_t>(v.y);
      r[q * 4 + 2] += rc - p.za * static_cast<uint32_t>(v.z);
      r[q * 4 + 3] += rc - p.za * static_cast<uint32_t>(v.w);
    }
  } else {
    for (int i = 0; i < 32; ++i)
      if (col0 + i < p.n) r[i] += rc - p.za * static_cast<uint32_t>(p.col_sum[col0 + i]);
  }
}

// Stores one 32-column int32 chunk of one output row.
__device__ __forceinline__ void store_chunk(const Params &p, uint32_t (&r)[32], int64_t row,
                                            int64_t col0) {
  if (row >= p.m) return;
  if (p.zp) zero_point_chunk(p, r, row, col0);
  int32_t *crow = p.c + row * p.ld_c + col0;
  if (col0 + 32 <= p.n && (p.ld_c % 4 == 0)) {
#pragma unroll
    for (int q = 0; q < 8; ++q)
      reinterpret_cast<uint4 *>(crow)[q] =
          make_uint4(r[q * 4], r[q * 4 + 1], r[q * 4 + 2], r[q * 4 + 3]);
  } else {
    for (int i = 0; i < 32; ++i)
      if (col0 + i < p.n) crow[i] = static_cast<int32_t>(r[i]);
  }
}

__global__ void __launch_bounds__(THREADS, 1)
    gemm_i8_kernel(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tb,
                   const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t *sa = smem, *sb = smem + STAGES * A_BYTES;
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + STAGES * STAGE_BYTES);
  uint64_t *full = bars, *empty = bars + STAGES, *acc_full = bars + 2 * STAGES;
  uint64_t *acc_empty = acc_full + 2, *drain = acc_empty + 2;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 4);  // one arrival per epilogue warp
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
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
        const int m0 = (tile / p.n_tiles) * BM, n0 = (tile % p.n_tiles) * BN;
        for (int kb = 0; kb < p.num_kb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, p.status, kErrTimeoutEmpty))
            goto producer_done;
          mbar_arrive_expect_tx(&full[stage], STAGE_BYTES);
          tma_load_2d(sa + stage * A_BYTES, &ta, &full[stage], kb * BK, m0);
          if (p.b_mn) {
#pragma unroll
            for (int j = 0; j < BN / MN_CHUNK; ++j)
              tma_load_2d(sb + stage * B_BYTES + j * MN_CHUNK_BYTES, &tb, &full[stage],
                          n0 + j * MN_CHUNK, kb * BK);
          } else {
            tma_load_2d(sb + stage * B_BYTES, &tb, &full[stage], kb * BK, n0);
          }
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
      const uint32_t idesc = idesc_i8(p.b_mn ? 1u : 0u, BM, BN);
      int stage = 0, acc = 0;
      uint32_t phase = 0, acc_phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x) {
        if (!(ok = mbar_wait(&acc_empty[acc], acc_phase ^ 1, abort_flag, p.status,
                             kErrTimeoutAccum)))
          break;
        tc_fence_after();
        for (int kb = 0; kb < p.num_kb; ++kb) {
          if (!(ok = mbar_wait(&full[stage], phase, abort_flag, p.status, kErrTimeoutFull))) break;
          tc_fence_after();
          const uint32_t a_addr = smem_u32(sa + stage * A_BYTES);
          const uint32_t b_addr = smem_u32(sb + stage * B_BYTES);
#pragma unroll
          for (int kk = 0; kk < BK / 32; ++kk)
            mma_i8_ss(tmem + acc * BN, make_sdesc_sw128(a_addr + kk * 32, 16, 1024),
                      b_desc_i8(b_addr, kk, p.b_mn), idesc, (kb | kk) ? 1u : 0u);
          mma_commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        mma_commit(&acc_full[acc]);
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1;
      }
      mma_commit(drain);
      if (!mbar_wait(drain, 0, nullptr, p.status, kErrTimeoutDrain)) *abort_flag = 1;
    }
  } else {
    const int sub = warp & 3;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x) {
      const int64_t m0 = static_cast<int64_t>(tile / p.n_tiles) * BM;
      const int64_t n0 = static_cast<int64_t>(tile % p.n_tiles) * BN;
      if (!mbar_wait_warp(&acc_full[acc], acc_phase, abort_flag, p.status, kErrTimeoutAccum))
        break;
      tc_fence_after();
      const int64_t row = m0 + sub * 32 + lane;
      const uint32_t t_row = tmem + (static_cast<uint32_t>(sub * 32) << 16) + acc * BN;
#pragma unroll 1
      for (int c = 0; c < BN; c += 32) {
        if (n0 + c >= p.n) break;
        uint32_t r[32];
        tmem_ld32_sync(t_row + c, r);
        store_chunk(p, r, row, n0 + c);
      }
      tc_fence_before();
      mbar_arrive_warp(&acc_empty[acc]);
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(P_THREADS, 1)
    gemm_i8_pair_kernel(const __grid_constant__ CUtensorMap ta,
                        const __grid_constant__ CUtensorMap tb, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t *sa = smem, *sb = smem + P_STAGES * P_A_BYTES;
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + P_STAGES * P_STAGE_BYTES);
  uint64_t *full = bars, *empty = bars + P_STAGES, *acc_full = bars + 2 * P_STAGES;
  uint64_t *acc_empty = acc_full + 2, *drain = acc_empty + 2;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int cluster = blockIdx.x >> 1, nclusters = gridDim.x >> 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < P_STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 16);  // 8 epilogue warps of each CTA (leader's copy)
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
    tmem_alloc_pair(tmem_slot, 512);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncwarp();
  cluster_sync();  // barriers initialised and TMEM allocated in both CTAs
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      const uint32_t full_leader0 = mapa_shared(smem_u32(&full[0]), 0);
      int stage = 0;
      uint32_t phase = 0;
      for (int tile = cluster; tile < p.num_tiles; tile += nclusters) {
        const int m0 = (tile / p.n_tiles) * (2 * BM) + static_cast<int>(rank) * BM;
        const int n0 = (tile % p.n_tiles) * BN + static_cast<int>(rank) * P_B_COLS;
        for (int kb = 0; kb < p.num_kb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, p.status, kErrTimeoutEmpty))
            goto producer_done;
          const uint32_t fbar = full_leader0 + stage * 8;
          if (leader) mbar_arrive_expect_tx(&full[stage], 2 * P_STAGE_BYTES);
          tma_load_2d_pair(sa + stage * P_A_BYTES, &ta, fbar, kb * BK, m0);
          if (p.b_mn)
            tma_load_2d_pair(sb + stage * P_B_BYTES, &tb, fbar, n0, kb * BK);
          else
            tma_load_2d_pair(sb + stage * P_B_BYTES, &tb, fbar, kb * BK, n0);
          if (++stage == P_STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    producer_done:;
    }
  } else if (warp == 1) {
    if (leader && lane == 0) {
      const uint32_t idesc = idesc_i8(p.b_mn ? 1u : 0u, 2 * BM, BN);
      int stage = 0, acc = 0;
      uint32_t phase = 0, acc_phase = 0;
      for (int tile = cluster; tile < p.num_tiles; tile += nclusters) {
        if (!mbar_wait(&acc_empty[acc], acc_phase ^ 1, abort_flag, p.status, kErrTimeoutAccum))
          break;
        tc_fence_after();
        const uint32_t d_tmem = tmem + static_cast<uint32_t>(acc * BN);
        bool ok = true;
        for (int kb = 0; kb < p.num_kb; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag, p.status, kErrTimeoutFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(sa + stage * P_A_BYTES);
          const uint32_t b_addr = smem_u32(sb + stage * P_B_BYTES);
#pragma unroll
          for (int kk = 0; kk < BK / 32; ++kk)
            mma_i8_ss_pair(d_tmem, make_sdesc_sw128(a_addr + kk * 32, 16, 1024),
                           b_desc_i8(b_addr, kk, p.b_mn), idesc, (kb | kk) != 0 ? 1u : 0u);
          mma_commit_pair(&empty[stage], 0x3);
          if (++stage == P_STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        mma_commit_pair(&acc_full[acc], 0x3);
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1;
      }
      mma_commit_pair(drain, 0x1);
      if (!mbar_wait(drain, 0, nullptr, p.status, kErrTimeoutDrain)) *abort_flag = 1;
    }
  } else {
    const int sub = warp & 3;
    const int half = (warp - 2) >> 2;  // 128-column half of the tile
    const uint32_t acc_empty_leader = mapa_shared(smem_u32(&acc_empty[0]), 0);
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int tile = cluster; tile < p.num_tiles; tile += nclusters) {
      const int64_t m0 = static_cast<int64_t>(tile / p.n_tiles) * (2 * BM) + rank * BM;
      const int64_t n0 = static_cast<int64_t>(tile % p.n_tiles) * BN;
      if (!mbar_wait_warp(&acc_full[acc], acc_phase, abort_flag, p.status, kErrTimeoutAccum))
        break;
      tc_fence_after();
      const int64_t row = m0 + sub * 32 + lane;
      const uint32_t t_row =
          tmem + (static_cast<uint32_t>(sub * 32) << 16) + static_cast<uint32_t>(acc * BN);
#pragma unroll 1
      for (int c = half * (BN / 2); c < (half + 1) * (BN / 2); c += 32) {
        if (n0 + c >= p.n) break;
        uint32_t r[32];
        tmem_ld32_sync(t_row + c, r);
        store_chunk(p, r, row, n0 + c);
      }
      tc_fence_before();
      mbar_arrive_cluster_warp(acc_empty_leader + acc * 8);
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1;
    }
  }
  tc_fence_before();
  __syncwarp();
  cluster_sync();  // every pair MMA has completed before either CTA frees TMEM
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, 512);
  }
}

// Clusters of gemm_i8_pair_kernel that fit on the device at once, cached per
// device (-1: the pair kernel cannot run here).
int i8_pair_clusters_resident(int device) {
  static std::atomic<int> cache[64];
  if (device < 0 || device >= 64) return -1;
  int v = cache[device].load(std::memory_order_relaxed);
  if (v != 0) return v;
  int n = -1;
  if (cudaFuncSetAttribute(gemm_i8_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(P_SMEM_BYTES)) == cudaSuccess) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2, 1, 1);
    cfg.blockDim = dim3(P_THREADS, 1, 1);
    cfg.dynamicSmemBytes = P_SMEM_BYTES;
    if (cudaOccupancyMaxActiveClusters(&n, gemm_i8_pair_kernel, &cfg) != cudaSuccess || n <= 0)
      n = -1;
  }
  (void)cudaGetLastError();
  cache[device].store(n, std::memory_order_relaxed);
  return n;
}

// B [K,N] -> Bt [N,K] for 1-byte elements, 32x32 tiles through shared memory.
__global__ void transpose_u8_kernel(const uint8_t *__restrict__ in, uint8_t *__restrict__ out,
                                    int64_t rows, int64_t cols, int64_t ld_in) {
  __shared__ uint8_t tile[32][33];
  const int64_t r0 = static_cast<int64_t>(blockIdx.y) * 32, c0 = static_cast<int64_t>(blockIdx.x) * 32;
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int64_t r = r0 + i, c = c0 + threadIdx.x;
    tile[i][threadIdx.x] = (r < rows && c < cols) ? in[r * ld_in + c] : 0;
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int64_t orow = c0 + i, ocol = r0 + threadIdx.x;
    if (orow < cols && ocol < rows) out[orow * rows + ocol] = tile[threadIdx.x][i];
  }
}

// Same transpose with 64 x 64 byte tiles and 16-byte global accesses, for
// rows/cols that are multiples of 16 bytes and 16-byte aligned rows (each
// thread moves one 16-byte row segment in and one 16-byte column segment out).
__global__ void __launch_bounds__(256) transpose_u8_v16_kernel(const uint8_t *__restrict__ in,
                                                               uint8_t *__restrict__ out,
                                                               int64_t rows, int64_t cols,
                                                               int64_t ld_in) {
  __shared__ uint8_t tile[64][64 + 4];
  const int64_t r0 = static_cast<int64_t>(blockIdx.y) * 64, c0 = static_cast<int64_t>(blockIdx.x) * 64;
  const int t = threadIdx.x, tr = t >> 2, tc = (t & 3) * 16;
  if (r0 + tr < rows && c0 + tc < cols) {
    const uint4 v = *reinterpret_cast<const uint4 *>(in + (r0 + tr) * ld_in + c0 + tc);
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int b = 0; b < 4; ++b) tile[tr][tc + i * 4 + b] = static_cast<uint8_t>(w[i] >> (8 * b));
  }
  __syncthreads();
  // out row (c0 + tr) gets bytes r0 + tc .. r0 + tc + 15 of column tr of the tile.
  if (c0 + tr < cols && r0 + tc < rows) {
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      w[i] = 0;
#pragma unroll
      for (int b = 0; b < 4; ++b) w[i] |= static_cast<uint32_t>(tile[tc + i * 4 + b][tr]) << (8 * b);
    }
    *reinterpret_cast<uint4 *>(out + (c0 + tr) * rows + r0 + tc) = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

// CUDA-core int8 GEMM (exact; any shape/stride). One thread per output;
// (A - za)(B - zb) per k in uint32 arithmetic (za = zb = 0: the plain GEMM).
__global__ void gemm_i8_simt_kernel(const int8_t *__restrict__ a, const int8_t *__restrict__ b,
                                    int32_t *__restrict__ c, int64_t m, int64_t n, int64_t k,
                                    int64_t lda, int64_t ldb, int64_t ldc, uint32_t za,
                                    uint32_t zb) {
  const int64_t row = blockIdx.y;
  const int64_t col = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (row >= m || col >= n) return;
  uint32_t acc = 0;
  for (int64_t h = 0; h < k; ++h)
    acc += (static_cast<uint32_t>(static_cast<int32_t>(a[row * lda + h])) - za) *
           (static_cast<uint32_t>(static_cast<int32_t>(b[h * ldb + col])) - zb);
  c[row * ldc + col] = static_cast<int32_t>(acc);
}

// Sum over k of each row of an int8 matrix x [rows, k] (row stride ld), one
// warp per row; 16-byte loads reduced with dp4a when the rows are aligned.
// The sums are exact for K < 2^24 and wrap modulo 2^32 beyond, which is all
// the zero-point identity needs.
__global__ void __launch_bounds__(256) i8_row_sums_kernel(const int8_t *__restrict__ x,
                                                          int64_t rows, int64_t k, int64_t ld,
                                                          int32_t *__restrict__ out) {
  const int64_t r = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (r >= rows) return;
  const int8_t *row = x + r * ld;
  uint32_t acc = 0;
  int64_t k0 = 0;
  if ((reinterpret_cast<uintptr_t>(row) & 15u) == 0) {
    k0 = k & ~int64_t{15};
#pragma unroll 4
    for (int64_t j = static_cast<int64_t>(lane) * 16; j < k0; j += 512) {
      const int4 v = *reinterpret_cast<const int4 *>(row + j);
      int s4 = __dp4a(v.x, 0x01010101, 0);
      s4 = __dp4a(v.y, 0x01010101, s4);
      s4 = __dp4a(v.z, 0x01010101, s4);
      s4 = __dp4a(v.w, 0x01010101, s4);
      acc += static_cast<uint32_t>(s4);
    }
  }
  for (int64_t j = k0 + lane; j < k; j += 32) acc += static_cast<uint32_t>(static_cast<int32_t>(row[j]));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if (lane == 0) out[r] = static_cast<int32_t>(acc);
}

// Sum over k of each column of an int8 matrix x [k, cols] (row stride ld).
// A CTA covers 512 columns and one K slice: lane l of each of the 8 warps
// owns columns 16l..16l+15 (one 16-byte load per row; a warp reads 512
// contiguous bytes), warp w takes rows w, w+8, ... of the slice. The warps'
// partial sums meet in shared memory, and each CTA adds its 512 totals to
// out (zeroed first) with integer atomics, whose result does not depend on
// their order.
constexpr int CS_COLS = 512;
__global__ void __launch_bounds__(256) i8_col_sums_kernel(const int8_t *__restrict__ x, int64_t k,
                                                          int64_t cols, int64_t ld,
                                                          int64_t k_slice,
                                                          int32_t *__restrict__ out) {
  __shared__ uint32_t part[8][CS_COLS];  // [warp][j * 32 + lane]: conflict-free
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t c0 = static_cast<int64_t>(blockIdx.x) * CS_COLS + lane * 16;
  const int64_t k_begin = static_cast<int64_t>(blockIdx.y) * k_slice;
  const int64_t k_end = k_begin + k_slice < k ? k_begin + k_slice : k;
  uint32_t s[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) s[j] = 0;
  const bool vec = c0 + 16 <= cols && ((reinterpret_cast<uintptr_t>(x) | ld) & 15) == 0;
  if (vec) {
#pragma unroll 4
    for (int64_t r = k_begin + warp; r < k_end; r += 8) {
      const int4 v = *reinterpret_cast<const int4 *>(x + r * ld + c0);
      const uint32_t w[4] = {static_cast<uint32_t>(v.x), static_cast<uint32_t>(v.y),
                             static_cast<uint32_t>(v.z), static_cast<uint32_t>(v.w)};
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int b = 0; b < 4; ++b)
          s[i * 4 + b] += static_cast<uint32_t>(static_cast<int32_t>(static_cast<int8_t>(w[i] >> (8 * b))));
    }
  } else {
    for (int64_t r = k_begin + warp; r < k_end; r += 8)
#pragma unroll
      for (int j = 0; j < 16; ++j)
        if (c0 + j < cols) s[j] += static_cast<uint32_t>(static_cast<int32_t>(x[r * ld + c0 + j]));
  }
#pragma unroll
  for (int j = 0; j < 16; ++j) part[warp][j * 32 + lane] = s[j];
  __syncthreads();
  for (int q = threadIdx.x; q < CS_COLS; q += 256) {
    const int64_t col = static_cast<int64_t>(blockIdx.x) * CS_COLS + q;
    if (col >= cols) break;
    uint32_t tot = 0;
#pragma unroll
    for (int w = 0; w < 8; ++w) tot += part[w][(q & 15) * 32 + (q >> 4)];
    atomicAdd(reinterpret_cast<unsigned int *>(out) + col, tot);
  }
}

// bf16 x bf16 -> f32, one fmaf per k in increasing order from +0 (the
// reference's typed bf16 reference). Coalesced over columns; A row values
// are loaded 16 steps ahead of the dependent fma chain.
__global__ void __launch_bounds__(256) gemm_bf16_fma_kernel(const __nv_bfloat16 *__restrict__ a,
                                                           const __nv_bfloat16 *__restrict__ b,
                                                           float *__restrict__ c, int64_t m,
                                                           int64_t n, int64_t k, int64_t lda,
                                                           int64_t ldb, int64_t ldc) {
  const int64_t row = blockIdx.y;
  const int64_t col = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (row >= m || col >= n) return;
  float acc = 0.0f;
  int64_t h0 = 0;
  for (; h0 + 16 <= k; h0 += 16) {
    float av[16], bv[16];
#pragma unroll
    for (int u = 0; u < 16; ++u) {
      av[u] = __bfloat162float(a[row * lda + h0 + u]);
      bv[u] = __bfloat162float(b[(h0 + u) * ldb + col]);
    }
#pragma unroll
    for (int u = 0; u < 16; ++u) acc = __fmaf_rn(av[u], bv[u], acc);
  }
  for (; h0 < k; ++h0)
    acc = __fmaf_rn(__bfloat162float(a[row * lda + h0]), __bfloat162float(b[h0 * ldb + col]), acc);
  c[row * ldc + col] = acc;
}

// Tiled bf16 x bf16 -> f32 fma GEMM: same chains as gemm_bf16_fma_kernel (one
// fmaf per k in increasing order from +0, bf16 widened exactly), with a CTA of
// 128 threads owning a (8*MR) x (16*NR) tile, each thread MR x NR chains, and
// 32-deep k-slices of A and B in a 3-stage cp.async shared-memory ring (rows
// must be 16-byte aligned: K, N and both row strides multiples of 8).
constexpr int FKC = 32, FAP = FKC + 8, FST = 3;

__device__ __forceinline__ void cp_async16_t(void *smem_dst, const void *gsrc) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem_dst)), "l"(gsrc)
               : "memory");
}

template <int MR, int NR>
__global__ void __launch_bounds__(128) gemm_bf16_fma_tiled_kernel(
    const __nv_bfloat16 *__restrict__ a, const __nv_bfloat16 *__restrict__ b,
    float *__restrict__ c, int64_t m, int64_t n, int64_t k, int64_t lda, int64_t ldb,
    int64_t ldc) {
  constexpr int TX = 16, TY = 8, TM = TY * MR, TN = TX * NR, NT = TX * TY;
  __shared__ __align__(16) __nv_bfloat16 as[FST][TM][FAP];
  __shared__ __align__(16) __nv_bfloat16 bs[FST][FKC][TN];
  const int tid = threadIdx.x, tx = tid % TX, ty = tid / TX;
  const int64_t row0 = static_cast<int64_t>(blockIdx.y) * TM;
  const int64_t col0 = static_cast<int64_t>(blockIdx.x) * TN;
  const int mrows = static_cast<int>(m - row0 < TM ? m - row0 : TM);
  const int ncols = static_cast<int>(n - col0 < TN ? n - col0 : TN);
  auto stage = [&](int64_t ci, int buf) {
    const int64_t h0 = ci * FKC;
    const int nr = static_cast<int>(k - h0 < FKC ? k - h0 : FKC);
    const int av = nr >> 3, bv = ncols >> 3;  // 8 bf16 per 16-byte copy
    for (int i = tid; i < mrows * av; i += NT) {
      const int r = i / av, q = (i - r * av) * 8;
      cp_async16_t(&as[buf][r][q], a + (row0 + r) * lda + h0 + q);
    }
    for (int i = tid; i < nr * bv; i += NT) {
      const int r = i / bv, q = (i - r * bv) * 8;
      cp_async16_t(&bs[buf][r][q], b + (h0 + r) * ldb + col0 + q);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  float acc[MR][NR];
#pragma unroll
  for (int r = 0; r < MR; ++r)
#pragma unroll
    for (int j = 0; j < NR; ++j) acc[r][j] = 0.0f;
  const int64_t nch = (k + FKC - 1) / FKC;
#pragma unroll
  for (int st = 0; st < FST - 1; ++st) {
    if (st < nch)
      stage(st, st);
    else
      asm volatile("cp.async.commit_group;" ::: "memory");
  }
  for (int64_t ci = 0; ci < nch; ++ci) {
    const int buf = static_cast<int>(ci % FST);
    asm volatile("cp.async.wait_group %0;" ::"n"(FST - 2) : "memory");
    __syncthreads();
    if (ci + FST - 1 < nch)
      stage(ci + FST - 1, static_cast<int>((ci + FST - 1) % FST));
    else
      asm volatile("cp.async.commit_group;" ::: "memory");
    const int nr = static_cast<int>(k - ci * FKC < FKC ? k - ci * FKC : FKC);
    for (int h = 0; h < nr; ++h) {
      float bvv[NR];
#pragma unroll
      for (int j = 0; j < NR; ++j) bvv[j] = __bfloat162float(bs[buf][h][tx * NR + j]);
#pragma unroll
      for (int r = 0; r < MR; ++r) {
        const float av = __bfloat162float(as[buf][ty * MR + r][h]);
#pragma unroll
        for (int j = 0; j < NR; ++j) acc[r][j] = __fmaf_rn(av, bvv[j], acc[r][j]);
      }
    }
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");
#pragma unroll
  for (int r = 0; r < MR; ++r) {
    const int64_t row = row0 + ty * MR + r;
    if (row >= m) continue;
#pragma unroll
    for (int j = 0; j < NR; ++j) {
      const int64_t col = col0 + tx * NR + j;
      if (col < n) c[row * ldc + col] = acc[r][j];
    }
  }
}

// Large-problem bf16 x bf16 -> f32 fma GEMM, same chains (one fmaf per k in
// increasing order from +0 per output, bf16 widened exactly), laid out like an
// SGEMM: 256 threads own a 128x128 tile, each thread 8x8 chains (rows
// 4*ty.. and 64+4*ty.., columns 4*tx.. and 64+4*tx..). 16-deep k-slices of A
// (stored transposed, [k][row]) and B ([k][col]) are widened to f32 once, when
// they are written to shared memory (two buffers; the next slice is fetched
// into registers while the current one is consumed), and read back with four
// 16-byte loads per 64 fmas. A k-slice past K is never multiplied (0*Inf
// would be NaN where the reference has no term): the last slice runs only
// its real depth. Rows must be 16-byte aligned (K, N and both row strides
// multiples of 8).
constexpr int GBM = 128, GBN = 128, GBK = 16, GPAD = 4;

__device__ __forceinline__ void bf16x8_to_f32(const uint4 v, float (&f)[8]) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}

__global__ void __launch_bounds__(256) gemm_bf16_fma_big_kernel(
    const __nv_bfloat16 *__restrict__ a, const __nv_bfloat16 *__restrict__ b,
    float *__restrict__ c, int64_t m, int64_t n, int64_t k, int64_t lda, int64_t ldb,
    int64_t ldc) {
  __shared__ __align__(16) float as[2][GBK][GBM + GPAD];
  __shared__ __align__(16) float bs[2][GBK][GBN + GPAD];
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const int64_t row0 = static_cast<int64_t>(blockIdx.y) * GBM;
  const int64_t col0 = static_cast<int64_t>(blockIdx.x) * GBN;
  // Staging roles: A row (tid & 127), k-half (tid >> 7); B k-row (tid >> 4),
  // 8-column group (tid & 15). One 16-byte global load each per slice.
  const int a_r = tid & 127, a_kh = (tid >> 7) * 8;
  const int b_k = tid >> 4, b_c = (tid & 15) * 8;
  const int64_t nslices = (k + GBK - 1) / GBK;
  uint4 ra = make_uint4(0, 0, 0, 0), rb = make_uint4(0, 0, 0, 0);
  auto fetch = [&](int64_t sl) {
    const int64_t h0 = sl * GBK;
    const int64_t ar = row0 + a_r, ak = h0 + a_kh;
    ra = (ar < m && ak < k) ? *reinterpret_cast<const uint4 *>(a + ar * lda + ak)
                            : make_uint4(0, 0, 0, 0);
    const int64_t bk = h0 + b_k, bc = col0 + b_c;
    rb = (bk < k && bc < n) ? *reinterpret_cast<const uint4 *>(b + bk * ldb + bc)
                            : make_uint4(0, 0, 0, 0);
  };
  auto stage = [&](int buf) {
    float f[8];
    bf16x8_to_f32(ra, f);
#pragma unroll
    for (int i = 0; i < 8; ++i) as[buf][a_kh + i][a_r] = f[i];
    bf16x8_to_f32(rb, f);
    *reinterpret_cast<float4 *>(&bs[buf][b_k][b_c]) = make_float4(f[0], f[1], f[2], f[3]);
    *reinterpret_cast<float4 *>(&bs[buf][b_k][b_c + 4]) = make_float4(f[4], f[5], f[6], f[7]);
  };
  float acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.0f;
  if (nslices > 0) {
    fetch(0);
    stage(0);
  }
  __syncthreads();
  for (int64_t sl = 0; sl < nslices; ++sl) {
    const int buf = static_cast<int>(sl & 1);
    if (sl + 1 < nslices) fetch(sl + 1);
    const int depth = static_cast<int>(k - sl * GBK < GBK ? k - sl * GBK : GBK);
    auto step = [&](int kk) {
      const float4 a0 = *reinterpret_cast<const float4 *>(&as[buf][kk][ty * 4]);
      const float4 a1 = *reinterpret_cast<const float4 *>(&as[buf][kk][64 + ty * 4]);
      const float4 b0 = *reinterpret_cast<const float4 *>(&bs[buf][kk][tx * 4]);
      const float4 b1 = *reinterpret_cast<const float4 *>(&bs[buf][kk][64 + tx * 4]);
      const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
      const float bv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = __fmaf_rn(av[i], bv[j], acc[i][j]);
    };
    if (depth == GBK) {
#pragma unroll
      for (int kk = 0; kk < GBK; ++kk) step(kk);
    } else {
      for (int kk = 0; kk < depth; ++kk) step(kk);
    }
    if (sl + 1 < nslices) stage(buf ^ 1);
    __syncthreads();
  }
  const bool vec_out = (ldc & 3) == 0 && (reinterpret_cast<uintptr_t>(c) & 15u) == 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int64_t r = row0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + (i - 4));
    if (r >= m) continue;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int64_t cc = col0 + h * 64 + tx * 4;
      float *dst = c + r * ldc + cc;
      if (vec_out && cc + 4 <= n) {
        *reinterpret_cast<float4 *>(dst) =
            make_float4(acc[i][h * 4], acc[i][h * 4 + 1], acc[i][h * 4 + 2], acc[i][h * 4 + 3]);
      } else {
#pragma unroll
        for (int j = 0; j < 4; ++j)
          if (cc + j < n) dst[j] = acc[i][h * 4 + j];
      }
    }
  }
}

template <int MR, int NR>
cudaError_t launch_bf16_fma_tiled(const void *a, const void *b, float *c, int64_t m, int64_t n,
                                  int64_t k, int64_t lda, int64_t ldb, int64_t ldc,
                                  cudaStream_t stream) {
  constexpr int TM = 8 * MR, TN = 16 * NR;
  const int64_t gy = (m + TM - 1) / TM, gx = (n + TN - 1) / TN;
  if (gy > 65535 || gx > 0x7fffffff) return cudaErrorInvalidConfiguration;
  gemm_bf16_fma_tiled_kernel<MR, NR><<<dim3(static_cast<unsigned>(gx), static_cast<unsigned>(gy)),
                                       128, 0, stream>>>(
      static_cast<const __nv_bfloat16 *>(a), static_cast<const __nv_bfloat16 *>(b), c, m, n, k,
      lda, ldb, ldc);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_transpose_u8(const void *in, void *out, int64_t rows, int64_t cols,
                                int64_t ld_in, cudaStream_t stream) {
  if (rows == 0 || cols == 0) return cudaSuccess;
  const bool v16 = rows % 16 == 0 && cols % 16 == 0 && ld_in % 16 == 0 &&
                   ((reinterpret_cast<uintptr_t>(in) | reinterpret_cast<uintptr_t>(out)) & 15u) == 0;
  if (v16) {
    const dim3 g16(static_cast<unsigned>((cols + 63) / 64), static_cast<unsigned>((rows + 63) / 64));
    if (g16.y > 65535u) return cudaErrorInvalidConfiguration;
    transpose_u8_v16_kernel<<<g16, 256, 0, stream>>>(static_cast<const uint8_t *>(in),
                                                    static_cast<uint8_t *>(out), rows, cols, ld_in);
    return cudaGetLastError();
  }
  dim3 grid(static_cast<unsigned>((cols + 31) / 32), static_cast<unsigned>((rows + 31) / 32));
  if (grid.y > 65535u) return cudaErrorInvalidConfiguration;
  transpose_u8_kernel<<<grid, dim3(32, 8), 0, stream>>>(static_cast<const uint8_t *>(in),
                                                        static_cast<uint8_t *>(out), rows, cols,
                                                        ld_in);
  return cudaGetLastError();
}

cudaError_t launch_i8_zero_point_sums(const int8_t *a, int64_t lda, const int8_t *b, int64_t ldb,
                                      int b_mn, int64_t m, int64_t n, int64_t k,
                                      const I8ZeroPoints &zp, int32_t *row_sum, int32_t *col_sum,
                                      int sms, cudaStream_t stream, LaunchInfo *info) {
  auto row_sums = [&](const int8_t *x, int64_t rows, int64_t ld, int32_t *out) -> cudaError_t {
    const int64_t blocks = (rows + 7) / 8;
    if (blocks > 0x7fffffff) return cudaErrorInvalidConfiguration;
    i8_row_sums_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(x, rows, k, ld, out);
    if (info) info->launches += 1;
    return cudaGetLastError();
  };
  cudaError_t e = cudaSuccess;
  if (zp.zb != 0 && m > 0 && (e = row_sums(a, m, lda, row_sum)) != cudaSuccess) return e;
  if (zp.za != 0 && n > 0) {
    if (!b_mn) return row_sums(b, n, ldb, col_sum);  // Bt [N,K]: its row sums
    if ((e = cudaMemsetAsync(col_sum, 0, static_cast<size_t>(n) * 4, stream)) != cudaSuccess)
      return e;
    // About two CTAs per SM: split K so the column groups x slices fill
    // them, each warp reading at least 8 rows.
    const int64_t gx = (n + CS_COLS - 1) / CS_COLS;
    int64_t slices = (2 * static_cast<int64_t>(sms) + gx - 1) / gx;
    if (slices > (k + 63) / 64) slices = (k + 63) / 64;
    if (slices < 1) slices = 1;
    if (slices > 65535) slices = 65535;
    const int64_t k_slice = (k + slices - 1) / slices;
    slices = (k + k_slice - 1) / k_slice;
    if (gx > 0x7fffffff) return cudaErrorInvalidConfiguration;
    if (k > 0) {
      i8_col_sums_kernel<<<dim3(static_cast<unsigned>(gx), static_cast<unsigned>(slices)), 256, 0,
                           stream>>>(b, k, n, ldb, k_slice, col_sum);
      if (info) info->launches += 1;
      e = cudaGetLastError();
    }
  }
  return e;
}

cudaError_t launch_gemm_i8_tc(const int8_t *a, int64_t lda, const int8_t *b, int64_t ldb,
                              int b_mn, int32_t *c, int64_t m, int64_t n, int64_t k, int64_t ld_c,
                              const I8ZeroPoints *zp, uint32_t *status, int sms,
                              cudaStream_t stream, LaunchInfo *info) {
  if (m == 0 || n == 0) return cudaSuccess;
  // TMA needs 16-byte aligned bases and row strides; the epilogue's vector
  // stores need a 16-byte aligned C. K tails are zero-filled by TMA.
  if (k == 0 || lda % 16 != 0 || ldb % 16 != 0 ||
      ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b) |
        reinterpret_cast<uintptr_t>(c)) & 15u) != 0)
    return cudaErrorNotSupported;
  int device = 0;
  cudaError_t e = cudaGetDevice(&device);
  if (e != cudaSuccess) return e;
  static const bool pair_on = [] {
    const char *v = getenv("MCB_GEMM_TC_PAIR");
    return !(v && v[0] == '0');
  }();
  const bool pair = m >= 2 * BM && pair_on && i8_pair_clusters_resident(device) > 0;
  // B box per CTA: MN-major 128 columns x BK rows; K-major BK bytes x (BN or
  // BN/2) rows.
  const int bt_rows = pair ? P_B_COLS : BN;
  CUtensorMap ta, tb;
  if (!encode_tmap_2d(&ta, CU_TENSOR_MAP_DATA_TYPE_UINT8, a, k, m, lda, BK, BM,
                      CU_TENSOR_MAP_SWIZZLE_128B))
    return cudaErrorNotSupported;
  const bool ok_b = b_mn ? encode_tmap_2d(&tb, CU_TENSOR_MAP_DATA_TYPE_UINT8, b, n, k, ldb,
                                          MN_CHUNK, BK, CU_TENSOR_MAP_SWIZZLE_128B)
                         : encode_tmap_2d(&tb, CU_TENSOR_MAP_DATA_TYPE_UINT8, b, k, n, ldb, BK,
                                          bt_rows, CU_TENSOR_MAP_SWIZZLE_128B);
  if (!ok_b) return cudaErrorNotSupported;
  Params p;
  p.m = m;
  p.n = n;
  p.ld_c = ld_c;
  p.n_tiles = static_cast<int>((n + BN - 1) / BN);
  const int64_t tile_rows = pair ? 2 * BM : BM;
  const int64_t tiles = ((m + tile_rows - 1) / tile_rows) * p.n_tiles;
  if (tiles > 0x7fffffff) return cudaErrorNotSupported;
  p.num_tiles = static_cast<int>(tiles);
  p.num_kb = static_cast<int>((k + BK - 1) / BK);
  p.b_mn = b_mn;
  p.zp = zp && (zp->za != 0 || zp->zb != 0) ? 1 : 0;
  p.za = zp ? static_cast<uint32_t>(zp->za) : 0u;
  p.zb = zp ? static_cast<uint32_t>(zp->zb) : 0u;
  p.kzz = static_cast<uint32_t>(static_cast<uint64_t>(k)) * p.za * p.zb;
  p.row_sum = zp && zp->zb != 0 ? zp->row_sum : nullptr;
  p.col_sum = zp && zp->za != 0 ? zp->col_sum : nullptr;
  if (p.zp && ((p.zb != 0 && !p.row_sum) || (p.za != 0 && !p.col_sum) ||
               (reinterpret_cast<uintptr_t>(p.col_sum) & 15u) != 0))
    return cudaErrorInvalidValue;
  p.c = c;
  p.status = status;
  int grid;
  if (pair) {
    int clusters = i8_pair_clusters_resident(device);
    if (clusters > sms / 2) clusters = sms / 2;
    if (clusters < 1) clusters = 1;
    grid = 2 * static_cast<int>(tiles < clusters ? tiles : clusters);
    gemm_i8_pair_kernel<<<grid, P_THREADS, P_SMEM_BYTES, stream>>>(ta, tb, p);
  } else {
    e = cudaFuncSetAttribute(gemm_i8_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(SMEM_BYTES));
    if (e != cudaSuccess) return e;
    grid = static_cast<int>(tiles < sms ? tiles : sms);
    gemm_i8_kernel<<<grid, THREADS, SMEM_BYTES, stream>>>(ta, tb, p);
  }
  if (info) {
    info->launches += 1;
    info->tile_m = static_cast<int>(tile_rows);
    info->tile_n = BN;
    info->tile_k = BK;
    info->stages = pair ? P_STAGES : STAGES;
    info->ctas = grid;
    info->set_route("tcgen05_i8_gemm");
  }
  return cudaGetLastError();
}

cudaError_t launch_gemm_i8_simt(const int8_t *a, const int8_t *b, int32_t *c, int64_t m, int64_t n,
                                int64_t k, int64_t lda, int64_t ldb, int64_t ldc, int32_t za,
                                int32_t zb, cudaStream_t stream, LaunchInfo *info) {
  if (m == 0 || n == 0) return cudaSuccess;
  if (m > 65535) return cudaErrorInvalidConfiguration;
  dim3 grid(static_cast<unsigned>((n + 255) / 256), static_cast<unsigned>(m));
  gemm_i8_simt_kernel<<<grid, 256, 0, stream>>>(a, b, c, m, n, k, lda, ldb, ldc,
                                                static_cast<uint32_t>(za),
                                                static_cast<uint32_t>(zb));
  if (info) {
    info->launches += 1;
    info->set_route("simt_i8_gemm");
  }
  return cudaGetLastError();
}

cudaError_t launch_gemm_bf16_fma(const void *a, const void *b, float *c, int64_t m, int64_t n,
                                 int64_t k, int64_t lda, int64_t ldb, int64_t ldc,
                                 cudaStream_t stream, LaunchInfo *info) {
  if (m == 0 || n == 0) return cudaSuccess;
  const bool vec = k % 8 == 0 && n % 8 == 0 && lda % 8 == 0 && ldb % 8 == 0 &&
                   (k == 0 || ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b)) &
                               15u) == 0);
  if (vec) {
    // 128x128 tiles once they fill the GPU; otherwise the per-thread block
    // shrinks until a launch has ~2 warps per SM sub-partition.
    const int64_t outputs = m * n;
    const int64_t big_tiles = ((m + GBM - 1) / GBM) * ((n + GBN - 1) / GBN);
    cudaError_t e;
    const char *route;
    if (big_tiles >= 148 && (m + GBM - 1) / GBM <= 65535) {
      gemm_bf16_fma_big_kernel<<<dim3(static_cast<unsigned>((n + GBN - 1) / GBN),
                                      static_cast<unsigned>((m + GBM - 1) / GBM)),
                                 256, 0, stream>>>(static_cast<const __nv_bfloat16 *>(a),
                                                   static_cast<const __nv_bfloat16 *>(b), c, m,
                                                   n, k, lda, ldb, ldc);
      e = cudaGetLastError();
      route = "simt_bf16_f32_fma_gemm_128x128";
    } else if (outputs / 8 >= 148LL * 4 * 2 * 32 && n >= 64) {
      e = launch_bf16_fma_tiled<2, 4>(a, b, c, m, n, k, lda, ldb, ldc, stream);
      route = "simt_bf16_f32_fma_gemm_tiled";
    } else {
      e = launch_bf16_fma_tiled<1, 2>(a, b, c, m, n, k, lda, ldb, ldc, stream);
      route = "simt_bf16_f32_fma_gemm_tiled";
    }
    if (e != cudaErrorInvalidConfiguration) {
      if (info) {
        info->launches = 1;
        info->set_route(route);
      }
      return e;
    }
  }
  if (m > 65535) return cudaErrorInvalidConfiguration;
  dim3 grid(static_cast<unsigned>((n + 255) / 256), static_cast<unsigned>(m));
  gemm_bf16_fma_kernel<<<grid, 256, 0, stream>>>(static_cast<const __nv_bfloat16 *>(a),
                                                 static_cast<const __nv_bfloat16 *>(b), c, m, n, k,
                                                 lda, ldb, ldc);
  if (info) {
    info->launches = 1;
    info->set_route("simt_bf16_f32_fma_gemm");
  }
  return cudaGetLastError();
}

}  // namespace mcb

// Family B chain on tcgen05 tensor cores with the intermediate kept on chip:
//
//   E[M,N2] = glue(A[M,K] * B[K,N1]) * W[N1,N2]      (src/fusion_emitter_family_b.cpp)
//
// where glue is a Family A epilogue on the intermediate (row bias or [M,N1]
// boundary, added or reverse-subtracted, then one activation). bf16 operands,
// f32 accumulation, E bf16 or f32.
//
// One work unit = 128 rows of A and one tile of up to 256 columns of E.
// Persistent CTAs (one per SM, 352 threads) loop over units:
//   warp 0      TMA producer of GEMM 1: for every 128-column chunk j of the
//               intermediate, K blocks of A (128x64, K-major) and B (64x128,
//               consumed MN-major from the row-major [K,N1] matrix) into a
//               3-stage ring.
//   warp 10     TMA producer of W: rows [128j, 128j+128) x the unit's E
//               columns, as 64-column chunks (MN-major B operand of GEMM 2).
//   warp 1      TMEM owner (S0 | S1 | E) and the single MMA issuer:
//               S_j = A B_j (M=128, N=128) into S[j%2]; after S_j, the
//               GEMM 2 step E += P_{j-1} W_{j-1} (M=128, N=E columns, K=128)
//               for the previous chunk, so the glue of chunk j-1 overlaps the
//               MMAs of chunk j.
//   warps 2-9   glue: two threads own row r (its TMEM lane), 64 columns
//               each. They read their intermediate values of S_j, applies the glue in f32 (values
//               past N1 or M become 0), writes them as bf16 P_j in the
//               128-byte-swizzled K-major layout GEMM 2 reads, and signals
//               the MMA warp. At the end of a unit the same threads read E
//               from TMEM and store it.
// The intermediate never reaches HBM: it lives in TMEM (f32) and shared
// memory (bf16, as GEMM 2's operand), one 128x128 chunk at a time.
//
// Roofline: 2*M*K*N1 + 2*M*N1*N2 FLOP against the bf16 dense tensor peak;
// GEMM 1 is recomputed for every 256-column tile of E beyond the first.
#include <cuda_bf16.h>

#include "common.cuh"
#include "epilogue.cuh"
#include "internal.h"

namespace mcb {
namespace {

constexpr int CM = 128;        // rows per unit
constexpr int CN1 = 128;       // intermediate columns per chunk (GEMM 1 N, GEMM 2 K)
constexpr int CK = 64;         // GEMM 1 K block
constexpr int CSTAGES = 3;
constexpr int A_BYTES = CM * CK * 2;         // 16 KiB
constexpr int B_BYTES = CK * CN1 * 2;        // 16 KiB: two 64-column chunks of 64 rows
constexpr int B_CHUNK_BYTES = CK * 64 * 2;   // 8 KiB
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int MAX_N2T = 256;                 // E columns per unit
constexpr int W_CHUNK_BYTES = CN1 * 64 * 2;  // 16 KiB: 128 rows x 64 columns of W
constexpr int W_BYTES = MAX_N2T / 64 * W_CHUNK_BYTES;
constexpr int P_CHUNK_BYTES = CM * 64 * 2;   // 16 KiB: 128 rows x 64 intermediate columns
constexpr int P_BYTES = 2 * P_CHUNK_BYTES;
constexpr int GLUE_THREADS = 256;  // 8 glue warps: two per TMEM lane quarter, 64 columns each
constexpr int THREADS = 64 + GLUE_THREADS + 32;  // + producer, MMA, W producer
constexpr uint32_t S_COL = 0, E_COL = 256;
constexpr int TMEM_COLS = 512;

struct Smem {
  uint8_t ab[CSTAGES][STAGE_BYTES];
  uint8_t w[W_BYTES];
  uint8_t p[P_BYTES];
  uint64_t full[CSTAGES], empty[CSTAGES];
  uint64_t s_full[2], s_free[2];
  uint64_t p_full, p_free;
  uint64_t w_full, w_empty;
  uint64_t e_full, e_empty;
  uint64_t drain;
  uint32_t tmem_slot;
  int abort_flag;
  float bias[2][CN1];  // a chunk's row bias in f32 (two buffers, alternating chunks)
  alignas(16) float bias_row[4096];  // the whole row bias when N1 <= 4096, staged once
};
constexpr int kBiasRowMax = 4096;
constexpr size_t SMEM_BYTES = sizeof(Smem) + 1024;

struct Params {
  int64_t m, k, n1, n2, ld_e;
  int n2_tiles, n2t, num_kb, n1_chunks;
  int64_t units;
  int e_kind;  // kOutF32 / kOutBf16
  void *e;
  uint32_t *status;
  Epilogue glue;
};

__global__ void __launch_bounds__(THREADS, 1)
    chain_tc_bf16_kernel(const __grid_constant__ CUtensorMap ta,
                         const __grid_constant__ CUtensorMap tb,
                         const __grid_constant__ CUtensorMap tw, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  Smem &sm = *reinterpret_cast<Smem *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  volatile int *abort_flag = &sm.abort_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < CSTAGES; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&sm.s_full[s], 1);
      mbar_init(&sm.s_free[s], GLUE_THREADS);
    }
    mbar_init(&sm.p_full, GLUE_THREADS);
    mbar_init(&sm.p_free, 1);
    mbar_init(&sm.w_full, 1);
    mbar_init(&sm.w_empty, 1);
    mbar_init(&sm.e_full, 1);
    mbar_init(&sm.e_empty, GLUE_THREADS);
    mbar_init(&sm.drain, 1);
    sm.abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&ta);
    tma_prefetch_desc(&tb);
    tma_prefetch_desc(&tw);
  }
  if (warp == 1) {
    tmem_alloc(&sm.tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_slot;
  const int nch = p.n1_chunks;

  if (warp == 0) {
    // ---------------- GEMM 1 producer ----------------
    if (lane == 0) {
      uint32_t it = 0;
      bool ok = true;
      for (int64_t u = blockIdx.x; u < p.units && ok; u += gridDim.x) {
        const int m0 = static_cast<int>(u / p.n2_tiles) * CM;
        for (int j = 0; j < nch && ok; ++j) {
          for (int kb = 0; kb < p.num_kb; ++kb, ++it) {
            const int s = it % CSTAGES;
            if (!(ok = mbar_wait(&sm.empty[s], ((it / CSTAGES) & 1) ^ 1, abort_flag, p.status,
                                 kErrTimeoutEmpty)))
              break;
            mbar_arrive_expect_tx(&sm.full[s], STAGE_BYTES);
            tma_load_2d(sm.ab[s], &ta, &sm.full[s], kb * CK, m0);
            tma_load_2d(sm.ab[s] + A_BYTES, &tb, &sm.full[s], j * CN1, kb * CK);
            tma_load_2d(sm.ab[s] + A_BYTES + B_CHUNK_BYTES, &tb, &sm.full[s], j * CN1 + 64,
                        kb * CK);
          }
        }
      }
    }
  } else if (warp == 2 + GLUE_THREADS / 32) {
    // ---------------- W producer ----------------
    if (lane == 0) {
      uint32_t wt = 0;
      const int wchunks = p.n2t / 64;
      bool ok = true;
      for (int64_t u = blockIdx.x; u < p.units && ok; u += gridDim.x) {
        const int n0 = static_cast<int>(u % p.n2_tiles) * p.n2t;
        for (int j = 0; j < nch; ++j, ++wt) {
          if (!(ok = mbar_wait(&sm.w_empty, (wt & 1) ^ 1, abort_flag, p.status,
                               kErrTimeoutEmpty)))
            break;
          mbar_arrive_expect_tx(&sm.w_full, wchunks * W_CHUNK_BYTES);
          for (int c = 0; c < wchunks; ++c)
            tma_load_2d(sm.w + c * W_CHUNK_BYTES, &tw, &sm.w_full, n0 + c * 64, j * CN1);
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      // S: A K-major, B MN-major (B [K,N1] row-major). E: P K-major, W MN-major.
      const uint32_t idesc_s = make_idesc(1, 1, 0, 1, CM, CN1);
      const uint32_t idesc_e = make_idesc(1, 1, 0, 1, CM, p.n2t);
      const uint32_t p_addr = smem_u32(sm.p), w_addr = smem_u32(sm.w);
      uint32_t it = 0, st = 0, pt = 0, uc = 0;
      bool ok = true;
      for (int64_t u = blockIdx.x; u < p.units && ok; u += gridDim.x, ++uc) {
        for (int j = 0; j <= nch && ok; ++j) {
          if (j < nch) {
            const int sb = st & 1;
            if (!(ok = mbar_wait(&sm.s_free[sb], ((st >> 1) & 1) ^ 1, abort_flag, p.status,
                                 kErrTimeoutAccum)))
              break;
            tc_fence_after();
            const uint32_t d = tmem + S_COL + sb * CN1;
            for (int kb = 0; kb < p.num_kb; ++kb, ++it) {
              const int s = it % CSTAGES;
              if (!(ok = mbar_wait(&sm.full[s], (it / CSTAGES) & 1, abort_flag, p.status,
                                   kErrTimeoutFull)))
                break;
              tc_fence_after();
              const uint32_t a_addr = smem_u32(sm.ab[s]), b_addr = a_addr + A_BYTES;
#pragma unroll
              for (int kk = 0; kk < CK / 16; ++kk)
                mma_f16_ss(d, make_sdesc_sw128(a_addr + kk * 32, 16, 1024),
                           make_sdesc_sw128(b_addr + kk * 2048, B_CHUNK_BYTES, 1024), idesc_s,
                           (kb | kk) ? 1u : 0u);
              mma_commit(&sm.empty[s]);
            }
            if (!ok) break;
            mma_commit(&sm.s_full[sb]);
            ++st;
          }
          if (j >= 1) {
            // GEMM 2 step for chunk j-1: E += P_{j-1} W_{j-1}.
            if (j == 1 && !(ok = mbar_wait(&sm.e_empty, (uc & 1) ^ 1, abort_flag, p.status,
                                           kErrTimeoutAccum)))
              break;
            if (!(ok = mbar_wait(&sm.w_full, pt & 1, abort_flag, p.status, kErrTimeoutFull)))
              break;
            if (!(ok = mbar_wait(&sm.p_full, pt & 1, abort_flag, p.status, kErrTimeoutAccum)))
              break;
            tc_fence_after();
#pragma unroll
            for (int kk = 0; kk < CN1 / 16; ++kk)
              mma_f16_ss(tmem + E_COL,
                         make_sdesc_sw128(p_addr + (kk >> 2) * P_CHUNK_BYTES + (kk & 3) * 32, 16,
                                          1024),
                         make_sdesc_sw128(w_addr + kk * 2048, W_CHUNK_BYTES, 1024), idesc_e,
                         ((j - 1) | kk) ? 1u : 0u);
            mma_commit(&sm.p_free);
            mma_commit(&sm.w_empty);
            ++pt;
          }
        }
        if (!ok) break;
        mma_commit(&sm.e_full);
      }
      mma_commit(&sm.drain);
      if (!mbar_wait(&sm.drain, 0, nullptr, p.status, kErrTimeoutDrain)) *abort_flag = 1;
    }
  } else {
    // ---------------- glue (warps 2-9) and output ----------------
    const int sub = warp & 3;
    const int half = (warp - 2) >> 2;  // this warp's 64 columns of each chunk
    const int r_local = sub * 32 + lane;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(sub * 32) << 16);
    uint8_t *p_row = sm.p + r_local * 128;
    const int rsw = r_local & 7;
    uint32_t sc = 0, pc = 0, uc = 0;
    bool ok = true;
    // A row bias of at most kBiasRowMax columns is the same for every unit:
    // staged once, so no chunk waits for a global load and a barrier.
    const bool bias_whole = p.glue.bias_mode == 1 && p.n1 <= kBiasRowMax;
    if (bias_whole) {
      for (int64_t i = threadIdx.x - 64; i < p.n1; i += GLUE_THREADS)
        sm.bias_row[i] = load_bias(p.glue, 0, i);
      named_bar_sync(1, GLUE_THREADS);
    }
    for (int64_t u = blockIdx.x; u < p.units && ok; u += gridDim.x, ++uc) {
      const int64_t row = (u / p.n2_tiles) * CM + r_local;
      const int64_t n0 = (u % p.n2_tiles) * p.n2t;
      for (int j = 0; j < nch; ++j) {
        const int sb = sc & 1;
        if (!(ok = mbar_wait_warp(&sm.s_full[sb], (sc >> 1) & 1, abort_flag, p.status,
                                  kErrTimeoutAccum)))
          break;
        tc_fence_after();
        // Glue in f32, 32 columns at a time straight from TMEM, each group
        // written as bf16 into P at once; columns past N1 and rows past M
        // give 0 (their A, B and W entries were zero-filled, and the boundary
        // has nothing there). The group loop is kept rolled and the
        // activation switch sits outside the element loops: the fully
        // unrolled form overflowed the instruction cache (ncu: stalls on
        // instruction fetch and branch resolution, 35 us per chunk).
        const int64_t col0 = static_cast<int64_t>(j) * CN1;
        const Epilogue &g = p.glue;
        // Consecutive chunks (also across units) alternate bias buffers, so
        // the barrier of chunk c+1 orders chunk c's reads before chunk c+2's
        // writes into the same buffer.
        const float *bs = bias_whole ? sm.bias_row + col0 : sm.bias[sb];
        if (g.bias_mode == 1 && !bias_whole) {
          // Row bias: thread r stages column col0 + r of this chunk; the four
          // glue warps then read the staged chunk (broadcast).
          if (half == 0)
            sm.bias[sb][r_local] = col0 + r_local < p.n1 ? load_bias(g, 0, col0 + r_local) : 0.0f;
          named_bar_sync(1, GLUE_THREADS);
        }
        const bool row_ok = row < p.m;
        const int64_t bbase = row * g.ld_bias + col0;
        const bool full_vec = g.bias_mode == 2 && row_ok && col0 + CN1 <= p.n1 &&
                              ((reinterpret_cast<uintptr_t>(g.bias) +
                                bbase * (g.bias_bf16 ? 2 : 4)) & 15u) == 0;
        const uint32_t s_addr = lane_base + S_COL + sb * CN1;
        bool p_ready = false;
#pragma unroll 1
        for (int grp = 2 * half; grp < 2 * half + 2; ++grp) {
          uint32_t r[32];
          tmem_ld32_sync(s_addr + grp * 32, r);
          float v[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
          const int64_t cg = col0 + grp * 32;  // first column of the group
          if (g.bias_mode == 1) {
            const float4 *b4 = reinterpret_cast<const float4 *>(bs + grp * 32);
#pragma unroll
            for (int q = 0; q < 8; ++q) {
              const float4 f = b4[q];
              const float bq[4] = {f.x, f.y, f.z, f.w};
#pragma unroll
              for (int h = 0; h < 4; ++h)
                v[4 * q + h] = g.bias_op == 1 ? bq[h] - v[4 * q + h] : v[4 * q + h] + bq[h];
            }
          } else if (full_vec && g.bias_bf16) {
            const uint4 *src = reinterpret_cast<const uint4 *>(
                reinterpret_cast<const __nv_bfloat16 *>(g.bias) + bbase + grp * 32);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const uint4 w4 = __ldg(src + q);
              const uint32_t ws[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
              for (int h = 0; h < 4; ++h) {
                const float b0 = __uint_as_float(ws[h] << 16);
                const float b1 = __uint_as_float(ws[h] & 0xffff0000u);
                float &x0 = v[q * 8 + 2 * h], &x1 = v[q * 8 + 2 * h + 1];
                x0 = g.bias_op == 1 ? b0 - x0 : x0 + b0;
                x1 = g.bias_op == 1 ? b1 - x1 : x1 + b1;
              }
            }
          } else if (full_vec) {
            const float4 *src = reinterpret_cast<const float4 *>(
                reinterpret_cast<const float *>(g.bias) + bbase + grp * 32);
#pragma unroll
            for (int q = 0; q < 8; ++q) {
              const float4 f = __ldg(src + q);
              const float bq[4] = {f.x, f.y, f.z, f.w};
#pragma unroll
              for (int h = 0; h < 4; ++h)
                v[4 * q + h] = g.bias_op == 1 ? bq[h] - v[4 * q + h] : v[4 * q + h] + bq[h];
            }
          } else if (g.bias_mode == 2 && row_ok) {
            for (int i = 0; i < 32; ++i)
              if (cg + i < p.n1) {
                const float bq = load_bias(g, row, cg + i);
                v[i] = g.bias_op == 1 ? bq - v[i] : v[i] + bq;
              }
          }
          switch (g.act) {
            case 0: break;
            case 1:
#pragma unroll
              for (int i = 0; i < 32; ++i) v[i] = fmaxf(v[i], 0.0f);
              break;
            case 2:
#pragma unroll
              for (int i = 0; i < 32; ++i) v[i] = apply_act<true>(v[i], 2);
              break;
            case 3:
#pragma unroll
              for (int i = 0; i < 32; ++i) v[i] = apply_act<true>(v[i], 3);
              break;
            case 4:
#pragma unroll
              for (int i = 0; i < 32; ++i) v[i] = apply_act<true>(v[i], 4);
              break;
            default:
#pragma unroll
              for (int i = 0; i < 32; ++i) v[i] = apply_act<true>(v[i], 5);
              break;
          }
          if (!row_ok) {
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] = 0.0f;
          } else if (cg + 32 > p.n1) {
#pragma unroll
            for (int i = 0; i < 32; ++i)
              if (cg + i >= p.n1) v[i] = 0.0f;
          }
          // P is free once GEMM 2 of the previous chunk has read it: waited
          // for only now, so the first group's loads and math overlap it.
          if (!p_ready) {
            if (!(ok = mbar_wait_warp(&sm.p_free, (pc & 1) ^ 1, abort_flag, p.status,
                                      kErrTimeoutAccum)))
              break;
            p_ready = true;
          }
          // 32 columns = 4 granules of 16 bytes of this row of P.
          uint8_t *pc_base = p_row + (grp >> 1) * P_CHUNK_BYTES;
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int jj = (grp & 1) * 4 + q;
            *reinterpret_cast<uint4 *>(pc_base + ((jj ^ rsw) << 4)) =
                make_uint4(pack_bf16x2(v[8 * q], v[8 * q + 1]), pack_bf16x2(v[8 * q + 2], v[8 * q + 3]),
                           pack_bf16x2(v[8 * q + 4], v[8 * q + 5]),
                           pack_bf16x2(v[8 * q + 6], v[8 * q + 7]));
          }
        }
        if (!ok) break;
        tc_fence_before();
        mbar_arrive(&sm.s_free[sb]);
        ++sc;
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        mbar_arrive(&sm.p_full);
        ++pc;
      }
      if (!ok) break;
      // ---- output: E row from TMEM ----
      if (!(ok = mbar_wait_warp(&sm.e_full, uc & 1, abort_flag, p.status, kErrTimeoutAccum)))
        break;
      tc_fence_after();
#pragma unroll 1
      for (int c0 = half * (p.n2t / 2); c0 < (half + 1) * (p.n2t / 2); c0 += 32) {
        uint32_t r[32];
        tmem_ld32_sync(lane_base + E_COL + c0, r);
        if (row >= p.m) continue;
        const int64_t col = n0 + c0;
        if (p.e_kind == kOutBf16) {
          __nv_bfloat16 *er = reinterpret_cast<__nv_bfloat16 *>(p.e) + row * p.ld_e + col;
          for (int i = 0; i < 32; ++i)
            if (col + i < p.n2) er[i] = __float2bfloat16_rn(__uint_as_float(r[i]));
        } else {
          float *er = reinterpret_cast<float *>(p.e) + row * p.ld_e + col;
          for (int i = 0; i < 32; ++i)
            if (col + i < p.n2) er[i] = __uint_as_float(r[i]);
        }
      }
      tc_fence_before();
      mbar_arrive(&sm.e_empty);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

}  // namespace

cudaError_t launch_chain_tc_bf16(const void *a, const void *b, const void *w, void *e, int64_t m,
                                 int64_t k, int64_t n1, int64_t n2, int64_t lda, int64_t ldb,
                                 int64_t ldw, int64_t lde, int e_kind, const Epilogue &glue,
                                 uint32_t *status, int sms, cudaStream_t stream,
                                 LaunchInfo *info) {
  if (m == 0 || n2 == 0) return cudaSuccess;
  if (k <= 0 || n1 <= 0 || glue.n_ops != 0) return cudaErrorNotSupported;
  CUtensorMap ta, tb, tw;
  if (!encode_tmap_2d(&ta, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, a, k, m, lda * 2, CK, CM,
                      CU_TENSOR_MAP_SWIZZLE_128B) ||
      !encode_tmap_2d(&tb, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, b, n1, k, ldb * 2, 64, CK,
                      CU_TENSOR_MAP_SWIZZLE_128B) ||
      !encode_tmap_2d(&tw, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, w, n2, n1, ldw * 2, 64, CN1,
                      CU_TENSOR_MAP_SWIZZLE_128B))
    return cudaErrorNotSupported;
  Params p;
  p.m = m;
  p.k = k;
  p.n1 = n1;
  p.n2 = n2;
  p.ld_e = lde;
  p.n2t = n2 >= MAX_N2T ? MAX_N2T : static_cast<int>((n2 + 63) / 64 * 64);
  p.n2_tiles = static_cast<int>((n2 + p.n2t - 1) / p.n2t);
  p.num_kb = static_cast<int>((k + CK - 1) / CK);
  p.n1_chunks = static_cast<int>((n1 + CN1 - 1) / CN1);
  p.units = ((m + CM - 1) / CM) * p.n2_tiles;
  if (p.units > 0x7fffffff) return cudaErrorNotSupported;
  p.e_kind = e_kind;
  p.e = e;
  p.status = status;
  p.glue = glue;
  cudaError_t err = cudaFuncSetAttribute(chain_tc_bf16_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(SMEM_BYTES));
  if (err != cudaSuccess) return err;
  const int grid = static_cast<int>(p.units < sms ? p.units : sms);
  chain_tc_bf16_kernel<<<grid, THREADS, SMEM_BYTES, stream>>>(ta, tb, tw, p);
  if (info) {
    info->launches = 1;
    info->tile_m = CM;
    info->tile_n = p.n2t;
    info->tile_k = CK;
    info->stages = CSTAGES;
    info->ctas = grid;
    info->set_route("tcgen05_bf16_chain_fused");
  }
  return cudaGetLastError();
}

}  // namespace mcb

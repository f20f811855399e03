// Matmul-softmax-matmul (Family C) on tcgen05 tensor cores, bf16, head dim
// HD = 64 or 128 (Dqk = Dv).
//
//   O[b,h] = softmax(scale * Q[b,h] K[b,h]^T) V[b,h]      (src/fusion_emitter_family_c.cpp)
//
// Two kernels: msm_tc2_bf16_kernel (query blocks of 256 rows, two query
// tiles per CTA; described with the kernel below) and msm_tc_bf16_kernel
// (blocks of 128 rows), whose design is:
//
// One work unit = (b, h, 128-row query block). Persistent CTAs (one per SM,
// 192 threads) loop over units; consecutive units share (b, h) so K/V stay
// in L2 for the CTAs running at the same time.
//
//   warp 0      TMA producer: Q (once per unit), K tiles into a 3-stage ring,
//               V tiles into a 2-stage ring (128 keys x HD dims, stored as
//               HD/64 column chunks of 128 rows x 128 bytes, 128B swizzle).
//   warp 1      TMEM owner (512 columns: S0 | S1 | O) and single-thread MMA
//               issuer: S_t = Q K_t^T (M=128, N=128, K=HD) into S[t%2], then
//               O += P_{t-1} V_{t-1} with P from shared memory and V consumed
//               MN-major. S_{t+1} is issued before PV_t so the tensor core
//               works on the next score tile while the softmax runs.
//   warps 2-5   softmax: thread r owns query row r (its TMEM lane). It loads
//               the 128 scores of its row, takes the row max in registers (no
//               shuffles), computes p = 2^(s*c - m*c) with c = scale*log2(e),
//               accumulates the row sum, writes P (bf16) in the 128B-swizzled
//               K-major layout the MMA reads, and signals the MMA warp.
//               The running max is lazy: O and l are rescaled (in TMEM, by
//               the owning thread) only when a tile's max exceeds the
//               reference max by more than 2^8 in probability, which keeps
//               every p <= 256 and makes rescales rare. At the end of a unit
//               the same threads read O, divide by l and store bf16.
// S and P never touch HBM.
//
// Roofline (config 3, [8,32,4096,128]): 4*B*H*S^2*D = 2.199 TFLOP (exp
// excluded) against the bf16 dense tensor peak; the exponentials
// (B*H*S^2 = 4.3e9 ex2 on the 16/clk/SM special-function units) are a
// co-bound of the same order.
#include <cuda_bf16.h>

#include "common.cuh"
#include "internal.h"

namespace mcb {
namespace {

constexpr int BQ = 128;       // query rows per unit
constexpr int BKV = 128;      // keys per tile
constexpr int KSTAGES = 3, VSTAGES = 2;
constexpr int CHUNK_BYTES = 128 * 128;   // 128 rows x 64 bf16 columns (one swizzle span)
constexpr int P_BYTES = BQ * BKV * 2;    // 32 KiB: the P tile, and O staged for its store
// A Q, K or V tile: 128 rows x HD bf16 columns, HD/64 chunks (16 or 32 KiB).
template <int HD>
constexpr int tile_bytes() {
  return BKV * HD * 2;
}
constexpr int THREADS = 192;  // 6 warps: producer, MMA, 4 softmax (one per TMEM lane quarter)
constexpr int TMEM_COLS = 512;
constexpr uint32_t S_COL0 = 0, O_COL = 256;

template <int HD>
struct Smem {
  uint8_t q[tile_bytes<HD>()];
  uint8_t k[KSTAGES][tile_bytes<HD>()];
  uint8_t v[VSTAGES][tile_bytes<HD>()];
  uint8_t p[P_BYTES];
  uint64_t q_full, q_empty;
  uint64_t k_full[KSTAGES], k_empty[KSTAGES];
  uint64_t v_full[VSTAGES], v_empty[VSTAGES];
  uint64_t s_full[2], s_free[2];
  uint64_t p_full, p_free;
  uint64_t o_full, o_empty;
  uint64_t drain;
  uint32_t tmem_slot;
  int abort_flag;
};
template <int HD>
constexpr size_t smem_bytes() {
  return sizeof(Smem<HD>) + 1024;
}

struct Params {
  int64_t heads, qblocks, nkv_tiles, units;
  int64_t o_s[3];  // output element strides [batch, head, row]
  float c;         // |scale| * log2(e)
  uint32_t s_neg;  // instruction-descriptor bit 13 (negate A) when scale < 0, else 0
  int o_tma;       // two-tile kernel: O leaves through shared memory and a TMA store
  int m_rows;      // query rows: rows of the last query block past it are not stored
  int n_tail;      // keys in the last key tile when N % 128 != 0, else 0
  __nv_bfloat16 *o;
  uint32_t *status;
};

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// TMA store of one 64-column x 128-row box from shared memory (bulk group of
// the issuing thread; commit and waits in common.cuh).
__device__ __forceinline__ void tma_store_4d(const void *tmap, const void *src, int32_t x,
                                             int32_t y, int32_t z, int32_t w) {
  asm volatile(
      "cp.async.bulk.tensor.4d.global.shared::cta.bulk_group [%0, {%2, %3, %4, %5}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(tmap)),
      "r"(smem_u32(src)), "r"(x), "r"(y), "r"(z), "r"(w)
      : "memory");
}

// K-major SW128 descriptor for the K=16 slice `kk` (0..7) of a 128x128 bf16
// tile stored as two 64-column halves of 16 KiB.
__device__ __forceinline__ uint64_t kmajor_desc(uint32_t base, int kk) {
  return make_sdesc_sw128(base + (kk >> 2) * CHUNK_BYTES + (kk & 3) * 32, 16, 1024);
}
// MN-major SW128 descriptor (V as the B operand): K = keys advance 16 rows of
// 128 bytes; the two 64-column halves are LBO = 16 KiB apart.
__device__ __forceinline__ uint64_t mnmajor_desc(uint32_t base, int kk) {
  return make_sdesc_sw128(base + kk * 2048, CHUNK_BYTES, 1024);
}

__device__ __forceinline__ void tma_load_4d(void *dst, const void *tmap, uint64_t *bar, int32_t x,
                                            int32_t y, int32_t z, int32_t w) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z), "r"(w)
      : "memory");
}

// One Q, K or V tile (rows r0.. of head h, batch b): HD/64 boxes of 64 columns.
template <int HD>
__device__ __forceinline__ void tma_load_tile(uint8_t *dst, const CUtensorMap *map, uint64_t *bar,
                                              int32_t r0, int32_t h, int32_t b) {
#pragma unroll
  for (int c = 0; c < HD / 64; ++c) tma_load_4d(dst + c * CHUNK_BYTES, map, bar, c * 64, r0, h, b);
}

// Scores of the keys past N in a partial last key tile become -inf, so they
// take part in neither the row max nor the sum (the tile's K and V rows past
// N were zero-filled by TMA).
__device__ __forceinline__ void mask_key_tail(uint32_t (&s)[128], int n_tail) {
#pragma unroll
  for (int i = 0; i < 128; ++i)
    if (i >= n_tail) s[i] = 0xff800000u;
}

// scale == 0 (c == 0): every weight is 2^0 = 1, but the -inf scores of the
// masked tail keys would give 0 * -inf = NaN in the exponent. For that case
// the last tile's weights are rebuilt as 1 for the n_tail real keys and 0
// past them; returns their sum.
__device__ __forceinline__ float zero_scale_tail_weights(uint32_t (&pk)[64], int n_tail) {
#pragma unroll
  for (int i = 0; i < 64; ++i)
    pk[i] = pack_bf16x2(2 * i < n_tail ? 1.0f : 0.0f, 2 * i + 1 < n_tail ? 1.0f : 0.0f);
  return static_cast<float>(n_tail);
}

// (batch, head, query block) of work unit u. 32-bit arithmetic (the launcher
// keeps units below 2^31): 64-bit division is a long software sequence that
// sat on the path between two units.
__device__ __forceinline__ void unit_coords(const Params &p, int64_t u, int32_t &b, int32_t &h,
                                            int32_t &qb) {
  const uint32_t uu = static_cast<uint32_t>(u), nqb = static_cast<uint32_t>(p.qblocks);
  const uint32_t nh = static_cast<uint32_t>(p.heads);
  const uint32_t bh = uu / nqb, bb = bh / nh;
  qb = static_cast<int32_t>(uu - bh * nqb);
  h = static_cast<int32_t>(bh - bb * nh);
  b = static_cast<int32_t>(bb);
}

template <int HD, bool kTail>
__global__ void __launch_bounds__(THREADS, 1)
    msm_tc_bf16_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                       const __grid_constant__ CUtensorMap tv, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  Smem<HD> &sm = *reinterpret_cast<Smem<HD> *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  volatile int *abort_flag = &sm.abort_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    mbar_init(&sm.q_full, 1);
    mbar_init(&sm.q_empty, 1);
    for (int s = 0; s < KSTAGES; ++s) {
      mbar_init(&sm.k_full[s], 1);
      mbar_init(&sm.k_empty[s], 1);
    }
    for (int s = 0; s < VSTAGES; ++s) {
      mbar_init(&sm.v_full[s], 1);
      mbar_init(&sm.v_empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&sm.s_full[s], 1);
      mbar_init(&sm.s_free[s], 128);
    }
    mbar_init(&sm.p_full, 128);
    mbar_init(&sm.p_free, 1);
    mbar_init(&sm.o_full, 1);
    mbar_init(&sm.o_empty, 128);
    mbar_init(&sm.drain, 1);
    sm.abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tq);
    tma_prefetch_desc(&tk);
    tma_prefetch_desc(&tv);
  }
  if (warp == 1) {
    tmem_alloc(&sm.tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_slot;
  const int64_t nkv = p.nkv_tiles;

  if (warp == 0) {
    // ---------------- producer ----------------
    if (lane == 0) {
      uint32_t kt = 0, vt = 0, uc = 0;
      for (int64_t u = blockIdx.x; u < p.units; u += gridDim.x, ++uc) {
        int32_t b, h, q0;
        unit_coords(p, u, b, h, q0);
        q0 *= BQ;
        if (!mbar_wait(&sm.q_empty, (uc & 1) ^ 1, abort_flag, p.status, kErrTimeoutEmpty)) break;
        mbar_arrive_expect_tx(&sm.q_full, tile_bytes<HD>());
        tma_load_tile<HD>(sm.q, &tq, &sm.q_full, q0, h, b);
        bool ok = true;
        for (int64_t t = 0; t < nkv && ok; ++t, ++kt, ++vt) {
          const int ks = kt % KSTAGES, vs = vt % VSTAGES;
          const int32_t key0 = static_cast<int32_t>(t * BKV);
          ok = mbar_wait(&sm.k_empty[ks], ((kt / KSTAGES) & 1) ^ 1, abort_flag, p.status,
                         kErrTimeoutEmpty);
          if (!ok) break;
          mbar_arrive_expect_tx(&sm.k_full[ks], tile_bytes<HD>());
          tma_load_tile<HD>(sm.k[ks], &tk, &sm.k_full[ks], key0, h, b);
          ok = mbar_wait(&sm.v_empty[vs], ((vt / VSTAGES) & 1) ^ 1, abort_flag, p.status,
                         kErrTimeoutEmpty);
          if (!ok) break;
          mbar_arrive_expect_tx(&sm.v_full[vs], tile_bytes<HD>());
          tma_load_tile<HD>(sm.v[vs], &tv, &sm.v_full[vs], key0, h, b);
        }
        if (!ok) break;
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      const uint32_t idesc_s = make_idesc(1, 1, 0, 0, BQ, BKV) | p.s_neg;
      const uint32_t idesc_o = make_idesc(1, 1, 0, 1, BQ, HD);
      const uint32_t q_addr = smem_u32(sm.q), p_addr = smem_u32(sm.p);
      uint32_t st = 0, pt = 0, uc = 0;
      bool ok = true;
      auto issue_s = [&]() -> bool {
        const int sb = st & 1, ks = st % KSTAGES;
        if (!mbar_wait(&sm.s_free[sb], ((st >> 1) & 1) ^ 1, abort_flag, p.status, kErrTimeoutAccum))
          return false;
        if (!mbar_wait(&sm.k_full[ks], (st / KSTAGES) & 1, abort_flag, p.status, kErrTimeoutFull))
          return false;
        tc_fence_after();
        const uint32_t k_addr = smem_u32(sm.k[ks]);
        const uint32_t d_tmem = tmem + S_COL0 + sb * BKV;
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk)
          mma_f16_ss(d_tmem, kmajor_desc(q_addr, kk), kmajor_desc(k_addr, kk), idesc_s,
                     kk ? 1u : 0u);
        mma_commit(&sm.k_empty[ks]);
        mma_commit(&sm.s_full[sb]);
        ++st;
        return true;
      };
      for (int64_t u = blockIdx.x; u < p.units && ok; u += gridDim.x, ++uc) {
        if (!mbar_wait(&sm.q_full, uc & 1, abort_flag, p.status, kErrTimeoutFull)) break;
        tc_fence_after();
        if (!(ok = issue_s())) break;
        for (int64_t t = 0; t < nkv; ++t) {
          if (t + 1 < nkv) {
            if (!(ok = issue_s())) break;
          } else {
            mma_commit(&sm.q_empty);  // every S MMA of this unit has been issued
          }
          if (t == 0 &&
              !(ok = mbar_wait(&sm.o_empty, (uc & 1) ^ 1, abort_flag, p.status, kErrTimeoutAccum)))
            break;
          const int vs = pt % VSTAGES;
          if (!(ok = mbar_wait(&sm.v_full[vs], (pt / VSTAGES) & 1, abort_flag, p.status,
                               kErrTimeoutFull)))
            break;
          if (!(ok = mbar_wait(&sm.p_full, pt & 1, abort_flag, p.status, kErrTimeoutAccum))) break;
          tc_fence_after();
          const uint32_t v_addr = smem_u32(sm.v[vs]);
#pragma unroll
          for (int kk = 0; kk < BKV / 16; ++kk)
            mma_f16_ss(tmem + O_COL, kmajor_desc(p_addr, kk), mnmajor_desc(v_addr, kk), idesc_o,
                       (t | kk) ? 1u : 0u);
          mma_commit(&sm.v_empty[vs]);
          mma_commit(&sm.p_free);
          ++pt;
        }
        if (!ok) break;
        mma_commit(&sm.o_full);
      }
      mma_commit(&sm.drain);
      if (!mbar_wait(&sm.drain, 0, nullptr, p.status, kErrTimeoutDrain)) *abort_flag = 1;
    }
  } else {
    // ---------------- softmax + output ----------------
    const int sub = warp & 3;
    const int row = sub * 32 + lane;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(sub * 32) << 16);
    uint8_t *p_row = sm.p + row * 128;
    const int rsw = row & 7;
    uint32_t s_cnt = 0, p_cnt = 0, uc = 0;
    bool ok = true;
    for (int64_t u = blockIdx.x; u < p.units && ok; u += gridDim.x, ++uc) {
      int32_t b, h, q0;
      unit_coords(p, u, b, h, q0);
      q0 *= BQ;
      float m_ref = -INFINITY, l = 0.0f;
      for (int64_t t = 0; t < nkv; ++t) {
        const int sb = s_cnt & 1;
        if (!(ok = mbar_wait_warp(&sm.s_full[sb], (s_cnt >> 1) & 1, abort_flag, p.status,
                             kErrTimeoutAccum)))
          break;
        tc_fence_after();
        uint32_t s[128];
        {
          uint32_t (&s0)[32] = *reinterpret_cast<uint32_t(*)[32]>(&s[0]);
          uint32_t (&s1)[32] = *reinterpret_cast<uint32_t(*)[32]>(&s[32]);
          uint32_t (&s2)[32] = *reinterpret_cast<uint32_t(*)[32]>(&s[64]);
          uint32_t (&s3)[32] = *reinterpret_cast<uint32_t(*)[32]>(&s[96]);
          const uint32_t a = lane_base + S_COL0 + sb * BKV;
          tmem_ld_32x32b_x32(a, s0);
          tmem_ld_32x32b_x32(a + 32, s1);
          tmem_ld_32x32b_x32(a + 64, s2);
          tmem_ld_32x32b_x32(a + 96, s3);
          tmem_ld_wait();
          reg_fence(s0);
          reg_fence(s1);
          reg_fence(s2);
          reg_fence(s3);
        }
        if (kTail && t + 1 == nkv) mask_key_tail(s, p.n_tail);
        tc_fence_before();
        mbar_arrive(&sm.s_free[sb]);
        ++s_cnt;
        float mx = __uint_as_float(s[0]);
#pragma unroll
        for (int i = 1; i < 128; ++i) mx = fmaxf(mx, __uint_as_float(s[i]));
        bool need = false;
        if (t == 0) {
          m_ref = mx;
        } else if ((mx - m_ref) * p.c > 8.0f) {
          need = true;
        }
        if (__any_sync(0xffffffffu, need)) {
          // Rescale O and l for the rows whose max grew: O must be complete
          // up to PV_{t-1} and PV_t cannot start before this thread signals.
          if (!(ok = mbar_wait_warp(&sm.p_free, (p_cnt - 1) & 1, abort_flag, p.status,
                               kErrTimeoutAccum)))
            break;
          tc_fence_after();
          const float f = need ? ex2((m_ref - mx) * p.c) : 1.0f;
          // Load / scale / store the HD O columns of this row, 32 at a time.
#pragma unroll 1
          for (int c0 = 0; c0 < HD; c0 += 32) {
            uint32_t o[32];
            tmem_ld32_sync(lane_base + O_COL + c0, o);
            uint32_t lo[16], hi[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              lo[i] = __float_as_uint(__uint_as_float(o[i]) * f);
              hi[i] = __float_as_uint(__uint_as_float(o[16 + i]) * f);
            }
            tmem_st_32x32b_x16(lane_base + O_COL + c0, lo);
            tmem_st_32x32b_x16(lane_base + O_COL + c0 + 16, hi);
          }
          tmem_st_wait();
          tc_fence_before();
          if (need) {
            l *= f;
            m_ref = mx;
          }
        }
        const float mc = m_ref * p.c;
        uint32_t pk[64];
        float psum = 0.0f;
#pragma unroll
        for (int i = 0; i < 64; ++i) {
          const float e0 = ex2(fmaf(__uint_as_float(s[2 * i]), p.c, -mc));
          const float e1 = ex2(fmaf(__uint_as_float(s[2 * i + 1]), p.c, -mc));
          psum += e0 + e1;
          pk[i] = pack_bf16x2(e0, e1);
        }
        if (kTail && t + 1 == nkv && p.c == 0.0f) psum = zero_scale_tail_weights(pk, p.n_tail);
        l += psum;
        // P buffer is free once PV of the previous tile has completed.
        if (!(ok = mbar_wait_warp(&sm.p_free, (p_cnt & 1) ^ 1, abort_flag, p.status,
                             kErrTimeoutAccum)))
          break;
#pragma unroll
        for (int u16 = 0; u16 < 16; ++u16) {
          const int chunk = u16 >> 3, j = u16 & 7;
          uint4 v4 = make_uint4(pk[u16 * 4], pk[u16 * 4 + 1], pk[u16 * 4 + 2], pk[u16 * 4 + 3]);
          *reinterpret_cast<uint4 *>(p_row + chunk * CHUNK_BYTES + ((j ^ rsw) << 4)) = v4;
        }
        fence_async_smem();
        mbar_arrive(&sm.p_full);
        ++p_cnt;
      }
      if (!ok) break;
      // ---- output: O / l -> bf16 ----
      if (!(ok = mbar_wait_warp(&sm.o_full, uc & 1, abort_flag, p.status, kErrTimeoutAccum)))
        break;
      tc_fence_after();
      const float inv = 1.0f / l;
      const bool row_live = q0 + row < p.m_rows;
      __nv_bfloat16 *orow =
          p.o + b * p.o_s[0] + h * p.o_s[1] + static_cast<int64_t>(q0 + row) * p.o_s[2];
#pragma unroll 1
      for (int c0 = 0; c0 < HD; c0 += 32) {
        uint32_t o[32];
        tmem_ld32_sync(lane_base + O_COL + c0, o);
        uint4 *dst = reinterpret_cast<uint4 *>(orow + c0);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint4 w;
          w.x = pack_bf16x2(__uint_as_float(o[q * 8 + 0]) * inv, __uint_as_float(o[q * 8 + 1]) * inv);
          w.y = pack_bf16x2(__uint_as_float(o[q * 8 + 2]) * inv, __uint_as_float(o[q * 8 + 3]) * inv);
          w.z = pack_bf16x2(__uint_as_float(o[q * 8 + 4]) * inv, __uint_as_float(o[q * 8 + 5]) * inv);
          w.w = pack_bf16x2(__uint_as_float(o[q * 8 + 6]) * inv, __uint_as_float(o[q * 8 + 7]) * inv);
          if (row_live) dst[q] = w;
        }
      }
      tc_fence_before();
      mbar_arrive(&sm.o_empty);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

// ---- two query tiles per CTA (query blocks of 256 rows) ---------------------------------
// The single-tile kernel above leaves one softmax warp per SM sub-partition,
// which cannot keep the exp2 unit busy while the tensor core waits for P. Here
// a work unit is a 256-row query block split into two 128-row tiles g = 0, 1,
// each with its own softmax warpgroup (warps 2-5 and 6-9, one warp per TMEM
// lane quarter each), its own S (TMEM columns 128g) and O (256 + HD g)
// accumulators and its own P buffer in shared memory. Each K/V tile is
// loaded once and used by both query tiles; K and V share one ring (3 stages
// of 32 KiB at HD = 128, 6 of 16 KiB at HD = 64),
// loaded in the order the MMA thread consumes them (K0, K1, V0, K2, V1, ...).
// The MMA thread issues S0(j+1), S1(j+1) as soon as the warpgroups have read
// S(j) into registers, then PV0(j), PV1(j) once P(j) is written, so the
// tensor core computes the next scores while both warpgroups exponentiate.
// The softmax arithmetic uses packed f32x2 FMA/ADD and three-input max.
// At the end of a unit each warpgroup stages its normalised O tile in its P
// buffer (free once the last PV has completed) and one thread writes it with
// a TMA store, so the next unit's first scores are not held up by 128
// threads' row-wise global stores.
constexpr int NQ = 2;
constexpr int UNIT_ROWS = NQ * BQ;
constexpr int THREADS2 = 64 + NQ * 128;
template <int HD>
constexpr int kv_stages() {
  return HD == 128 ? 3 : 6;
}

template <int HD>
struct Smem2 {
  static constexpr int KV_STAGES = kv_stages<HD>();
  uint8_t q[NQ][tile_bytes<HD>()];
  uint8_t kv[KV_STAGES][tile_bytes<HD>()];
  uint8_t p[NQ][P_BYTES];
  uint64_t q_full, q_empty;
  uint64_t kv_full[KV_STAGES], kv_empty[KV_STAGES];
  uint64_t s_full[NQ], s_free[NQ];
  uint64_t p_full[NQ], p_free[NQ];
  uint64_t o_full[NQ], o_empty[NQ];
  uint64_t o_staged[NQ], o_read[NQ];  // O staged in P_g; P_g read by the O store
  uint64_t drain;
  uint32_t tmem_slot;
  int abort_flag;
};
template <int HD>
constexpr size_t smem2_bytes() {
  return sizeof(Smem2<HD>) + 1024;
}
static_assert(smem2_bytes<128>() <= 232448 && smem2_bytes<64>() <= 232448,
              "two-tile MSM exceeds the opt-in shared memory per block");
static_assert(smem_bytes<128>() <= 232448, "single-tile MSM exceeds the opt-in shared memory");

template <int HD, bool kTail>
__global__ void __launch_bounds__(THREADS2, 1)
    msm_tc2_bf16_kernel(const __grid_constant__ CUtensorMap tq,
                        const __grid_constant__ CUtensorMap tk,
                        const __grid_constant__ CUtensorMap tv,
                        const __grid_constant__ CUtensorMap to, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  constexpr int KV_STAGES = kv_stages<HD>();
  Smem2<HD> &sm = *reinterpret_cast<Smem2<HD> *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  volatile int *abort_flag = &sm.abort_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    mbar_init(&sm.q_full, 1);
    mbar_init(&sm.q_empty, 1);
    for (int s = 0; s < KV_STAGES; ++s) {
      mbar_init(&sm.kv_full[s], 1);
      mbar_init(&sm.kv_empty[s], 1);
    }
    for (int g = 0; g < NQ; ++g) {
      mbar_init(&sm.s_full[g], 1);
      mbar_init(&sm.s_free[g], 128);
      mbar_init(&sm.p_full[g], 128);
      mbar_init(&sm.p_free[g], 1);
      mbar_init(&sm.o_full[g], 1);
      mbar_init(&sm.o_empty[g], 128);
      mbar_init(&sm.o_staged[g], 128);
      mbar_init(&sm.o_read[g], 1);
    }
    mbar_init(&sm.drain, 1);
    sm.abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tq);
    tma_prefetch_desc(&tk);
    tma_prefetch_desc(&tv);
    if (p.o_tma) tma_prefetch_desc(&to);
  }
  if (warp == 1) {
    tmem_alloc(&sm.tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_slot;
  const int64_t nkv = p.nkv_tiles;

  if (warp == 0) {
    // ---------------- producer ----------------
    if (lane == 0) {
      uint32_t kvc = 0, uc = 0;
      bool ok = true;
      auto load_tile = [&](const CUtensorMap *map, int32_t key0, int32_t h, int32_t b) -> bool {
        const int s = kvc % KV_STAGES;
        if (!mbar_wait(&sm.kv_empty[s], ((kvc / KV_STAGES) & 1) ^ 1, abort_flag, p.status,
                       kErrTimeoutEmpty))
          return false;
        mbar_arrive_expect_tx(&sm.kv_full[s], tile_bytes<HD>());
        tma_load_tile<HD>(sm.kv[s], map, &sm.kv_full[s], key0, h, b);
        ++kvc;
        return true;
      };
      for (int64_t u = blockIdx.x; u < p.units && ok; u += gridDim.x, ++uc) {
        int32_t b, h, q0;
        unit_coords(p, u, b, h, q0);
        q0 *= UNIT_ROWS;
        if (!mbar_wait(&sm.q_empty, (uc & 1) ^ 1, abort_flag, p.status, kErrTimeoutEmpty)) break;
        mbar_arrive_expect_tx(&sm.q_full, NQ * tile_bytes<HD>());
        for (int g = 0; g < NQ; ++g) tma_load_tile<HD>(sm.q[g], &tq, &sm.q_full, q0 + g * BQ, h, b);
        if (!(ok = load_tile(&tk, 0, h, b))) break;
        for (int64_t t = 0; t < nkv && ok; ++t) {
          if (t + 1 < nkv && !(ok = load_tile(&tk, static_cast<int32_t>((t + 1) * BKV), h, b)))
            break;
          ok = load_tile(&tv, static_cast<int32_t>(t * BKV), h, b);
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      const uint32_t idesc_s = make_idesc(1, 1, 0, 0, BQ, BKV) | p.s_neg;
      const uint32_t idesc_o = make_idesc(1, 1, 0, 1, BQ, HD);
      uint32_t kvc = 0, s_cnt = 0, p_cnt = 0, uc = 0;
      bool ok = true;
      auto kv_stage = [&](uint32_t &addr) -> int {
        const int s = kvc % KV_STAGES;
        if (!mbar_wait(&sm.kv_full[s], (kvc / KV_STAGES) & 1, abort_flag, p.status,
                       kErrTimeoutFull))
          return -1;
        addr = smem_u32(sm.kv[s]);
        return s;
      };
      auto s_round = [&]() -> bool {  // S_g = Q_g K^T for both query tiles
        uint32_t k_addr;
        const int s = kv_stage(k_addr);
        if (s < 0) return false;
        for (int g = 0; g < NQ; ++g) {
          if (!mbar_wait(&sm.s_free[g], (s_cnt & 1) ^ 1, abort_flag, p.status, kErrTimeoutAccum))
            return false;
          tc_fence_after();
          const uint32_t q_addr = smem_u32(sm.q[g]);
#pragma unroll
          for (int kk = 0; kk < HD / 16; ++kk)
            mma_f16_ss(tmem + S_COL0 + g * BKV, kmajor_desc(q_addr, kk), kmajor_desc(k_addr, kk),
                       idesc_s, kk ? 1u : 0u);
          mma_commit(&sm.s_full[g]);
        }
        mma_commit(&sm.kv_empty[s]);
        ++kvc;
        ++s_cnt;
        return true;
      };
      auto pv_round = [&](int64_t t) -> bool {  // O_g += P_g V for both query tiles
        uint32_t v_addr;
        const int s = kv_stage(v_addr);
        if (s < 0) return false;
        for (int g = 0; g < NQ; ++g) {
          if (t == 0 &&
              !mbar_wait(&sm.o_empty[g], (uc & 1) ^ 1, abort_flag, p.status, kErrTimeoutAccum))
            return false;
          if (!mbar_wait(&sm.p_full[g], p_cnt & 1, abort_flag, p.status, kErrTimeoutAccum))
            return false;
          tc_fence_after();
          const uint32_t p_addr = smem_u32(sm.p[g]);
#pragma unroll
          for (int kk = 0; kk < BKV / 16; ++kk)
            mma_f16_ss(tmem + O_COL + g * HD, kmajor_desc(p_addr, kk), mnmajor_desc(v_addr, kk),
                       idesc_o, (t | kk) ? 1u : 0u);
          mma_commit(&sm.p_free[g]);
          // Query tile g's output is final after its last PV: its epilogue
          // need not wait for the other tile's.
          if (t + 1 == nkv) mma_commit(&sm.o_full[g]);
        }
        mma_commit(&sm.kv_empty[s]);
        ++kvc;
        ++p_cnt;
        return true;
      };
      for (int64_t u = blockIdx.x; u < p.units && ok; u += gridDim.x, ++uc) {
        if (!mbar_wait(&sm.q_full, uc & 1, abort_flag, p.status, kErrTimeoutFull)) break;
        tc_fence_after();
        if (!(ok = s_round())) break;
        for (int64_t t = 0; t < nkv; ++t) {
          if (t + 1 < nkv) {
            if (!(ok = s_round())) break;
          } else {
            mma_commit(&sm.q_empty);  // every S MMA of this unit has been issued
          }
          if (!(ok = pv_round(t))) break;
        }
        if (!ok) break;
      }
      mma_commit(&sm.drain);
      if (!mbar_wait(&sm.drain, 0, nullptr, p.status, kErrTimeoutDrain)) *abort_flag = 1;
    }
  } else {
    // ---------------- softmax + output (warpgroup g owns query tile g) ----------------
    const int g = (warp - 2) >> 2;
    const int sub = warp & 3;
    const int row = sub * 32 + lane;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(sub * 32) << 16);
    const uint32_t s_col = S_COL0 + g * BKV, o_col = O_COL + g * HD;
    uint8_t *p_row = sm.p[g] + row * 128;
    const int rsw = row & 7;
    const bool leader = (threadIdx.x & 127) == 0;  // issues this warpgroup's O stores
    uint32_t s_cnt = 0, p_cnt = 0, uc = 0;
    bool ok = true;
    for (int64_t u = blockIdx.x; u < p.units && ok; u += gridDim.x, ++uc) {
      int32_t b, h, q0;
      unit_coords(p, u, b, h, q0);
      q0 = q0 * UNIT_ROWS + g * BQ;
      float m_ref = -INFINITY, l = 0.0f;
      for (int64_t t = 0; t < nkv; ++t) {
        if (!(ok = mbar_wait_warp(&sm.s_full[g], s_cnt & 1, abort_flag, p.status,
                                  kErrTimeoutAccum)))
          break;
        tc_fence_after();
        uint32_t s[128];
        {
          uint32_t (&s0)[32] = *reinterpret_cast<uint32_t(*)[32]>(&s[0]);
          uint32_t (&s1)[32] = *reinterpret_cast<uint32_t(*)[32]>(&s[32]);
          uint32_t (&s2)[32] = *reinterpret_cast<uint32_t(*)[32]>(&s[64]);
          uint32_t (&s3)[32] = *reinterpret_cast<uint32_t(*)[32]>(&s[96]);
          const uint32_t a = lane_base + s_col;
          tmem_ld_32x32b_x32(a, s0);
          tmem_ld_32x32b_x32(a + 32, s1);
          tmem_ld_32x32b_x32(a + 64, s2);
          tmem_ld_32x32b_x32(a + 96, s3);
          tmem_ld_wait();
          reg_fence(s0);
          reg_fence(s1);
          reg_fence(s2);
          reg_fence(s3);
        }
        if (kTail && t + 1 == nkv) mask_key_tail(s, p.n_tail);
        tc_fence_before();
        mbar_arrive(&sm.s_free[g]);
        ++s_cnt;
        // Row max: four chains of three-input max, two scores per step.
        float m4[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) m4[i] = __uint_as_float(s[i]);
#pragma unroll
        for (int i = 4; i < 128; i += 8)
#pragma unroll
          for (int j = 0; j < 4; ++j)
            m4[j] = fmax3(m4[j], __uint_as_float(s[i + 2 * j]), __uint_as_float(s[i + 2 * j + 1]));
        const float mx = fmax3(m4[0], m4[1], fmaxf(m4[2], m4[3]));
        bool need = false;
        if (t == 0) {
          m_ref = mx;
        } else if ((mx - m_ref) * p.c > 8.0f) {
          need = true;
        }
        if (__any_sync(0xffffffffu, need)) {
          // Rescale O and l for the rows whose max grew: O must be complete
          // up to PV_{t-1} and PV_t cannot start before this thread signals.
          if (!(ok = mbar_wait_warp(&sm.p_free[g], (p_cnt - 1) & 1, abort_flag, p.status,
                                    kErrTimeoutAccum)))
            break;
          tc_fence_after();
          const float f = need ? ex2((m_ref - mx) * p.c) : 1.0f;
          // 16 columns at a time: the 128 scores stay live across this loop.
#pragma unroll 1
          for (int c0 = 0; c0 < HD; c0 += 16) {
            uint32_t o[16];
            tmem_ld16_sync(lane_base + o_col + c0, o);
#pragma unroll
            for (int i = 0; i < 16; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * f);
            tmem_st_32x32b_x16(lane_base + o_col + c0, o);
          }
          tmem_st_wait();
          tc_fence_before();
          if (need) {
            l *= f;
            m_ref = mx;
          }
        }
        const float mc = m_ref * p.c;
        const uint64_t c2 = f2_pack(p.c, p.c), nmc2 = f2_pack(-mc, -mc);
        uint32_t pk[64];
        uint64_t ps[4] = {0, 0, 0, 0};  // +0.0f pairs
#pragma unroll
        for (int i = 0; i < 64; ++i) {
          float x0, x1;
          f2_unpack(f2_fma(f2_pack(__uint_as_float(s[2 * i]), __uint_as_float(s[2 * i + 1])), c2,
                           nmc2),
                    x0, x1);
          const float e0 = ex2(x0), e1 = ex2(x1);
          ps[i & 3] = f2_add(ps[i & 3], f2_pack(e0, e1));
          pk[i] = pack_bf16x2(e0, e1);
        }
        {
          float a0, a1;
          f2_unpack(f2_add(f2_add(ps[0], ps[1]), f2_add(ps[2], ps[3])), a0, a1);
          float tile_sum = a0 + a1;
          if (kTail && t + 1 == nkv && p.c == 0.0f)
            tile_sum = zero_scale_tail_weights(pk, p.n_tail);
          l += tile_sum;
        }
        // P_g is free once PV_g of the previous tile has completed.
        if (!(ok = mbar_wait_warp(&sm.p_free[g], (p_cnt & 1) ^ 1, abort_flag, p.status,
                                  kErrTimeoutAccum)))
          break;
        // At a unit's first tile P_g may still be the source of the previous
        // unit's O store.
        if (t == 0 && uc > 0 && p.o_tma) {
          if (leader) {
            bulk_wait_read_all();
            mbar_arrive(&sm.o_read[g]);
          }
          if (!(ok = mbar_wait_warp(&sm.o_read[g], (uc - 1) & 1, abort_flag, p.status,
                                    kErrTimeoutAccum)))
            break;
        }
#pragma unroll
        for (int u16 = 0; u16 < 16; ++u16) {
          const int chunk = u16 >> 3, j = u16 & 7;
          uint4 v4 = make_uint4(pk[u16 * 4], pk[u16 * 4 + 1], pk[u16 * 4 + 2], pk[u16 * 4 + 3]);
          *reinterpret_cast<uint4 *>(p_row + chunk * CHUNK_BYTES + ((j ^ rsw) << 4)) = v4;
        }
        fence_async_smem();
        mbar_arrive(&sm.p_full[g]);
        ++p_cnt;
      }
      if (!ok) break;
      // ---- output: O_g / l -> bf16 ----
      if (!(ok = mbar_wait_warp(&sm.o_full[g], uc & 1, abort_flag, p.status, kErrTimeoutAccum)))
        break;
      tc_fence_after();
      const float inv = 1.0f / l;
      if (p.o_tma) {
        // Stage the tile in P_g (free: the last PV_g has completed) in the
        // 128-byte-swizzled layout of the TMA box, then one thread stores it.
        // Coalescing through TMA keeps the per-row 16-byte stores of 128
        // threads off the load/store unit between two work units.
#pragma unroll 1
        for (int c0 = 0; c0 < HD; c0 += 32) {
          uint32_t o[32];
          tmem_ld32_sync(lane_base + o_col + c0, o);
          uint8_t *dst = p_row + (c0 >> 6) * CHUNK_BYTES;
          const int j0 = (c0 & 63) >> 3;
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint4 w;
            w.x = pack_bf16x2(__uint_as_float(o[q * 8 + 0]) * inv, __uint_as_float(o[q * 8 + 1]) * inv);
            w.y = pack_bf16x2(__uint_as_float(o[q * 8 + 2]) * inv, __uint_as_float(o[q * 8 + 3]) * inv);
            w.z = pack_bf16x2(__uint_as_float(o[q * 8 + 4]) * inv, __uint_as_float(o[q * 8 + 5]) * inv);
            w.w = pack_bf16x2(__uint_as_float(o[q * 8 + 6]) * inv, __uint_as_float(o[q * 8 + 7]) * inv);
            *reinterpret_cast<uint4 *>(dst + (((j0 + q) ^ rsw) << 4)) = w;
          }
        }
        fence_async_smem();
        mbar_arrive(&sm.o_staged[g]);
        tc_fence_before();
        mbar_arrive(&sm.o_empty[g]);
        if (leader) {
          if (!(ok = mbar_wait(&sm.o_staged[g], uc & 1, abort_flag, p.status, kErrTimeoutAccum)))
            break;
#pragma unroll
          for (int c = 0; c < HD / 64; ++c)
            tma_store_4d(&to, sm.p[g] + c * CHUNK_BYTES, c * 64, q0, h, b);
          bulk_commit();
        }
      } else {
        const bool row_live = q0 + row < p.m_rows;
        __nv_bfloat16 *orow =
            p.o + b * p.o_s[0] + h * p.o_s[1] + static_cast<int64_t>(q0 + row) * p.o_s[2];
#pragma unroll 1
        for (int c0 = 0; c0 < HD; c0 += 32) {
          uint32_t o[32];
          tmem_ld32_sync(lane_base + o_col + c0, o);
          uint4 *dst = reinterpret_cast<uint4 *>(orow + c0);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint4 w;
            w.x = pack_bf16x2(__uint_as_float(o[q * 8 + 0]) * inv, __uint_as_float(o[q * 8 + 1]) * inv);
            w.y = pack_bf16x2(__uint_as_float(o[q * 8 + 2]) * inv, __uint_as_float(o[q * 8 + 3]) * inv);
            w.z = pack_bf16x2(__uint_as_float(o[q * 8 + 4]) * inv, __uint_as_float(o[q * 8 + 5]) * inv);
            w.w = pack_bf16x2(__uint_as_float(o[q * 8 + 6]) * inv, __uint_as_float(o[q * 8 + 7]) * inv);
            if (row_live) dst[q] = w;
          }
        }
        tc_fence_before();
        mbar_arrive(&sm.o_empty[g]);
      }
    }
    // Outstanding O stores must finish reading shared memory (and land)
    // before the block exits.
    if (p.o_tma && leader) bulk_wait_all();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

}  // namespace

bool encode_tmap_4d_bf16(CUtensorMap *map, const void *base, uint64_t d0, uint64_t d1, uint64_t d2,
                         uint64_t d3, uint64_t s1, uint64_t s2, uint64_t s3);

cudaError_t launch_msm_tc_bf16(const void *q, const void *k, const void *v, void *o,
                               const MsmShape &s, float scale, uint32_t *status, int sms,
                               cudaStream_t stream, LaunchInfo *info) {
  if (s.m <= 0 || s.n <= 0 || s.dqk != s.dv || (s.dqk != 64 && s.dqk != 128))
    return cudaErrorNotSupported;
  const int hd = static_cast<int>(s.dqk);
  CUtensorMap tq, tk, tv;
  auto enc = [&](CUtensorMap *map, const void *base, int64_t rows, const int64_t *st) {
    // dims {HD, rows, heads, batch}; byte strides of rows/heads/batch. A unit
    // dimension gets a harmless stride (TMA only needs it 16-byte aligned).
    const uint64_t srow = static_cast<uint64_t>(st[2]) * 2;
    const uint64_t sh = s.heads > 1 ? static_cast<uint64_t>(st[1]) * 2 : srow * rows;
    const uint64_t sb = s.batch > 1 ? static_cast<uint64_t>(st[0]) * 2 : sh * s.heads;
    return encode_tmap_4d_bf16(map, base, hd, rows, s.heads, s.batch, srow, sh, sb);
  };
  // cudaErrorNotSupported (nothing launched) lets the caller take another kernel.
  if (!enc(&tq, q, s.m, s.q_s) || !enc(&tk, k, s.n, s.k_s) || !enc(&tv, v, s.n, s.v_s))
    return cudaErrorNotSupported;
  // Query blocks of 256 rows run two tiles per CTA; otherwise one. The
  // two-tile kernel stores O by TMA when O's layout can be described by a
  // tensor map (16-byte aligned base and strides), else with plain stores.
  // Ragged M: the last query block is partly past M (TMA zero-fills Q there
  // and the stores skip those rows). Two-tile units unless that would
  // waste more than half a unit on a short problem.
  const bool two = s.m % UNIT_ROWS == 0 || s.m % UNIT_ROWS > BQ || s.m >= 8 * UNIT_ROWS;
  CUtensorMap to;
  const bool o_tma = two && enc(&to, o, s.m, s.o_s);
  if (!o_tma) to = tq;  // unused by the kernel
  Params p;
  p.heads = s.heads;
  p.qblocks = (s.m + (two ? UNIT_ROWS : BQ) - 1) / (two ? UNIT_ROWS : BQ);
  p.nkv_tiles = (s.n + BKV - 1) / BKV;
  p.m_rows = static_cast<int>(s.m);
  p.n_tail = static_cast<int>(s.n % BKV);
  p.units = s.batch * s.heads * p.qblocks;
  if (p.units > 0x7fffffff) return cudaErrorNotSupported;  // unit indices are 32-bit
  for (int i = 0; i < 3; ++i) p.o_s[i] = s.o_s[i];
  p.o_tma = o_tma ? 1 : 0;
  // softmax(scale * S) with scale < 0 equals softmax(|scale| * (-S)). The S
  // MMA negates Q (the A operand) instead, which is exact (the negated
  // products and their sum round symmetrically), so the softmax code always
  // sees a non-negative factor and its row maximum is the exponent maximum.
  p.c = fabsf(scale) * 1.4426950408889634f;
  p.s_neg = scale < 0.0f ? kIdescNegateA : 0u;
  p.o = static_cast<__nv_bfloat16 *>(o);
  p.status = status;
  cudaError_t e;
  int grid = static_cast<int>(p.units < sms ? p.units : sms);
  // Key-tail masking is compiled only into the instantiations that need it,
  // so full key tiles run exactly the unmasked loop.
  auto run2 = [&](auto kernel, size_t smem) -> cudaError_t {
    cudaError_t err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           static_cast<int>(smem));
    if (err != cudaSuccess) return err;
    kernel<<<grid, THREADS2, smem, stream>>>(tq, tk, tv, to, p);
    return cudaSuccess;
  };
  auto run1 = [&](auto kernel, size_t smem) -> cudaError_t {
    cudaError_t err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           static_cast<int>(smem));
    if (err != cudaSuccess) return err;
    kernel<<<grid, THREADS, smem, stream>>>(tq, tk, tv, p);
    return cudaSuccess;
  };
  const bool tail = p.n_tail != 0;
  if (hd == 128) {
    if (two)
      e = tail ? run2(msm_tc2_bf16_kernel<128, true>, smem2_bytes<128>())
               : run2(msm_tc2_bf16_kernel<128, false>, smem2_bytes<128>());
    else
      e = tail ? run1(msm_tc_bf16_kernel<128, true>, smem_bytes<128>())
               : run1(msm_tc_bf16_kernel<128, false>, smem_bytes<128>());
  } else {
    if (two)
      e = tail ? run2(msm_tc2_bf16_kernel<64, true>, smem2_bytes<64>())
               : run2(msm_tc2_bf16_kernel<64, false>, smem2_bytes<64>());
    else
      e = tail ? run1(msm_tc_bf16_kernel<64, true>, smem_bytes<64>())
               : run1(msm_tc_bf16_kernel<64, false>, smem_bytes<64>());
  }
  if (e != cudaSuccess) return e;
  if (info) {
    info->launches = 1;
    info->tile_m = two ? UNIT_ROWS : BQ;
    info->tile_n = BKV;
    info->tile_k = hd;
    info->stages = two ? (hd == 128 ? kv_stages<128>() : kv_stages<64>()) : KSTAGES;
    info->ctas = grid;
    info->set_route("tcgen05_bf16_msm");
  }
  return cudaGetLastError();
}

}  // namespace mcb

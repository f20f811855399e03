// bf16 (or f16) GEMM with a fused epilogue on the B200's 5th-generation
// tensor cores. f16 operands change only the MMA's operand format, the TMA
// element type and the epilogue's output conversion.
//
//   Y[M,N] = act(X[M,K] * W (+|r-) bias)      (Family A, src/fusion_emitter_family_a.cpp)
//
// Two kernels: gemm_tc_bf16_pair_kernel (M >= 256; CTA pairs with
// tcgen05.mma.cta_group::2, described with the kernel below) and
// gemm_tc_bf16_kernel (single SM), whose design is:
//
// Design (one persistent CTA per SM, 192 threads, warp-specialised):
//   warp 0      TMA producer: streams 128x64 tiles of X and 64x256 (or 256x64
//               for W^T) tiles of W into a 4-stage shared-memory ring
//               (128-byte swizzle), signalling `full[s]` by transaction bytes.
//   warp 1      allocates 512 TMEM columns (two 128x256 f32 accumulators);
//               one thread issues tcgen05.mma (M=128, N=256, K=16, bf16 in,
//               f32 accumulate), releases each stage with tcgen05.commit on
//               `empty[s]`, and hands a finished accumulator to the epilogue
//               with a commit on `acc_full[a]`.
//   warps 2-5   epilogue: tcgen05.ld 32 columns at a time from the TMEM lanes
//               their warp may access (warp % 4), add the bias, apply the
//               activation, round to bf16/f32 and store, then release the
//               accumulator on `acc_empty[a]` so the MMA of the next tile
//               overlaps this tile's epilogue.
// X is K-major; W [K,N] row-major is consumed MN-major straight from HBM
// (no transpose pass); W^T [N,K] is consumed K-major.
//
// Roofline (config 2, 8192x4096x4096): 2*M*N*K = 274.9 GFLOP against the
// bf16 dense tensor peak; ideal HBM traffic X + W + Y = 160 MiB.
#include <cuda_bf16.h>

#include <algorithm>
#include <atomic>
#include <cstdlib>
#include <cstring>
#include <type_traits>

#ifndef MCB_PAIR_EPI_WARPS
#define MCB_PAIR_EPI_WARPS 8
#endif

#include "common.cuh"
#include "epilogue.cuh"
#include "internal.h"

namespace mcb {
namespace {

constexpr int BM = 128, BN = 256, BK = 64, STAGES = 4;
constexpr int A_BYTES = BM * BK * 2;  // 16 KiB
constexpr int B_BYTES = BN * BK * 2;  // 32 KiB
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int THREADS = 192;
constexpr int TMEM_COLS = 2 * BN;
constexpr int BAR_BYTES = 256;
constexpr size_t SMEM_BYTES = static_cast<size_t>(STAGES) * STAGE_BYTES + BAR_BYTES + 1024;

struct Params {
  int64_t m, n, k, ld_y;
  int n_tiles, num_tiles, num_kb;
  int w_transposed, y_kind, in_f16;  // y_kind: kOutF32 / kOutBf16 / kOutF16
  int y_tma;  // CTA-pair kernel: 0, or y_kind (16-bit) when whole tiles are staged per warp
  int y_lsu;  // staged chunks leave shared memory by coalesced st.global (1) or a TMA store (0)
  void *y;
  uint32_t *status;
  long long spin_limit;  // clock64 cycles a pipeline wait may take before the kernel aborts
  int stall_loads;       // self-test only: the producer issues no loads (the waits must time out)
  // Stream-K (CTA-pair kernel): tiles [0, sk_first_tile) run whole, one per
  // cluster in turn; tiles [sk_first_tile, num_tiles) are split in chains
  // (see the stream-K work split below).
  int sk_first_tile;
  int sk_tiles, sk_chains, sk_w;  // split tiles, chains, last-share reduction (K blocks)
  int *sk_flag;    // per (split tile, CTA rank): 1 once the tail's partial is written; 0 between launches
  float *sk_part;  // tail partial accumulators: per (cluster, CTA rank) 128x256 f32
  int sk_test_no_release;  // self-test only: tails never raise their flag (owners' waits run out)
  Epilogue epi;
};

// Epilogue of one 32-column chunk held by one thread (one output row):
// epilogue_values applies the bias / boundary and the activation (row < M
// only: a full [M,N] bias or boundary has no row past M); epilogue_chunk
// adds the row guard and stores the row's 32 values itself;
// epilogue_chunk_tma (CTA-pair kernel, 16-bit outputs) stages the warp's 32
// rows in shared memory and stores them with one TMA copy.
// kChain: the general op chain (its own kernel instantiation, so the
// bias + activation kernels compile exactly as without it).
// `bias_smem` (optional): the chunk's 32 row-bias bf16 values already staged
// in shared memory (read as 4 broadcast 16-byte loads instead of global ones).
template <bool kChain>
__device__ __forceinline__ void epilogue_values(const Params &p, const uint32_t (&r)[32],
                                                int64_t row, int64_t col0,
                                                const uint4 *bias_smem, float (&v)[32]) {
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
  const Epilogue &e = p.epi;
  const bool full_chunk = col0 + 32 <= p.n;
  if constexpr (kChain) {
    epilogue_chain_chunk(e, v, row, col0, p.n);
  } else if (e.bias_mode == 1 && e.bias_bf16 && e.bias_aligned16 && full_chunk) {
    // Row-broadcast bf16 bias: every lane reads the same 64 bytes.
    const uint4 *bp = reinterpret_cast<const uint4 *>(
        reinterpret_cast<const __nv_bfloat16 *>(e.bias) + col0);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const uint4 w4 = bias_smem ? bias_smem[q] : __ldg(bp + q);
      const uint32_t ws[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        const float b0 = __uint_as_float(ws[h] << 16);
        const float b1 = __uint_as_float(ws[h] & 0xffff0000u);
        float &x0 = v[q * 8 + h * 2], &x1 = v[q * 8 + h * 2 + 1];
        if (e.bias_op == 1) {
          x0 = b0 - x0;
          x1 = b1 - x1;
        } else {  // two adds in one packed f32x2 instruction
          f2_unpack(f2_add(f2_pack(x0, x1), f2_pack(b0, b1)), x0, x1);
        }
      }
    }
  } else if (e.bias_mode == 1 && e.bias_f16 && e.bias_aligned16 && full_chunk) {
    const uint4 *bp = reinterpret_cast<const uint4 *>(reinterpret_cast<const __half *>(e.bias) + col0);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const uint4 w4 = __ldg(bp + q);
      const uint32_t ws[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        const float b0 = __half2float(__ushort_as_half(static_cast<unsigned short>(ws[h] & 0xffffu)));
        const float b1 = __half2float(__ushort_as_half(static_cast<unsigned short>(ws[h] >> 16)));
        float &x0 = v[q * 8 + h * 2], &x1 = v[q * 8 + h * 2 + 1];
        x0 = e.bias_op == 1 ? b0 - x0 : x0 + b0;
        x1 = e.bias_op == 1 ? b1 - x1 : x1 + b1;
      }
    }
  } else if (e.bias_mode != 0) {
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      if (col0 + i < p.n) {
        const float b = load_bias(e, row, col0 + i);
        v[i] = e.bias_op == 1 ? b - v[i] : v[i] + b;
      }
    }
  }
  // The hardware tanh / exp approximations (~2^-11 relative) are used only
  // when the result is rounded to bf16 (8 mantissa bits) anyway; f32 and f16
  // outputs take CUDA's accurate tanhf / expf.
  const int act = kChain ? 0 : e.act;
  if (act != 0 && p.y_kind == kOutBf16) {
    if (act == 2) {
      // GELU-tanh on pairs: 0.5 x (1 + tanh(c0 x (1 + c1 x^2))) with packed
      // f32x2 multiplies/FMAs (half the FMA-pipe instructions) and the
      // hardware tanh.
      const uint64_t c0 = f2_pack(kGeluC0, kGeluC0), c1 = f2_pack(kGeluC1, kGeluC1);
      const uint64_t one = f2_pack(1.0f, 1.0f), half = f2_pack(0.5f, 0.5f);
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const uint64_t x = f2_pack(v[2 * i], v[2 * i + 1]);
        const uint64_t u = f2_mul(f2_mul(x, c0), f2_fma(f2_mul(x, x), c1, one));
        float u0, u1;
        f2_unpack(u, u0, u1);
        const uint64_t hx = f2_mul(x, half);
        f2_unpack(f2_fma(f2_pack(tanh_fast(u0), tanh_fast(u1)), hx, hx), v[2 * i], v[2 * i + 1]);
      }
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] = apply_act<true>(v[i], act);
    }
  } else if (act != 0) {
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = apply_act<false>(v[i], act);
  }
}

template <bool kChain>
__device__ __forceinline__ void epilogue_chunk(const Params &p, const uint32_t (&r)[32],
                                               int64_t row, int64_t col0,
                                               const uint4 *bias_smem = nullptr) {
  if (row >= p.m) return;
  float v[32];
  epilogue_values<kChain>(p, r, row, col0, bias_smem, v);
  const bool full_chunk = col0 + 32 <= p.n;
  if (p.y_kind == kOutF16) {
    __half *yr = reinterpret_cast<__half *>(p.y) + row * p.ld_y + col0;
    if (full_chunk) {
      uint4 *dst = reinterpret_cast<uint4 *>(yr);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        uint4 o;
        o.x = pack_f16x2(v[q * 8 + 0], v[q * 8 + 1]);
        o.y = pack_f16x2(v[q * 8 + 2], v[q * 8 + 3]);
        o.z = pack_f16x2(v[q * 8 + 4], v[q * 8 + 5]);
        o.w = pack_f16x2(v[q * 8 + 6], v[q * 8 + 7]);
        dst[q] = o;
      }
    } else {
      for (int i = 0; i < 32; ++i)
        if (col0 + i < p.n) yr[i] = __float2half_rn(v[i]);
    }
  } else if (p.y_kind == kOutBf16) {
    __nv_bfloat16 *yr = reinterpret_cast<__nv_bfloat16 *>(p.y) + row * p.ld_y + col0;
    if (full_chunk) {
      uint4 *dst = reinterpret_cast<uint4 *>(yr);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        uint4 o;
        o.x = pack_bf16x2(v[q * 8 + 0], v[q * 8 + 1]);
        o.y = pack_bf16x2(v[q * 8 + 2], v[q * 8 + 3]);
        o.z = pack_bf16x2(v[q * 8 + 4], v[q * 8 + 5]);
        o.w = pack_bf16x2(v[q * 8 + 6], v[q * 8 + 7]);
        dst[q] = o;
      }
    } else {
      for (int i = 0; i < 32; ++i)
        if (col0 + i < p.n) yr[i] = __float2bfloat16_rn(v[i]);
    }
  } else {
    float *yr = reinterpret_cast<float *>(p.y) + row * p.ld_y + col0;
    if (full_chunk) {
      float4 *dst = reinterpret_cast<float4 *>(yr);
#pragma unroll
      for (int q = 0; q < 8; ++q)
        dst[q] = make_float4(v[q * 4], v[q * 4 + 1], v[q * 4 + 2], v[q * 4 + 3]);
    } else {
      for (int i = 0; i < 32; ++i)
        if (col0 + i < p.n) yr[i] = v[i];
    }
  }
}

// One warp's 32 rows x 32 columns through shared memory: `stage` is the
// warp's 2 KiB buffer (512-byte aligned), written in the 64-byte-swizzled
// layout of the TMA box (16-byte piece q of row r at r * 64 + ((q ^ (r >> 1
// & 3)) << 4): four wavefronts per warp-wide 16-byte store), then lane 0
// issues the store of box (col0, row0). Rows past M and columns past N fall
// outside the tensor map and are not written. Per-row 16-byte global stores
// instead cost the load/store unit one L2 transaction per row and piece.
// With p.y_lsu (an output in another GPU's memory, which no tensor map may
// cover) the warp instead reads the buffer back transposed, lane l taking
// piece l & 3 of rows l / 4 + 8 i, so each st.global.v4 writes 8 rows x 64
// contiguous bytes; rows past M and columns past N are skipped.
template <int kYKind>
__device__ __forceinline__ void epilogue_chunk_tma(const Params &p, const uint32_t (&r)[32],
                                                   int64_t row, int64_t col0, int64_t row0,
                                                   const uint4 *bias_smem, uint8_t *stage,
                                                   const CUtensorMap *tmap_y, int lane) {
  float v[32];
  const bool live = row < p.m;
  if (live) epilogue_values<false>(p, r, row, col0, bias_smem, v);
  if (lane == 0 && !p.y_lsu) bulk_wait_read_all();  // the previous chunk's store has read the buffer
  __syncwarp();
  if (live) {
    uint8_t *dst = stage + lane * 64;
    const int sw = (lane >> 1) & 3;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      uint4 o;
      if constexpr (kYKind == kOutF16) {
        o.x = pack_f16x2(v[q * 8 + 0], v[q * 8 + 1]);
        o.y = pack_f16x2(v[q * 8 + 2], v[q * 8 + 3]);
        o.z = pack_f16x2(v[q * 8 + 4], v[q * 8 + 5]);
        o.w = pack_f16x2(v[q * 8 + 6], v[q * 8 + 7]);
      } else {
        o.x = pack_bf16x2(v[q * 8 + 0], v[q * 8 + 1]);
        o.y = pack_bf16x2(v[q * 8 + 2], v[q * 8 + 3]);
        o.z = pack_bf16x2(v[q * 8 + 4], v[q * 8 + 5]);
        o.w = pack_bf16x2(v[q * 8 + 6], v[q * 8 + 7]);
      }
      *reinterpret_cast<uint4 *>(dst + ((q ^ sw) << 4)) = o;
    }
  }
  if (p.y_lsu) {
    __syncwarp();
    const int q = lane & 3;
    uint16_t *y = reinterpret_cast<uint16_t *>(p.y);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int rr = (lane >> 2) + 8 * i;
      const int64_t grow = row0 + rr;
      const int64_t gcol = col0 + q * 8;
      if (grow < p.m && gcol < p.n) {
        const uint4 o =
            *reinterpret_cast<const uint4 *>(stage + rr * 64 + ((q ^ ((rr >> 1) & 3)) << 4));
        uint16_t *dst = y + grow * p.ld_y + gcol;
        if (gcol + 8 <= p.n) {
          *reinterpret_cast<uint4 *>(dst) = o;
        } else {
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const uint32_t w = e < 2 ? o.x : e < 4 ? o.y : e < 6 ? o.z : o.w;
            if (gcol + e < p.n) dst[e] = static_cast<uint16_t>(w >> ((e & 1) * 16));
          }
        }
      }
    }
    __syncwarp();  // every lane has read the buffer before the next chunk writes it
    return;
  }
  fence_async_smem();
  __syncwarp();
  if (lane == 0) {
    tma_store_2d(tmap_y, stage, static_cast<int32_t>(col0), static_cast<int32_t>(row0));
    bulk_commit();
  }
}

template <bool kChain>
__global__ void __launch_bounds__(THREADS, 1)
    gemm_tc_bf16_kernel(const __grid_constant__ CUtensorMap tmap_x,
                        const __grid_constant__ CUtensorMap tmap_w, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t *sa = smem;
  uint8_t *sb = smem + STAGES * A_BYTES;
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + STAGES * STAGE_BYTES);
  uint64_t *full = bars;
  uint64_t *empty = bars + STAGES;
  uint64_t *acc_full = bars + 2 * STAGES;
  uint64_t *acc_empty = acc_full + 2;
  uint64_t *drain = acc_empty + 2;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

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
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmap_x);
    tma_prefetch_desc(&tmap_w);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0 && !p.stall_loads) {
      int stage = 0;
      uint32_t phase = 0;
      for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x) {
        const int m0 = (tile / p.n_tiles) * BM;
        const int n0 = (tile % p.n_tiles) * BN;
        for (int kb = 0; kb < p.num_kb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, p.status, kErrTimeoutEmpty,
                         p.spin_limit))
            goto producer_done;
          mbar_arrive_expect_tx(&full[stage], STAGE_BYTES);
          tma_load_2d(sa + stage * A_BYTES, &tmap_x, &full[stage], kb * BK, m0);
          if (p.w_transposed) {
            tma_load_2d(sb + stage * B_BYTES, &tmap_w, &full[stage], kb * BK, n0);
          } else {
#pragma unroll
            for (int j = 0; j < BN / 64; ++j)
              tma_load_2d(sb + stage * B_BYTES + j * (64 * BK * 2), &tmap_w, &full[stage],
                          n0 + j * 64, kb * BK);
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
      const uint32_t fmt = p.in_f16 ? 0u : 1u;  // kind::f16 operand format: f16 0, bf16 1
      const uint32_t idesc = make_idesc(fmt, fmt, 0, p.w_transposed ? 0u : 1u, BM, BN);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x) {
        if (!mbar_wait(&acc_empty[acc], acc_phase ^ 1, abort_flag, p.status, kErrTimeoutAccum,
                       p.spin_limit))
          break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        bool ok = true;
        for (int kb = 0; kb < p.num_kb; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag, p.status, kErrTimeoutFull, p.spin_limit)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(sa + stage * A_BYTES);
          const uint32_t b_addr = smem_u32(sb + stage * B_BYTES);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            // K-major SW128: advancing K by 16 bf16 = 32 bytes inside the row.
            const uint64_t adesc = make_sdesc_sw128(a_addr + kk * 32, 16, 1024);
            // W^T is K-major like X. W itself is MN-major: 64-column chunks
            // are LBO = 64*BK*2 bytes apart, 8-row K groups SBO = 1024 apart,
            // and K advances by 16 rows = 2048 bytes.
            const uint64_t bdesc = p.w_transposed
                                       ? make_sdesc_sw128(b_addr + kk * 32, 16, 1024)
                                       : make_sdesc_sw128(b_addr + kk * 2048, 64 * BK * 2, 1024);
            mma_f16_ss(d_tmem, adesc, bdesc, idesc, (kb | kk) != 0 ? 1u : 0u);
          }
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
      // Drain: every MMA this thread issued must finish before TMEM is freed.
      mma_commit(drain);
      if (!mbar_wait(drain, 0, nullptr, p.status, kErrTimeoutDrain)) *abort_flag = 1;
    }
  } else {
    const int sub = warp & 3;  // TMEM lanes [32*sub, 32*sub+32)
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x) {
      const int64_t m0 = static_cast<int64_t>(tile / p.n_tiles) * BM;
      const int64_t n0 = static_cast<int64_t>(tile % p.n_tiles) * BN;
      if (!mbar_wait_warp(&acc_full[acc], acc_phase, abort_flag, p.status, kErrTimeoutAccum,
                          p.spin_limit))
        break;
      tc_fence_after();
      const int64_t row = m0 + sub * 32 + lane;
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(sub * 32) << 16) +
                             static_cast<uint32_t>(acc * BN);
#pragma unroll 1
      for (int c = 0; c < BN; c += 32) {
        if (n0 + c >= p.n) break;
        uint32_t r[32];
        tmem_ld32_sync(t_row + c, r);
        epilogue_chunk<kChain>(p, r, row, n0 + c);
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
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// ---- CTA-pair (2-SM) variant ---------------------------------------------------
// A cluster of two CTAs on two SMs computes a 256x256 tile with
// tcgen05.mma.cta_group::2 (M=256, N=256, K=16): CTA r holds rows
// [128r, 128r+128) of the X tile and columns [128r, 128r+128) of the W tile
// in its own shared memory, so each SM stages half of W per tile (B operand
// traffic per SM halves versus the single-SM kernel), and its TMEM receives
// its own 128 rows x 256 columns of the f32 accumulator. The leader CTA
// (rank 0) issues every MMA; both CTAs' TMA loads count on the leader's
// `full` barrier, MMA completion is committed to both CTAs' `empty` /
// `acc_full` barriers, and both epilogues release the leader's `acc_empty`.
// Eight epilogue warps per CTA (two per TMEM lane quarter, one 128-column
// half each) halve the epilogue time that the last tile of every CTA exposes.
constexpr int P_BN_CTA = BN / 2;  // W columns staged per CTA
constexpr int P_A_BYTES = BM * BK * 2;        // 16 KiB
constexpr int P_B_BYTES = P_BN_CTA * BK * 2;  // 16 KiB
constexpr int P_STAGE_BYTES = P_A_BYTES + P_B_BYTES;
constexpr int P_STAGES = 6;
// Epilogue warps: P_EPI_WARPS / 4 per TMEM lane quarter, each owning
// P_COLS_PER_WARP consecutive columns of the 256-column tile.
constexpr int P_EPI_WARPS = MCB_PAIR_EPI_WARPS;
constexpr int P_EPI_THREADS = P_EPI_WARPS * 32;
constexpr int P_COLS_PER_WARP = BN * 4 / P_EPI_WARPS;
constexpr int P_THREADS = 64 + P_EPI_THREADS;  // producer, MMA, epilogue warps
constexpr int P_BIAS_BYTES = P_EPI_WARPS * P_COLS_PER_WARP * 2;  // per warp: its bf16 bias slice
constexpr int P_YST_BYTES = P_EPI_WARPS * 2048;  // per warp: 32 rows x 32 16-bit outputs
constexpr int P_YST_OFF = P_STAGES * P_STAGE_BYTES;  // 1024-aligned
constexpr int P_BAR_OFF = P_YST_OFF + P_YST_BYTES;
constexpr size_t P_SMEM_BYTES =
    static_cast<size_t>(P_BAR_OFF) + BAR_BYTES + P_BIAS_BYTES + 1024;

// ---- stream-K work split ----------------------------------------------------------
// Tiles [0, sk_first_tile) run whole, cluster c taking c, c + G, ... The last
// sk_tiles tiles (fewer than the G clusters) are split in chains: chain i
// holds k consecutive tiles and k + 1 consecutive clusters, and its k * KB
// K-block iterations are cut at k boundaries b_1 < ... < b_k, one strictly
// inside each tile (b_j in tile j - 1). Cluster j of the chain computes the
// tail of tile j - 1 (from b_j) first and the head of tile j (up to b_{j+1})
// last; every split tile thus has exactly two parts, its tail finished early
// by the next cluster and its head finished last by its owner. The owner's
// producer fetches the tail's partial accumulator into the freed stages of
// its ring while its last MMAs run, and its epilogue adds it in. The last
// cluster of a chain holds only a tail that is also computed last, so its
// share is `sk_w` K blocks x k/(k+1) shorter (the time its partial takes to
// write), the other clusters' shares 1/k of that longer.
enum : int { kUnitWhole = 0, kUnitTail = 1, kUnitHead = 2 };
struct Unit {
  int tile, kb0, kb1, role, sk_tile;  // sk_tile: index among the split tiles
};
constexpr int64_t kSlotFloats = 2 * BM * BN / 2;  // 128 rows x 256 columns per CTA

struct ChainPos {
  int t0, k, j;  // chain's first split tile, tiles in the chain, cluster within it
};
// Chain position of stream-K cluster c (false: c takes no stream-K work).
__host__ __device__ inline bool sk_chain_pos(int sk_tiles, int chains, int c, ChainPos &cp) {
  if (chains <= 0 || c >= sk_tiles + chains) return false;
  const int kq = sk_tiles / chains, kr = sk_tiles % chains;
  const int big = kr * (kq + 2);  // clusters of the kr chains of kq + 1 tiles
  int i;
  if (c < big) {
    i = c / (kq + 2);
    cp.j = c % (kq + 2);
    cp.k = kq + 1;
  } else {
    i = kr + (c - big) / (kq + 1);
    cp.j = (c - big) % (kq + 1);
    cp.k = kq;
  }
  cp.t0 = i * kq + (i < kr ? i : kr);
  return true;
}
// Boundary b_jj (1 <= jj <= k) of a chain of k tiles of kb K blocks each.
__host__ __device__ inline int sk_boundary(int k, int kb, int w, int jj) {
  const int delta = (w * k + k) / (k + 1);  // ceil(w * k / (k + 1))
  const int last = k * kb / (k + 1) - delta;  // the last cluster's share
  return static_cast<int>(static_cast<int64_t>(jj) * (k * kb - last) / k);
}

// Units of one cluster in order: its whole tiles, then its tail and head
// parts. Producer, MMA and epilogue walk the same sequence.
struct UnitIter {
  int tile, phase;  // phase: 0 whole tiles, 1 tail, 2 head, 3 done
  ChainPos cp;
  bool in_sk;
  __device__ UnitIter(const Params &p, int cluster, int g) : tile(cluster), phase(0) {
    in_sk = sk_chain_pos(p.sk_tiles, p.sk_chains, cluster, cp);
  }
  __device__ bool next(const Params &p, int g, Unit &u) {
    if (phase == 0) {
      if (tile < p.sk_first_tile) {
        u = {tile, 0, p.num_kb, kUnitWhole, -1};
        tile += g;
        return true;
      }
      phase = in_sk ? 1 : 3;
    }
    if (phase == 1) {
      phase = 2;
      if (cp.j > 0) {  // tail of split tile t0 + j - 1
        const int t = cp.t0 + cp.j - 1;
        const int b = sk_boundary(cp.k, p.num_kb, p.sk_w, cp.j) - (cp.j - 1) * p.num_kb;
        u = {p.sk_first_tile + t, b, p.num_kb, kUnitTail, t};
        return true;
      }
    }
    if (phase == 2) {
      phase = 3;
      if (cp.j < cp.k) {  // head of split tile t0 + j (owner)
        const int t = cp.t0 + cp.j;
        const int b = sk_boundary(cp.k, p.num_kb, p.sk_w, cp.j + 1) - cp.j * p.num_kb;
        u = {p.sk_first_tile + t, 0, b, kUnitHead, t};
        return true;
      }
    }
    return false;
  }
};

// Global flag of one split tile's tail part (per CTA rank): written with
// release semantics at GPU scope once the partial is in memory, read with
// acquire by the owner's producer.
__device__ __forceinline__ void flag_release_gpu(int *f, int v) {
  asm volatile("st.release.gpu.global.b32 [%0], %1;" ::"l"(f), "r"(v) : "memory");
}
__device__ __forceinline__ int flag_acquire_gpu(const int *f) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(f) : "memory");
  return v;
}
// 16 KiB piece of a partial slot into shared memory, counted on `bar`.
__device__ __forceinline__ void bulk_load_g2s(void *smem_dst, const void *src, uint32_t bytes,
                                              uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(smem_u32(smem_dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// kSK: the stream-K instantiation. Its epilogue warps agree on every
// pipeline wait through a CTA barrier (all leave together on a timeout).
// The one wait on another cluster is an owner's producer waiting (bounded by
// spin_limit) for the flag of its tile's tail part, which the next cluster
// computes as its first unit and never waits for anything itself.
template <bool kChain, bool kSK>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(P_THREADS, 1)
    gemm_tc_bf16_pair_kernel(const __grid_constant__ CUtensorMap tmap_x,
                             const __grid_constant__ CUtensorMap tmap_w,
                             const __grid_constant__ CUtensorMap tmap_y, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t *sa = smem;
  uint8_t *sb = smem + P_STAGES * P_A_BYTES;
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + P_BAR_OFF);
  uint64_t *full = bars;
  uint64_t *empty = bars + P_STAGES;
  uint64_t *acc_full = bars + 2 * P_STAGES;
  uint64_t *acc_empty = acc_full + 2;
  uint64_t *drain = acc_empty + 2;
  uint64_t *part_full = drain + 1;  // stream-K: the tail's partial is in the ring
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(part_full + 1);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);
  volatile int *part_stage = reinterpret_cast<volatile int *>(tmem_slot + 2);  // 4 ring stages

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int cluster = blockIdx.x >> 1;
  const int nclusters = gridDim.x >> 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < P_STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 2 * P_EPI_WARPS);  // epilogue warps of both CTAs (leader's copy)
    }
    mbar_init(drain, 1);
    mbar_init(part_full, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmap_x);
    tma_prefetch_desc(&tmap_w);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncwarp();
  cluster_sync();  // barriers initialised and TMEM allocated in both CTAs
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // Set-up above overlaps the previous kernel's tail when this launch is
  // programmatic. Before the dependency wait only L2 prefetches are issued
  // (hints: they read nothing into the SM and cannot return stale data):
  // the first P_STAGES K blocks of this CTA's first tile, so the first loads
  // after the wait hit L2 instead of HBM.
  if (warp == 0 && lane == 0) {
    UnitIter first(p, cluster, nclusters);
    Unit u0;
    if (!first.next(p, nclusters, u0)) u0 = {0, 0, 0, kUnitWhole, -1};
    const int m0 = (u0.tile / p.n_tiles) * (2 * BM) + static_cast<int>(rank) * BM;
    const int n0 = (u0.tile % p.n_tiles) * BN + static_cast<int>(rank) * P_BN_CTA;
    for (int kb = u0.kb0; kb < u0.kb0 + P_STAGES && kb < u0.kb1; ++kb) {
      tma_prefetch_l2_2d(&tmap_x, kb * BK, m0);
      if (p.w_transposed) {
        tma_prefetch_l2_2d(&tmap_w, kb * BK, n0);
      } else {
#pragma unroll
        for (int j = 0; j < P_BN_CTA / 64; ++j) tma_prefetch_l2_2d(&tmap_w, n0 + j * 64, kb * BK);
      }
    }
  }
  grid_dependency_wait();
  grid_launch_dependents();

  if (warp == 0) {
    if (lane == 0) {
      const uint32_t full_leader0 = mapa_shared(smem_u32(&full[0]), 0);
      int stage = 0;
      uint32_t phase = 0;
      UnitIter units(p, cluster, nclusters);
      Unit u;
      while (units.next(p, nclusters, u)) {
        const int m0 = (u.tile / p.n_tiles) * (2 * BM) + static_cast<int>(rank) * BM;
        const int n0 = (u.tile % p.n_tiles) * BN + static_cast<int>(rank) * P_BN_CTA;
        for (int kb = u.kb0; kb < u.kb1; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, p.status, kErrTimeoutEmpty,
                         p.spin_limit))
            goto producer_done;
          const uint32_t fbar = full_leader0 + stage * 8;
          if (leader) mbar_arrive_expect_tx(&full[stage], 2 * P_STAGE_BYTES);
          tma_load_2d_pair(sa + stage * P_A_BYTES, &tmap_x, fbar, kb * BK, m0);
          if (p.w_transposed) {
            tma_load_2d_pair(sb + stage * P_B_BYTES, &tmap_w, fbar, kb * BK, n0);
          } else {
#pragma unroll
            for (int j = 0; j < P_BN_CTA / 64; ++j)
              tma_load_2d_pair(sb + stage * P_B_BYTES + j * (64 * BK * 2), &tmap_w, fbar,
                               n0 + j * 64, kb * BK);
          }
          if (++stage == P_STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if constexpr (kSK) {
          if (u.role == kUnitHead) {
            // The owner's last unit: once the tail's flag is up, fetch its
            // partial (this CTA's 128 rows, 128 KiB) into the next four ring
            // stages as the MMAs free them. The stages are fixed first, then
            // published by the expect-tx arrival the epilogue acquires.
            const int *flag = p.sk_flag + u.sk_tile * 2 + rank;
            const long long t0 = clock64();
            while (flag_acquire_gpu(flag) != 1) {
              if (*abort_flag) goto producer_done;
              if (clock64() - t0 > p.spin_limit) {
                atomicOr(p.status, kErrTimeoutPeer);
                *abort_flag = 1;
                goto producer_done;
              }
            }
            asm volatile("fence.proxy.async.global;" ::: "memory");
            const float *slot = p.sk_part + (static_cast<int64_t>(cluster + 1) * 2 + rank) * kSlotFloats;
            for (int i = 0; i < 4; ++i) part_stage[i] = (stage + i) % P_STAGES;
            mbar_arrive_expect_tx(part_full, 4 * P_STAGE_BYTES);
            for (int i = 0; i < 4; ++i) {
              if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, p.status, kErrTimeoutEmpty,
                             p.spin_limit))
                goto producer_done;
              bulk_load_g2s(sa + stage * P_A_BYTES, slot + (2 * i) * (P_A_BYTES / 4), P_A_BYTES,
                            part_full);
              bulk_load_g2s(sb + stage * P_B_BYTES, slot + (2 * i + 1) * (P_B_BYTES / 4),
                            P_B_BYTES, part_full);
              if (++stage == P_STAGES) {
                stage = 0;
                phase ^= 1;
              }
            }
            // The copies must have landed before the block can exit.
            mbar_wait(part_full, 0, abort_flag, p.status, kErrTimeoutPeer, p.spin_limit);
          }
        }
      }
    producer_done:;
    }
  } else if (warp == 1) {
    if (leader && lane == 0) {
      const uint32_t fmt = p.in_f16 ? 0u : 1u;  // kind::f16 operand format: f16 0, bf16 1
      const uint32_t idesc = make_idesc(fmt, fmt, 0, p.w_transposed ? 0u : 1u, 2 * BM, BN);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      UnitIter units(p, cluster, nclusters);
      Unit u;
      while (units.next(p, nclusters, u)) {
        if (!mbar_wait(&acc_empty[acc], acc_phase ^ 1, abort_flag, p.status, kErrTimeoutAccum,
                       p.spin_limit))
          break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        bool ok = true;
        for (int kb = u.kb0; kb < u.kb1; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag, p.status, kErrTimeoutFull, p.spin_limit)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(sa + stage * P_A_BYTES);
          const uint32_t b_addr = smem_u32(sb + stage * P_B_BYTES);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            const uint64_t adesc = make_sdesc_sw128(a_addr + kk * 32, 16, 1024);
            const uint64_t bdesc = p.w_transposed
                                       ? make_sdesc_sw128(b_addr + kk * 32, 16, 1024)
                                       : make_sdesc_sw128(b_addr + kk * 2048, 64 * BK * 2, 1024);
            mma_f16_ss_pair(d_tmem, adesc, bdesc, idesc, (kb != u.kb0 || kk != 0) ? 1u : 0u);
          }
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
    const int cbeg = ((warp - 2) >> 2) * P_COLS_PER_WARP;  // this warp's columns of the tile
    const uint32_t acc_empty_leader = mapa_shared(smem_u32(&acc_empty[0]), 0);
    uint8_t *bias_slice = smem + P_BAR_OFF + BAR_BYTES + (warp - 2) * P_COLS_PER_WARP * 2;
    uint8_t *y_stage = smem + P_YST_OFF + (warp - 2) * 2048;
    int acc = 0;
    uint32_t acc_phase = 0;
    UnitIter units(p, cluster, nclusters);
    Unit u;
    while (units.next(p, nclusters, u)) {
      const int64_t m0 = static_cast<int64_t>(u.tile / p.n_tiles) * (2 * BM) + rank * BM;
      const int64_t n0 = static_cast<int64_t>(u.tile % p.n_tiles) * BN;
      // Stage this warp's 128-column slice of a row-broadcast bf16 bias in
      // shared memory while the tile's MMAs still run (lane l: 4 columns).
      const uint4 *bias_sm = nullptr;
      if constexpr (!kChain) {
        const Epilogue &e = p.epi;
        if (e.bias_mode == 1 && e.bias_bf16 && e.bias_aligned16 &&
            n0 + cbeg + P_COLS_PER_WARP <= p.n) {
          // lane l stages bytes [l * B, l * B + B) of the slice, B = 2 * cols / 32
          using Piece = typename std::conditional<P_COLS_PER_WARP == 128, uint2, uint32_t>::type;
          const Piece bv = __ldg(reinterpret_cast<const Piece *>(
                                     reinterpret_cast<const __nv_bfloat16 *>(e.bias) + n0 + cbeg) +
                                 lane);
          __syncwarp();  // the previous tile's reads of the slice are done
          reinterpret_cast<Piece *>(bias_slice)[lane] = bv;
          __syncwarp();
          bias_sm = reinterpret_cast<const uint4 *>(bias_slice);
        }
      }
      const bool ok = mbar_wait_warp(&acc_full[acc], acc_phase, abort_flag, p.status,
                                     kErrTimeoutAccum, p.spin_limit);
      if constexpr (kSK) {
        if (named_bar_or(1, P_EPI_THREADS, !ok)) break;  // every epilogue warp leaves together
      } else {
        if (!ok) break;
      }
      tc_fence_after();
      const int64_t row = m0 + sub * 32 + lane;
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(sub * 32) << 16) +
                             static_cast<uint32_t>(acc * BN);
      if (!kSK || u.role != kUnitTail) {
        bool have_part = false;  // stream-K owner: the tail's partial sits in the ring
        if constexpr (kSK) {
          if (u.role == kUnitHead) {
            const bool okp = mbar_wait_warp(part_full, 0, abort_flag, p.status, kErrTimeoutPeer,
                                            p.spin_limit);
            if (named_bar_or(1, P_EPI_THREADS, !okp)) break;
            have_part = true;
          }
        }
#pragma unroll 1
        for (int c = cbeg; c < cbeg + P_COLS_PER_WARP; c += 32) {
          if (n0 + c >= p.n) break;
          uint32_t r[32];
          tmem_ld32_sync(t_row + c, r);
          if constexpr (kSK) {
            if (have_part) {
              // Chunk c / 32 of the slot is one 16 KiB piece: ring stage
              // part_stage[piece / 2], its A half for even pieces, B for odd.
              const int piece = c >> 5;
              const int st = part_stage[piece >> 1];
              const float4 *src =
                  reinterpret_cast<const float4 *>(piece & 1 ? sb + st * P_B_BYTES
                                                             : sa + st * P_A_BYTES) +
                  sub * 32 + lane;
#pragma unroll
              for (int q = 0; q < 8; ++q) {
                const float4 f = src[q * BM];
                r[4 * q] = __float_as_uint(__uint_as_float(r[4 * q]) + f.x);
                r[4 * q + 1] = __float_as_uint(__uint_as_float(r[4 * q + 1]) + f.y);
                r[4 * q + 2] = __float_as_uint(__uint_as_float(r[4 * q + 2]) + f.z);
                r[4 * q + 3] = __float_as_uint(__uint_as_float(r[4 * q + 3]) + f.w);
              }
            }
          }
          const uint4 *bias_c = bias_sm ? bias_sm + ((c - cbeg) >> 3) : nullptr;
          if (!kChain && p.y_tma == kOutBf16)
            epilogue_chunk_tma<kOutBf16>(p, r, row, n0 + c, m0 + sub * 32, bias_c, y_stage,
                                         &tmap_y, lane);
          else if (!kChain && p.y_tma == kOutF16)
            epilogue_chunk_tma<kOutF16>(p, r, row, n0 + c, m0 + sub * 32, bias_c, y_stage,
                                        &tmap_y, lane);
          else
            epilogue_chunk<kChain>(p, r, row, n0 + c, bias_c);
        }
        // The copies have read the slot (part_full completed): the flag is
        // ready for the next launch.
        if (have_part && warp == 2 && lane == 0) p.sk_flag[u.sk_tile * 2 + rank] = 0;
      } else {
        // Tail part: its accumulator goes to this cluster's slot. Layout:
        // float4 q of chunk (32 columns) c for row r at (c * 8 + q) * 128 + r,
        // so a warp-wide float4 store covers 512 contiguous bytes and chunk c
        // is 16 KiB at c * 16 KiB. The CTA barrier orders every thread's
        // stores before the flag's release at GPU scope.
        const int r_local = sub * 32 + lane;
        float4 *mine = reinterpret_cast<float4 *>(
            p.sk_part + (static_cast<int64_t>(cluster) * 2 + rank) * kSlotFloats);
#pragma unroll 1
        for (int c = cbeg; c < cbeg + P_COLS_PER_WARP; c += 32) {
          uint32_t r[32];
          tmem_ld32_sync(t_row + c, r);
#pragma unroll
          for (int q = 0; q < 8; ++q)
            mine[((c >> 5) * 8 + q) * BM + r_local] =
                make_float4(__uint_as_float(r[4 * q]), __uint_as_float(r[4 * q + 1]),
                            __uint_as_float(r[4 * q + 2]), __uint_as_float(r[4 * q + 3]));
        }
        named_bar_sync(1, P_EPI_THREADS);
        if (warp == 2 && lane == 0 && !p.sk_test_no_release)
          flag_release_gpu(p.sk_flag + u.sk_tile * 2 + rank, 1);
      }
      tc_fence_before();
      mbar_arrive_cluster_warp(acc_empty_leader + acc * 8);
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1;
    }
    // The TMA stores must finish reading shared memory (and land) before
    // the block exits.
    if (p.y_tma && !p.y_lsu && lane == 0) bulk_wait_all();
  }

  tc_fence_before();
  __syncwarp();
  cluster_sync();  // every pair MMA has completed before either CTA frees TMEM
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, TMEM_COLS);
  }
}

}  // namespace

namespace {

// Clusters of the pair kernel that fit on the device at once (one CTA per SM;
// a GPC with an odd number of usable SMs leaves one SM out), cached per device.
int pair_clusters_resident(int device) {
  static std::atomic<int> cache[64];
  if (device < 0 || device >= 64) return 0;
  int v = cache[device].load(std::memory_order_relaxed);
  if (v != 0) return v;
  if (cudaFuncSetAttribute(gemm_tc_bf16_pair_kernel<false, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(P_SMEM_BYTES)) != cudaSuccess) {
    (void)cudaGetLastError();
    cache[device].store(-1, std::memory_order_relaxed);
    return -1;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2, 1, 1);
  cfg.blockDim = dim3(P_THREADS, 1, 1);
  cfg.dynamicSmemBytes = P_SMEM_BYTES;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, gemm_tc_bf16_pair_kernel<false, false>, &cfg) != cudaSuccess ||
      n <= 0) {
    (void)cudaGetLastError();
    n = -1;  // pair kernel unavailable on this device: use the single-SM kernel
  }
  cache[device].store(n, std::memory_order_relaxed);
  return n;
}

bool pair_kernel_enabled() {
  static const bool on = [] {
    const char *e = getenv("MCB_GEMM_TC_PAIR");
    return !(e && e[0] == '0');
  }();
  return on;
}

// Programmatic dependent launch of the CTA-pair kernel; MCB_GEMM_PDL=0 turns
// it off (A/B measurement).
bool pdl_enabled() {
  static const bool on = [] {
    const char *e = getenv("MCB_GEMM_PDL");
    return !(e && e[0] == '0');
  }();
  return on;
}

// Stream-K mode, read at every launch: MCB_GEMM_STREAM_K=0 never, =1
// whenever it cuts the busiest cluster's K blocks by 5% (tests and
// measurement), unset: only when the last wave fills at most 70% of the
// clusters. Measured on B200 (back to back, bias + GELU, K = N = 4096, 74
// clusters; rows: tiles in the last wave, stream-K vs whole tiles): 256: 4,
// 24.2 vs 29.0 us; 768: 48, 28.2 vs 31.2; 3072: 44, 80.0 vs 83.0; 4096: 34,
// 112.4 vs 118.7; 6144: 14, 166.1 vs 173.0; but 2048: 54, 53.7 vs 53.1 and
// 1024: 64, 32.5 vs 30.8. A nearly full last wave already runs at the
// power-capped clock the whole GPU's tensor throughput sets, so its few idle
// clusters cost little.
int stream_k_mode() {
  const char *e = getenv("MCB_GEMM_STREAM_K");
  if (!e || !e[0]) return 2;
  return e[0] == '1' ? 1 : 0;
}

// K blocks the last cluster of a stream-K chain gives up so that its
// partial (written last) is in memory when its owner needs it: ~2.5 us of
// partial write at ~0.38 us per 256x256x64 pair K block.
constexpr int kSkW = 7;

// The largest K-block load of any stream-K cluster (its share of the split
// tiles), or -1 when a chain would have an empty part (every boundary must
// lie strictly inside its tile).
int sk_max_share(int sk_tiles, int chains, int kb, int w) {
  const int kq = sk_tiles / chains;
  int worst = 0;
  for (int k : {kq, kq + 1}) {
    if (k < 1 || (k == kq + 1 && sk_tiles % chains == 0)) continue;
    int prev = 0;
    for (int jj = 1; jj <= k; ++jj) {
      const int b = sk_boundary(k, kb, w, jj);
      if (b <= (jj - 1) * kb || b >= jj * kb) return -1;
      worst = std::max(worst, b - prev);
      prev = b;
    }
    if (k * kb - prev < 1) return -1;
    worst = std::max(worst, k * kb - prev);
  }
  return worst;
}

// TMA-staged output stores in the CTA-pair kernel (16-bit outputs with
// 16-byte aligned rows); MCB_GEMM_Y_TMA=0 (read at every launch) turns them
// off, for measurement.
bool y_tma_enabled() {
  const char *e = getenv("MCB_GEMM_Y_TMA");
  return !(e && e[0] == '0');
}

}  // namespace

cudaError_t launch_gemm_tc_bf16(const void *x, const void *w, void *y, int64_t m, int64_t n,
                                int64_t k, int64_t ld_x, int64_t ld_w, int64_t ld_y,
                                int w_transposed, int y_kind, const Epilogue &epi,
                                uint32_t *status, int sms, cudaStream_t stream, LaunchInfo *info,
                                int in_f16, const GemmStreamK *sk, int no_tma_store) {
  if (m == 0 || n == 0) return cudaSuccess;
  const bool chain = epi.n_ops > 0;
  // Rows of 256 go to CTA pairs (M = 256 per MMA, W tile split between the
  // two SMs); shorter problems keep one 128-row tile per SM.
  int device = 0;
  cudaError_t e = cudaGetDevice(&device);
  if (e != cudaSuccess) return e;
  const bool pair = m >= 2 * BM && pair_kernel_enabled() && pair_clusters_resident(device) > 0;
  if (pair) {
    for (auto *kernel : {gemm_tc_bf16_pair_kernel<true, false>, gemm_tc_bf16_pair_kernel<false, false>,
                         gemm_tc_bf16_pair_kernel<false, true>}) {
      e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(P_SMEM_BYTES));
      if (e != cudaSuccess) return e;
    }
  }
  const int w_rows = pair ? P_BN_CTA : BN;  // W^T box height per CTA
  CUtensorMap tx, tw;
  const CUtensorMapDataType dt =
      in_f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  if (!encode_tmap_2d(&tx, dt, x, k, m, ld_x * 2, BK, BM, CU_TENSOR_MAP_SWIZZLE_128B))
    return cudaErrorInvalidValue;
  const bool ok_w =
      w_transposed
          ? encode_tmap_2d(&tw, dt, w, k, n, ld_w * 2, BK, w_rows, CU_TENSOR_MAP_SWIZZLE_128B)
          : encode_tmap_2d(&tw, dt, w, n, k, ld_w * 2, 64, BK, CU_TENSOR_MAP_SWIZZLE_128B);
  if (!ok_w) return cudaErrorInvalidValue;
  CUtensorMap ty;
  memset(&ty, 0, sizeof(ty));
  int y_tma = 0;
  if (pair && !chain && (y_kind == kOutBf16 || y_kind == kOutF16) &&
      reinterpret_cast<uintptr_t>(y) % 16 == 0 && (ld_y * 2) % 16 == 0 && y_tma_enabled()) {
    // no_tma_store (y in another GPU's memory): staged chunks, coalesced
    // st.global, no tensor map over y.
    if (!no_tma_store &&
        !encode_tmap_2d(&ty, y_kind == kOutF16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                               : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                        y, n, m, ld_y * 2, 32, 32, CU_TENSOR_MAP_SWIZZLE_64B))
      return cudaErrorInvalidValue;
    y_tma = y_kind;
  }
  Params p;
  p.m = m;
  p.n = n;
  p.k = k;
  p.ld_y = ld_y;
  p.n_tiles = static_cast<int>((n + BN - 1) / BN);
  const int64_t tile_rows = pair ? 2 * BM : BM;
  const int64_t tiles = ((m + tile_rows - 1) / tile_rows) * p.n_tiles;
  if (tiles > 0x7fffffff) return cudaErrorInvalidConfiguration;
  p.num_tiles = static_cast<int>(tiles);
  p.num_kb = static_cast<int>((k + BK - 1) / BK);
  p.w_transposed = w_transposed;
  p.y_kind = y_kind;
  p.in_f16 = in_f16;
  p.y = y;
  p.status = status;
  p.spin_limit = kSpinTimeoutCycles;
  p.stall_loads = 0;
  p.y_tma = y_tma;
  p.y_lsu = y_tma && no_tma_store ? 1 : 0;
  p.sk_first_tile = p.num_tiles;  // whole tiles only unless stream-K applies below
  p.sk_tiles = 0;
  p.sk_chains = 0;
  p.sk_w = kSkW;
  p.sk_flag = nullptr;
  p.sk_part = nullptr;
  p.sk_test_no_release = 0;
  p.epi = epi;
  int grid;
  bool use_sk = false;
  if (pair) {
    int clusters = pair_clusters_resident(device);
    if (clusters > sms / 2) clusters = sms / 2;
    if (clusters < 1) clusters = 1;
    // Stream-K when the last wave leaves clusters idle (4096 rows: 34 tiles
    // on 74 clusters): every full wave stays whole-tile and the last wave's
    // tiles are split in chains.
    const int sk_mode = stream_k_mode();
    if (sk && !chain && sk->flags && sk->part && clusters <= sk->clusters && sk_mode != 0) {
      const int64_t g = clusters;
      const int64_t waves = (tiles + g - 1) / g;
      const int64_t dp = (waves - 1) * g;
      const int64_t skt = tiles - dp;  // 1..g
      const int64_t chains = std::min(g - skt, skt);
      const int share = chains >= 1 ? sk_max_share(static_cast<int>(skt), static_cast<int>(chains),
                                                   p.num_kb, kSkW)
                                    : -1;
      // Worth it when the busiest cluster's K blocks drop by 5% or more
      // (and, by default, when the last wave is at most 70% full).
      if (share > 0 && skt <= sk->max_tiles &&
          ((waves - 1) * p.num_kb + share) * 100 <= waves * p.num_kb * 95 &&
          (sk_mode == 1 || 10 * skt <= 7 * g)) {
        use_sk = true;
        p.sk_first_tile = static_cast<int>(dp);
        p.sk_tiles = static_cast<int>(skt);
        p.sk_chains = static_cast<int>(chains);
        p.sk_flag = sk->flags;
        p.sk_part = sk->part;
      }
    }
    grid = 2 * static_cast<int>(use_sk ? clusters : (tiles < clusters ? tiles : clusters));
    // Programmatic stream serialization: the kernel's set-up (barriers, TMEM
    // allocation, L2 prefetches) may start while the previous kernel in the
    // stream drains; the kernel waits for it before its first load or store.
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(grid), 1, 1);
    cfg.blockDim = dim3(P_THREADS, 1, 1);
    cfg.dynamicSmemBytes = P_SMEM_BYTES;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (chain)
      e = cudaLaunchKernelEx(&cfg, gemm_tc_bf16_pair_kernel<true, false>, tx, tw, ty, p);
    else if (use_sk)
      e = cudaLaunchKernelEx(&cfg, gemm_tc_bf16_pair_kernel<false, true>, tx, tw, ty, p);
    else
      e = cudaLaunchKernelEx(&cfg, gemm_tc_bf16_pair_kernel<false, false>, tx, tw, ty, p);
    if (e != cudaSuccess) return e;
  } else {
    // Per-device function attribute; cheap, so set on every launch.
    e = cudaFuncSetAttribute(chain ? gemm_tc_bf16_kernel<true> : gemm_tc_bf16_kernel<false>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(SMEM_BYTES));
    if (e != cudaSuccess) return e;
    grid = static_cast<int>(tiles < sms ? tiles : sms);
    if (chain)
      gemm_tc_bf16_kernel<true><<<grid, THREADS, SMEM_BYTES, stream>>>(tx, tw, p);
    else
      gemm_tc_bf16_kernel<false><<<grid, THREADS, SMEM_BYTES, stream>>>(tx, tw, p);
  }
  if (info) {
    info->launches = 1;
    info->tile_m = static_cast<int>(tile_rows);
    info->tile_n = BN;
    info->tile_k = BK;
    info->stages = pair ? P_STAGES : STAGES;
    info->ctas = grid;
    info->stream_k = use_sk;
    info->set_route(in_f16 ? "tcgen05_f16_gemm_epilogue" : "tcgen05_bf16_gemm_epilogue");
  }
  return cudaGetLastError();
}

// Self-test of the bounded waits: one single-SM GEMM tile (128x64 . 64x256)
// whose producer issues no loads, so the MMA thread's wait for the first
// stage must run out after `spin_limit` cycles, record kErrTimeoutFull in
// *status and abort the CTA (the epilogue warps leave through the abort
// flag, TMEM is freed). x must hold 128x64 and w 64x256 16-byte-aligned bf16
// elements (they are never read), y 128x256 bf16 (never written).
cudaError_t launch_gemm_tc_stall_selftest(const void *x, const void *w, void *y,
                                          long long spin_limit, uint32_t *status,
                                          cudaStream_t stream) {
  CUtensorMap tx, tw;
  if (!encode_tmap_2d(&tx, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, x, BK, BM, BK * 2, BK, BM,
                      CU_TENSOR_MAP_SWIZZLE_128B) ||
      !encode_tmap_2d(&tw, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, w, BN, BK, BN * 2, 64, BK,
                      CU_TENSOR_MAP_SWIZZLE_128B))
    return cudaErrorInvalidValue;
  Params p = {};
  p.m = BM;
  p.n = BN;
  p.k = BK;
  p.ld_y = BN;
  p.n_tiles = 1;
  p.num_tiles = 1;
  p.num_kb = 1;
  p.y_kind = kOutBf16;
  p.y = y;
  p.status = status;
  p.spin_limit = spin_limit;
  p.stall_loads = 1;
  cudaError_t e = cudaFuncSetAttribute(gemm_tc_bf16_kernel<false>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(SMEM_BYTES));
  if (e != cudaSuccess) return e;
  gemm_tc_bf16_kernel<false><<<1, THREADS, SMEM_BYTES, stream>>>(tx, tw, p);
  return cudaGetLastError();
}

// Self-test of the one wait on another cluster: a stream-K launch of two
// 256x256 tiles (K = 4096: chains of one tile over two clusters) whose tails
// never raise their flags, so each owner's producer gives up after
// `spin_limit` cycles, records kErrTimeoutPeer and aborts its CTA; the
// owner's epilogue leaves through its own bounded wait, the tails finish
// normally. x: 256x4096, w: 4096x512 bf16 (16-byte aligned, never needed
// valid), y: 256x512 bf16; `part` 4 clusters x 2 ranks x 128 KiB, `flags`
// 4 ints, zero.
cudaError_t launch_gemm_tc_peer_stall_selftest(const void *x, const void *w, void *y, float *part,
                                               int *flags, long long spin_limit, uint32_t *status,
                                               cudaStream_t stream) {
  constexpr int kM = 256, kN = 512, kK = 4096;
  CUtensorMap tx, tw, ty;
  memset(&ty, 0, sizeof(ty));
  if (!encode_tmap_2d(&tx, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, x, kK, kM, kK * 2, BK, BM,
                      CU_TENSOR_MAP_SWIZZLE_128B) ||
      !encode_tmap_2d(&tw, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, w, kN, kK, kN * 2, 64, BK,
                      CU_TENSOR_MAP_SWIZZLE_128B))
    return cudaErrorInvalidValue;
  Params p = {};
  p.m = kM;
  p.n = kN;
  p.k = kK;
  p.ld_y = kN;
  p.n_tiles = kN / BN;
  p.num_tiles = p.n_tiles;
  p.num_kb = kK / BK;
  p.y_kind = kOutBf16;
  p.y = y;
  p.status = status;
  p.spin_limit = spin_limit;
  p.sk_first_tile = 0;
  p.sk_tiles = p.num_tiles;
  p.sk_chains = p.num_tiles;
  p.sk_w = kSkW;
  p.sk_flag = flags;
  p.sk_part = part;
  p.sk_test_no_release = 1;
  if (sk_max_share(p.sk_tiles, p.sk_chains, p.num_kb, kSkW) <= 0) return cudaErrorInvalidValue;
  cudaError_t e = cudaFuncSetAttribute(gemm_tc_bf16_pair_kernel<false, true>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(P_SMEM_BYTES));
  if (e != cudaSuccess) return e;
  const int clusters = p.sk_tiles + p.sk_chains;  // chains of one tile: two clusters each
  gemm_tc_bf16_pair_kernel<false, true><<<2 * clusters, P_THREADS, P_SMEM_BYTES, stream>>>(
      tx, tw, ty, p);
  return cudaGetLastError();
}

}  // namespace mcb

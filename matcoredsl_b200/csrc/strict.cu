// Strict f32 kernels on CUDA cores, bit-exact with MatcoreDSL's strict leaf.
//
// Arithmetic contract (compiler/lib/runtime/closed_host_v1.cpp:401-415 and
// compiler/lib/mlir/MatcoreCpuFusedGemmCandidate.h:19-31): every output is a
// reduction in increasing index order from a +0 seed, each step one binary32
// multiply rounded on its own followed by one binary32 add. __fmul_rn and
// __fadd_rn are never contracted into an FMA, and this file is also compiled
// with -fmad=false and without flush-to-zero, so subnormals survive exactly
// as on the CPU. For the fused pair the intermediate C is rounded to binary32
// (it lives in shared memory or in a scratch panel) before the second GEMM.
//
// Work decomposition (B200: 148 SMs): one CTA owns a panel of R rows; its
// threads stride over output columns so global loads of B/D are coalesced
// and every thread carries R independent reduction chains to hide the
// dependent-add latency.
#include <cstdlib>

#include "common.cuh"
#include "internal.h"

namespace mcb {
namespace {

// acc[r] += sum_h A[r, h] * B[h] for h in [0, k), in increasing h, each step
// one binary32 multiply then one binary32 add (never fused). A row r starts at
// a + r * lda (contiguous in h); B steps by ldb. Operands are loaded kU steps
// ahead of the dependent add chain so the loads overlap instead of each one
// paying a full memory round trip; the reduction order is unchanged.
// kLdgA selects the read-only cache for A (inputs); data written earlier in
// the same kernel (the panel) must use plain loads.
template <int R, bool kLdgA>
__device__ __forceinline__ void strict_rows(const float *__restrict__ a, int64_t lda,
                                            const float *__restrict__ b, int64_t ldb, int64_t k,
                                            int rows, float (&acc)[R]) {
  constexpr int kU = 16;
  int64_t h0 = 0;
  for (; h0 + kU <= k; h0 += kU) {
    float bv[kU], av[R][kU];
#pragma unroll
    for (int u = 0; u < kU; ++u) bv[u] = __ldg(b + (h0 + u) * ldb);
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int u = 0; u < kU; ++u)
        av[r][u] = r < rows ? (kLdgA ? __ldg(a + r * lda + h0 + u) : a[r * lda + h0 + u]) : 0.0f;
#pragma unroll
    for (int u = 0; u < kU; ++u)
#pragma unroll
      for (int r = 0; r < R; ++r) acc[r] = __fadd_rn(acc[r], __fmul_rn(av[r][u], bv[u]));
  }
  for (; h0 < k; ++h0) {
    const float bv = __ldg(b + h0 * ldb);
#pragma unroll
    for (int r = 0; r < R; ++r)
      if (r < rows)
        acc[r] = __fadd_rn(acc[r], __fmul_rn(kLdgA ? __ldg(a + r * lda + h0) : a[r * lda + h0], bv));
  }
}

// One CTA per panel of R rows. Phase 1 writes the panel C[R, N] (binary32) to
// `panel` (shared memory when it fits, else this CTA's slice of a global
// scratch buffer); phase 2 reduces it against D.
template <int R, bool kSmemPanel>
__global__ void __launch_bounds__(256) strict_pair_kernel(
    const float *__restrict__ a, const float *__restrict__ b, const float *__restrict__ d,
    float *__restrict__ e, float *__restrict__ scratch, int64_t m, int64_t k, int64_t n,
    int64_t p, int64_t lda, int64_t ldb, int64_t ldd, int64_t lde) {
  extern __shared__ float smem_panel[];
  const int64_t r0 = static_cast<int64_t>(blockIdx.x) * R;
  if (r0 >= m) return;
  const int rows = static_cast<int>(m - r0 < R ? m - r0 : R);
  float *panel = kSmemPanel ? smem_panel : scratch + static_cast<int64_t>(blockIdx.x) * R * n;

  // Phase 1: C[r, j] = sum_h A[r0+r, h] * B[h, j]
  for (int64_t j = threadIdx.x; j < n; j += blockDim.x) {
    float acc[R];
#pragma unroll
    for (int r = 0; r < R; ++r) acc[r] = 0.0f;
    strict_rows<R, true>(a + r0 * lda, lda, b + j, ldb, k, rows, acc);
#pragma unroll
    for (int r = 0; r < R; ++r)
      if (r < rows) panel[r * n + j] = acc[r];
  }
  __syncthreads();
  // Phase 2: E[r0+r, q] = sum_j C[r, j] * D[j, q]
  for (int64_t q = threadIdx.x; q < p; q += blockDim.x) {
    float acc[R];
#pragma unroll
    for (int r = 0; r < R; ++r) acc[r] = 0.0f;
    strict_rows<R, false>(panel, n, d + q, ldd, n, rows, acc);
#pragma unroll
    for (int r = 0; r < R; ++r)
      if (r < rows) e[(r0 + r) * lde + q] = acc[r];
  }
}

// ---- staged fused pair (operands through shared memory) -------------------------
// Same arithmetic as strict_pair_kernel (one thread per output column, R
// independent row chains, increasing k, separate multiply and add, C rounded
// to binary32 in shared memory), but B, the A rows and then D are streamed
// through a double-buffered shared-memory ring of KC-row chunks with 16-byte
// cp.async copies: the whole CTA issues the copies of chunk c+1 before it
// reduces chunk c, so a global round trip is paid once per chunk instead of
// once per 16 reduction steps per thread. Used when every row is 16-byte
// aligned and N, P <= 1024 (one column per thread).
__device__ __forceinline__ void cp_async16(void *smem_dst, const void *gsrc) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem_dst)), "l"(gsrc)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Bulk prefetch of [ptr, ptr + bytes) into L2 (16-byte granules, whole
// granules only: the range is shrunk to 16-byte boundaries).
__device__ __forceinline__ void prefetch_l2_range(const void *ptr, int64_t bytes) {
  uintptr_t lo = (reinterpret_cast<uintptr_t>(ptr) + 15) & ~static_cast<uintptr_t>(15);
  const uintptr_t hi = (reinterpret_cast<uintptr_t>(ptr) + bytes) & ~static_cast<uintptr_t>(15);
  while (lo < hi) {
    const uint32_t chunk = static_cast<uint32_t>(hi - lo > (1u << 20) ? (1u << 20) : hi - lo);
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(lo), "r"(chunk) : "memory");
    lo += chunk;
  }
}
// This CTA's 1/gridDim.x share of [ptr, ptr + bytes).
__device__ __forceinline__ void prefetch_l2_share(const void *ptr, int64_t bytes) {
  const int64_t share = ((bytes + gridDim.x - 1) / gridDim.x + 15) & ~static_cast<int64_t>(15);
  const int64_t off = share * blockIdx.x;
  if (off < bytes)
    prefetch_l2_range(static_cast<const char *>(ptr) + off, bytes - off < share ? bytes - off : share);
}

struct StagedShape {
  int kc;           // rows per chunk
  int wmax;         // max(n, p) rounded up to 4: row pitch of a chunk in floats
};

template <int R>
__global__ void __launch_bounds__(1024) strict_pair_staged_kernel(
    const float *__restrict__ a, const float *__restrict__ b, const float *__restrict__ d,
    float *__restrict__ e, int64_t m, int64_t k, int64_t n, int64_t p, int64_t lda,
    int64_t ldb, int64_t ldd, int64_t lde, StagedShape sh) {
  extern __shared__ __align__(16) float smem_f[];
  const int kc = sh.kc, pitch = sh.wmax;
  float *ring = smem_f;                              // [2][kc][pitch]
  float *a_s = ring + 2 * kc * pitch;                // [2][R][kc]
  float *panel = a_s + 2 * R * kc;                   // [R][n]
  const int64_t r0 = static_cast<int64_t>(blockIdx.x) * R;
  if (r0 >= m) return;
  const int rows = static_cast<int>(m - r0 < R ? m - r0 : R);
  const int tid = threadIdx.x, nthr = blockDim.x;
  if (tid == 0) {
    // Every CTA streams all of B and D: pull this CTA's share of both spans
    // (and its own A rows) into L2 up front, so the chunk copies below hit L2
    // instead of paying a DRAM round trip each.
    prefetch_l2_share(b, ((k - 1) * ldb + n) * 4);
    prefetch_l2_share(d, ((n - 1) * ldd + p) * 4);
    prefetch_l2_range(a + r0 * lda, ((rows - 1) * lda + k) * 4);
  }

  // Copies chunk c of a [K x W] row-major operand (rows of W floats at stride
  // ld) into ring buffer `buf`, plus (phase 1) the matching A columns.
  auto stage = [&](const float *src, int64_t ld, int64_t w, int64_t ktot, int64_t c, int buf,
                   bool with_a) {
    const int64_t h0 = c * kc;
    const int nr = static_cast<int>(ktot - h0 < kc ? ktot - h0 : kc);
    const int v4 = static_cast<int>(w >> 2);
    float *dst = ring + buf * kc * pitch;
    for (int i = tid; i < nr * v4; i += nthr) {
      const int rr = i / v4, cc = (i - rr * v4) * 4;
      cp_async16(dst + rr * pitch + cc, src + (h0 + rr) * ld + cc);
    }
    if (with_a) {
      const int av4 = nr >> 2;
      float *ad = a_s + buf * R * kc;
      for (int i = tid; i < rows * av4; i += nthr) {
        const int rr = i / av4, cc = (i - rr * av4) * 4;
        cp_async16(ad + rr * kc + cc, a + (r0 + rr) * lda + h0 + cc);
      }
    }
    cp_async_commit();
  };

  // Phase 1: C[r, j] = sum_h A[r0+r, h] * B[h, j]
  {
    float acc[R];
#pragma unroll
    for (int r = 0; r < R; ++r) acc[r] = 0.0f;
    const int64_t nch = (k + kc - 1) / kc;
    if (nch > 0) stage(b, ldb, n, k, 0, 0, true);
    for (int64_t c = 0; c < nch; ++c) {
      const int buf = static_cast<int>(c & 1);
      if (c + 1 < nch) {
        stage(b, ldb, n, k, c + 1, buf ^ 1, true);
        cp_async_wait<1>();
      } else {
        cp_async_wait<0>();
      }
      __syncthreads();
      const int nr = static_cast<int>(k - c * kc < kc ? k - c * kc : kc);
      if (tid < n) {
        const float *bs = ring + buf * kc * pitch + tid;
        const float *as = a_s + buf * R * kc;
        for (int h = 0; h < nr; ++h) {
          const float bv = bs[h * pitch];
#pragma unroll
          for (int r = 0; r < R; ++r) acc[r] = __fadd_rn(acc[r], __fmul_rn(as[r * kc + h], bv));
        }
      }
      __syncthreads();  // buffer `buf` is refilled by the next iteration's copies
    }
    if (tid < n) {
#pragma unroll
      for (int r = 0; r < R; ++r) panel[r * n + tid] = acc[r];
    }
    __syncthreads();
  }
  // Phase 2: E[r0+r, q] = sum_j C[r, j] * D[j, q]
  {
    float acc[R];
#pragma unroll
    for (int r = 0; r < R; ++r) acc[r] = 0.0f;
    const int64_t nch = (n + kc - 1) / kc;
    stage(d, ldd, p, n, 0, 0, false);
    for (int64_t c = 0; c < nch; ++c) {
      const int buf = static_cast<int>(c & 1);
      if (c + 1 < nch) {
        stage(d, ldd, p, n, c + 1, buf ^ 1, false);
        cp_async_wait<1>();
      } else {
        cp_async_wait<0>();
      }
      __syncthreads();
      const int nr = static_cast<int>(n - c * kc < kc ? n - c * kc : kc);
      if (tid < p) {
        const float *ds = ring + buf * kc * pitch + tid;
        const float *cs = panel + c * kc;
        for (int h = 0; h < nr; ++h) {
          const float dv = ds[h * pitch];
#pragma unroll
          for (int r = 0; r < R; ++r) acc[r] = __fadd_rn(acc[r], __fmul_rn(cs[r * n + h], dv));
        }
      }
      __syncthreads();
    }
    if (tid < p) {
#pragma unroll
      for (int r = 0; r < R; ++r)
        if (r < rows) e[(r0 + r) * lde + tid] = acc[r];
    }
  }
}

// ---- tiled strict GEMM ------------------------------------------------------------
// C[M,N] = A[M,K] B[K,N] with each output a strict chain (increasing k, +0
// seed, separate binary32 multiply and add). A CTA computes a (TY*MR) x
// (TX*NR) tile; each thread an MR x NR block of chains, so one pair of shared
// memory reads feeds MR*NR multiply-adds. KC-deep slices of the A and B tiles
// go through a 3-stage shared-memory ring with cp.async (16-byte copies when
// every row is 16-byte aligned, 4-byte copies otherwise); two slices are in
// flight while one is reduced. Out-of-range rows and columns are never
// copied and their chains are never stored.
constexpr int TKC = 32;       // k-slice depth
constexpr int TAP = TKC + 4;  // padded A-tile row pitch (floats)
constexpr int TST = 3;        // ring stages

__device__ __forceinline__ void cp_async4(void *smem_dst, const void *gsrc) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(smem_dst)), "l"(gsrc)
               : "memory");
}

template <int MR, int NR, int TX, int TY, bool kVec>
__global__ void __launch_bounds__(TX *TY) strict_tiled_kernel(
    const float *__restrict__ a, const float *__restrict__ b, float *__restrict__ c, int64_t m,
    int64_t k, int64_t n, int64_t lda, int64_t ldb, int64_t ldc) {
  constexpr int TM = TY * MR, TN = TX * NR, NT = TX * TY;
  __shared__ __align__(16) float as[TST][TM][TAP];
  __shared__ __align__(16) float bs[TST][TKC][TN];
  const int tid = threadIdx.x, tx = tid % TX, ty = tid / TX;
  const int64_t row0 = static_cast<int64_t>(blockIdx.y) * TM;
  const int64_t col0 = static_cast<int64_t>(blockIdx.x) * TN;
  const int mrows = static_cast<int>(m - row0 < TM ? m - row0 : TM);
  const int ncols = static_cast<int>(n - col0 < TN ? n - col0 : TN);

  auto stage = [&](int64_t cidx, int buf) {
    const int64_t h0 = cidx * TKC;
    const int nr = static_cast<int>(k - h0 < TKC ? k - h0 : TKC);
    if (kVec && nr == TKC && mrows == TM && ncols == TN) {  // full tile: constant divisors
#pragma unroll
      for (int i = tid; i < TM * (TKC / 4); i += NT) {
        const int r = i / (TKC / 4), q = (i % (TKC / 4)) * 4;
        cp_async16(&as[buf][r][q], a + (row0 + r) * lda + h0 + q);
      }
#pragma unroll
      for (int i = tid; i < TKC * (TN / 4); i += NT) {
        const int r = i / (TN / 4), q = (i % (TN / 4)) * 4;
        cp_async16(&bs[buf][r][q], b + (h0 + r) * ldb + col0 + q);
      }
    } else if (kVec) {  // nr, ncols and every row start are multiples of 4 floats
      const int av = nr >> 2, bv = ncols >> 2;
      for (int i = tid; i < mrows * av; i += NT) {
        const int r = i / av, q = (i - r * av) * 4;
        cp_async16(&as[buf][r][q], a + (row0 + r) * lda + h0 + q);
      }
      for (int i = tid; i < nr * bv; i += NT) {
        const int r = i / bv, q = (i - r * bv) * 4;
        cp_async16(&bs[buf][r][q], b + (h0 + r) * ldb + col0 + q);
      }
    } else {
      for (int i = tid; i < mrows * nr; i += NT) {
        const int r = i / nr, q = i - r * nr;
        cp_async4(&as[buf][r][q], a + (row0 + r) * lda + h0 + q);
      }
      for (int i = tid; i < nr * ncols; i += NT) {
        const int r = i / ncols, q = i - r * ncols;
        cp_async4(&bs[buf][r][q], b + (h0 + r) * ldb + col0 + q);
      }
    }
    cp_async_commit();
  };

  // When launched programmatically (the second GEMM of a two-pass pair):
  // wait for the previous grid, whose output this one reads, and let the
  // next launch start its own set-up. No-ops otherwise.
  grid_dependency_wait();
  grid_launch_dependents();
  float acc[MR][NR];
#pragma unroll
  for (int r = 0; r < MR; ++r)
#pragma unroll
    for (int j = 0; j < NR; ++j) acc[r][j] = 0.0f;
  const int64_t nch = (k + TKC - 1) / TKC;
#pragma unroll
  for (int st = 0; st < TST - 1; ++st) {
    if (st < nch)
      stage(st, st);
    else
      cp_async_commit();  // empty group keeps the per-iteration accounting uniform
  }
  for (int64_t ci = 0; ci < nch; ++ci) {
    const int buf = static_cast<int>(ci % TST);
    cp_async_wait<TST - 2>();  // slice ci has landed
    __syncthreads();           // ... for every thread, and slice ci-1 is no longer read
    if (ci + TST - 1 < nch)
      stage(ci + TST - 1, static_cast<int>((ci + TST - 1) % TST));
    else
      cp_async_commit();
    const int nr = static_cast<int>(k - ci * TKC < TKC ? k - ci * TKC : TKC);
    int h = 0;
    for (; h + 4 <= nr; h += 4) {
      float a4[MR][4];
#pragma unroll
      for (int r = 0; r < MR; ++r) {
        const float4 v = *reinterpret_cast<const float4 *>(&as[buf][ty * MR + r][h]);
        a4[r][0] = v.x;
        a4[r][1] = v.y;
        a4[r][2] = v.z;
        a4[r][3] = v.w;
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        float bv[NR];
        if (NR == 4) {
          const float4 v = *reinterpret_cast<const float4 *>(&bs[buf][h + u][tx * NR]);
          bv[0] = v.x;
          bv[1 % NR] = v.y;
          bv[2 % NR] = v.z;
          bv[3 % NR] = v.w;
        } else {
          const float2 v = *reinterpret_cast<const float2 *>(&bs[buf][h + u][tx * NR]);
          bv[0] = v.x;
          bv[1 % NR] = v.y;
        }
#pragma unroll
        for (int r = 0; r < MR; ++r)
#pragma unroll
          for (int j = 0; j < NR; ++j) acc[r][j] = __fadd_rn(acc[r][j], __fmul_rn(a4[r][u], bv[j]));
      }
    }
    for (; h < nr; ++h) {
#pragma unroll
      for (int r = 0; r < MR; ++r) {
        const float av = as[buf][ty * MR + r][h];
#pragma unroll
        for (int j = 0; j < NR; ++j)
          acc[r][j] = __fadd_rn(acc[r][j], __fmul_rn(av, bs[buf][h][tx * NR + j]));
      }
    }
  }
  cp_async_wait<0>();
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

__global__ void fill_zero_kernel(float *__restrict__ y, int64_t rows, int64_t cols, int64_t ld) {
  const int64_t total = rows * cols;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    y[(i / cols) * ld + (i % cols)] = 0.0f;
}

// Rows per CTA: the largest R in {4, 2, 1} that still gives at least two CTAs
// per SM, so small problems are spread over the whole GPU.
int pick_rows(int64_t m, int sms) {
  if ((m + 3) / 4 >= 2 * sms) return 4;
  if ((m + 1) / 2 >= 2 * sms) return 2;
  if ((m + 3) / 4 >= sms) return 4;
  return (m + 1) / 2 >= sms ? 2 : 1;
}

// Large strict GEMM: 256 threads own a 128x128 tile of C, each thread 8x8
// chains (rows 4ty.. and 64+4ty.., columns 4tx.. and 64+4tx..). Every chain
// is the strict one: starting from +0, c = __fadd_rn(c, __fmul_rn(a, b)) for
// k = 0, 1, 2, ... in order, so the result is bit-identical to the CPU leaf
// however the tile is laid out. 16-deep k-slices of A (stored transposed,
// [k][row]) and B ([k][col]) are double-buffered in shared memory, the next
// slice fetched into registers (16-byte loads) while the current one is
// consumed; a partial last slice runs only its real depth.
constexpr int SBM = 128, SBN = 128, SBK = 16, SBPAD = 4;

__global__ void __launch_bounds__(256, 2) strict_big_kernel(
    const float *__restrict__ a, const float *__restrict__ b, float *__restrict__ c, int64_t m,
    int64_t k, int64_t n, int64_t lda, int64_t ldb, int64_t ldc) {
  __shared__ __align__(16) float as[2][SBK][SBM + SBPAD];
  __shared__ __align__(16) float bs[2][SBK][SBN + SBPAD];
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const int64_t row0 = static_cast<int64_t>(blockIdx.y) * SBM;
  const int64_t col0 = static_cast<int64_t>(blockIdx.x) * SBN;
  const int ar = tid & 127, aq = (tid >> 7) * 4;
  const int bk = tid >> 5, bc = (tid & 31) * 4;
  float4 ra[2], rb[2];
  auto fetch = [&](int64_t sl) {
    const int64_t h0 = sl * SBK;
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int64_t gr = row0 + ar, gk = h0 + aq + i * 8;
      ra[i] = (gr < m && gk < k) ? *reinterpret_cast<const float4 *>(a + gr * lda + gk)
                                 : make_float4(0.f, 0.f, 0.f, 0.f);
      const int64_t kb = h0 + bk + i * 8, gc = col0 + bc;
      rb[i] = (kb < k && gc < n) ? *reinterpret_cast<const float4 *>(b + kb * ldb + gc)
                                 : make_float4(0.f, 0.f, 0.f, 0.f);
    }
  };
  auto stage = [&](int buf) {
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int kq = aq + i * 8;
      as[buf][kq][ar] = ra[i].x;
      as[buf][kq + 1][ar] = ra[i].y;
      as[buf][kq + 2][ar] = ra[i].z;
      as[buf][kq + 3][ar] = ra[i].w;
      *reinterpret_cast<float4 *>(&bs[buf][bk + i * 8][bc]) = rb[i];
    }
  };
  float acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.0f;
  const int64_t nslices = (k + SBK - 1) / SBK;
  if (nslices > 0) {
    fetch(0);
    stage(0);
  }
  __syncthreads();
  for (int64_t sl = 0; sl < nslices; ++sl) {
    const int buf = static_cast<int>(sl & 1);
    if (sl + 1 < nslices) fetch(sl + 1);
    const int depth = static_cast<int>(k - sl * SBK < SBK ? k - sl * SBK : SBK);
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
        for (int j = 0; j < 8; ++j) acc[i][j] = __fadd_rn(acc[i][j], __fmul_rn(av[i], bv[j]));
    };
    if (depth == SBK) {
#pragma unroll
      for (int kk = 0; kk < SBK; ++kk) step(kk);
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

// One tiled strict GEMM launch: 16 x 64 tiles (16 x 32 when N is small),
// 16-byte copies when every row allows them.
template <int MR, int NR>
cudaError_t launch_tiled_variant(const float *a, const float *b, float *c, int64_t m, int64_t k,
                                 int64_t n, int64_t lda, int64_t ldb, int64_t ldc, bool vec,
                                 bool pdl, cudaStream_t stream, LaunchInfo *info) {
  constexpr int TX = 16, TY = 8, TM = TY * MR, TN = TX * NR;
  const int64_t gy = (m + TM - 1) / TM, gx = (n + TN - 1) / TN;
  if (gy > 65535 || gx > 0x7fffffff) return cudaErrorInvalidConfiguration;
  const dim3 grid(static_cast<unsigned>(gx), static_cast<unsigned>(gy));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(TX * TY, 1, 1);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e =
      vec ? cudaLaunchKernelEx(&cfg, strict_tiled_kernel<MR, NR, TX, TY, true>, a, b, c, m, k, n,
                               lda, ldb, ldc)
          : cudaLaunchKernelEx(&cfg, strict_tiled_kernel<MR, NR, TX, TY, false>, a, b, c, m, k, n,
                               lda, ldb, ldc);
  if (e != cudaSuccess) return e;
  if (info) {
    info->launches += 1;
    info->tile_m = TM;
    info->tile_n = TN;
    info->tile_k = TKC;
    info->ctas += static_cast<int>(grid.x * grid.y);
  }
  return cudaGetLastError();
}

// One tiled strict GEMM launch. The per-thread block shrinks (8 -> 4 -> 2
// chains) with the problem: 2x4 while a launch still has about four warps per
// SM sub-partition (2368 on 148 SMs), 2x2 down to one warp per sub-partition
// (fewer instructions per multiply-add outweigh the thinner latency hiding:
// config 1's C = A*B runs 14% faster than with 1x2), else 1x2; 16-byte copies
// when every row allows them.
cudaError_t launch_tiled(const float *a, const float *b, float *c, int64_t m, int64_t k, int64_t n,
                         int64_t lda, int64_t ldb, int64_t ldc, int sms, cudaStream_t stream,
                         LaunchInfo *info, bool pdl = false) {
  const auto al16 = [](const void *ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; };
  const bool vec = k % 4 == 0 && n % 4 == 0 && lda % 4 == 0 && ldb % 4 == 0 &&
                   (k == 0 || (al16(a) && al16(b)));
  const int64_t warp_slots = static_cast<int64_t>(sms) * 4 * 32;  // one warp per sub-partition
  const int64_t outputs = m * n;
  // At least one 128x128 tile per SM: 8x8 chains per thread.
  const int64_t big_rows = (m + SBM - 1) / SBM, big_cols = (n + SBN - 1) / SBN;
  if (vec && big_rows * big_cols >= sms && big_rows <= 65535) {
    strict_big_kernel<<<dim3(static_cast<unsigned>(big_cols), static_cast<unsigned>(big_rows)), 256,
                        0, stream>>>(a, b, c, m, k, n, lda, ldb, ldc);
    if (info) {
      info->launches += 1;
      info->tile_m = SBM;
      info->tile_n = SBN;
      info->tile_k = SBK;
      info->ctas += static_cast<int>(big_rows * big_cols);
    }
    return cudaGetLastError();
  }
  if (outputs / 8 >= 4 * warp_slots && n >= 64)
    return launch_tiled_variant<2, 4>(a, b, c, m, k, n, lda, ldb, ldc, vec, pdl, stream, info);
  if (outputs / 4 >= warp_slots && n >= 32)
    return launch_tiled_variant<2, 2>(a, b, c, m, k, n, lda, ldb, ldc, vec, pdl, stream, info);
  return launch_tiled_variant<1, 2>(a, b, c, m, k, n, lda, ldb, ldc, vec, pdl, stream, info);
}

}  // namespace

cudaError_t launch_strict_gemm(const float *a, const float *b, float *c, int64_t m, int64_t k,
                               int64_t n, int64_t lda, int64_t ldb, int64_t ldc, int sms,
                               cudaStream_t stream, LaunchInfo *info) {
  if (m == 0 || n == 0) return cudaSuccess;
  if (info) {
    info->launches = 0;
    info->ctas = 0;
  }
  const cudaError_t err = launch_tiled(a, b, c, m, k, n, lda, ldb, ldc, sms, stream, info);
  if (info) info->set_route("strict_f32_simt_gemm_tiled");
  return err;
}

cudaError_t launch_strict_pair_two_pass(const float *a, const float *b, const float *d, float *e,
                                        float *c_buf, int64_t m, int64_t k, int64_t n, int64_t p,
                                        int64_t lda, int64_t ldb, int64_t ldd, int64_t lde,
                                        int sms, cudaStream_t stream, LaunchInfo *info) {
  if (info) {
    info->launches = 0;
    info->ctas = 0;
  }
  if (m == 0 || p == 0) return cudaSuccess;
  // The second GEMM is launched programmatically: its CTAs are scheduled as
  // the first one's finish and wait in-kernel for the whole first grid
  // (MCB_STRICT_PDL=0 turns this off, for measurement).
  static const bool pdl = [] {
    const char *v = getenv("MCB_STRICT_PDL");
    return !(v && v[0] == '0');
  }();
  cudaError_t err = launch_tiled(a, b, c_buf, m, k, n, lda, ldb, n, sms, stream, info);
  if (err == cudaSuccess)
    err = launch_tiled(c_buf, d, e, m, n, p, n, ldd, lde, sms, stream, info, pdl);
  if (info) info->set_route("strict_f32_simt_pair_two_pass");
  return err;
}

int64_t strict_pair_scratch_floats(int64_t m, int64_t n, int sms, int smem_limit_bytes) {
  const int R = pick_rows(m, sms);
  if (static_cast<int64_t>(R) * n * 4 <= smem_limit_bytes) return 0;
  return ((m + R - 1) / R) * R * n;
}

cudaError_t launch_strict_pair(const float *a, const float *b, const float *d, float *e,
                               float *scratch, int64_t m, int64_t k, int64_t n, int64_t p,
                               int64_t lda, int64_t ldb, int64_t ldd, int64_t lde, int sms,
                               int smem_limit_bytes, cudaStream_t stream, LaunchInfo *info) {
  if (m == 0 || p == 0) return cudaSuccess;
  if (info) info->launches = 0;
  if (n == 0) {  // empty consumer reduction: E = +0
    fill_zero_kernel<<<sms, 256, 0, stream>>>(e, m, p, lde);
    if (info) {
      info->launches = 1;
      info->set_route("strict_f32_zero_reduction");
    }
    return cudaGetLastError();
  }
  const int R = pick_rows(m, sms);
  // Staged kernel: 16-byte aligned rows, one column per thread.
  const auto al16 = [](const void *ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; };
  if (k > 0 && n <= 1024 && p <= 1024 && n % 4 == 0 && p % 4 == 0 && k % 4 == 0 &&
      lda % 4 == 0 && ldb % 4 == 0 && ldd % 4 == 0 && al16(a) && al16(b) && al16(d)) {
    StagedShape sh;
    sh.wmax = static_cast<int>(n > p ? n : p);
    const int64_t fixed = static_cast<int64_t>(R) * n * 4;
    // Largest chunk (32 or 16 rows) whose two buffers fit; two CTAs per SM
    // when the whole footprint stays under ~110 KB.
    sh.kc = 32;
    auto bytes = [&](int kc) { return (2LL * kc * sh.wmax + 2LL * R * kc) * 4 + fixed; };
    if (bytes(32) > 110 * 1024) sh.kc = 16;
    const int64_t smem = bytes(sh.kc);
    if (smem <= smem_limit_bytes) {
      const int threads = static_cast<int>(((sh.wmax + 31) / 32) * 32);
      const int64_t ctas = (m + R - 1) / R;
      if (ctas > 0x7fffffff) return cudaErrorInvalidConfiguration;
      cudaError_t err = cudaSuccess;
      switch (R) {
        case 4:
          err = cudaFuncSetAttribute(strict_pair_staged_kernel<4>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
          if (err == cudaSuccess)
            strict_pair_staged_kernel<4><<<(unsigned)ctas, threads, smem, stream>>>(
                a, b, d, e, m, k, n, p, lda, ldb, ldd, lde, sh);
          break;
        case 2:
          err = cudaFuncSetAttribute(strict_pair_staged_kernel<2>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
          if (err == cudaSuccess)
            strict_pair_staged_kernel<2><<<(unsigned)ctas, threads, smem, stream>>>(
                a, b, d, e, m, k, n, p, lda, ldb, ldd, lde, sh);
          break;
        default:
          err = cudaFuncSetAttribute(strict_pair_staged_kernel<1>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
          if (err == cudaSuccess)
            strict_pair_staged_kernel<1><<<(unsigned)ctas, threads, smem, stream>>>(
                a, b, d, e, m, k, n, p, lda, ldb, ldd, lde, sh);
          break;
      }
      if (err != cudaSuccess) return err;
      if (info) {
        info->launches = 1;
        info->tile_m = R;
        info->tile_n = threads;
        info->tile_k = sh.kc;
        info->ctas = static_cast<int>(ctas);
        info->set_route("strict_f32_simt_pair_staged");
      }
      return cudaGetLastError();
    }
  }
  const int64_t panel_bytes = static_cast<int64_t>(R) * n * 4;
  const bool in_smem = panel_bytes <= smem_limit_bytes;
  if (!in_smem && scratch == nullptr) return cudaErrorInvalidValue;
  const int64_t ctas = (m + R - 1) / R;
  if (ctas > 0x7fffffff) return cudaErrorInvalidConfiguration;
  const int threads = (n >= 256 || p >= 256) ? 256 : 128;
  const size_t smem = in_smem ? static_cast<size_t>(panel_bytes) : 0;
#define MCB_PAIR_CASE(RR)                                                                    \
  case RR:                                                                                   \
    if (in_smem) {                                                                           \
      if (smem > 48 * 1024)                                                                  \
        cudaFuncSetAttribute(strict_pair_kernel<RR, true>,                                   \
                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);        \
      strict_pair_kernel<RR, true><<<(unsigned)ctas, threads, smem, stream>>>(              \
          a, b, d, e, scratch, m, k, n, p, lda, ldb, ldd, lde);                              \
    } else {                                                                                 \
      strict_pair_kernel<RR, false><<<(unsigned)ctas, threads, 0, stream>>>(                \
          a, b, d, e, scratch, m, k, n, p, lda, ldb, ldd, lde);                              \
    }                                                                                        \
    break;
  switch (R) {
    MCB_PAIR_CASE(4)
    MCB_PAIR_CASE(2)
    default:
      MCB_PAIR_CASE(1)
  }
#undef MCB_PAIR_CASE
  if (info) {
    info->launches = 1;
    info->tile_m = R;
    info->tile_n = threads;
    info->ctas = static_cast<int>(ctas);
    info->set_route(in_smem ? "strict_f32_simt_pair_smem_panel"
                            : "strict_f32_simt_pair_scratch_panel");
  }
  return cudaGetLastError();
}

// The fused pair with the intermediate panel always in a caller-supplied
// fixed-size scratch array of `scratch_floats` floats. Rows are processed in
// as many back-to-back launches (same stream) as the array needs, so only one
// panel of R x N floats has to fit. Returns cudaErrorInvalidValue when even a
// single-row panel (N floats) does not fit.
cudaError_t launch_strict_pair_fixed_scratch(const float *a, const float *b, const float *d,
                                             float *e, float *scratch, int64_t scratch_floats,
                                             int64_t m, int64_t k, int64_t n, int64_t p,
                                             int64_t lda, int64_t ldb, int64_t ldd, int64_t lde,
                                             int sms, cudaStream_t stream, LaunchInfo *info,
                                             bool *panel_too_large) {
  if (info) info->launches = 0;
  *panel_too_large = false;
  if (m == 0 || p == 0) return cudaSuccess;
  if (n == 0) {  // empty consumer reduction: E = +0, no panel
    fill_zero_kernel<<<sms, 256, 0, stream>>>(e, m, p, lde);
    if (info) {
      info->launches = 1;
      info->set_route("strict_f32_zero_reduction");
    }
    return cudaGetLastError();
  }
  int R = pick_rows(m, sms);
  while (R > 1 && static_cast<int64_t>(R) * n > scratch_floats) R /= 2;
  if (static_cast<int64_t>(R) * n > scratch_floats) {
    *panel_too_large = true;  // nothing launched
    return cudaErrorInvalidValue;
  }
  const int64_t rows_per_launch = (scratch_floats / (static_cast<int64_t>(R) * n)) * R;
  const int threads = (n >= 256 || p >= 256) ? 256 : 128;
  int launches = 0;
  for (int64_t r0 = 0; r0 < m; r0 += rows_per_launch) {
    const int64_t mc = m - r0 < rows_per_launch ? m - r0 : rows_per_launch;
    const int64_t ctas = (mc + R - 1) / R;
    if (ctas > 0x7fffffff) return cudaErrorInvalidConfiguration;
    const float *ac = k ? a + r0 * lda : a;
    float *ec = e + r0 * lde;
    switch (R) {
      case 4:
        strict_pair_kernel<4, false><<<(unsigned)ctas, threads, 0, stream>>>(
            ac, b, d, ec, scratch, mc, k, n, p, lda, ldb, ldd, lde);
        break;
      case 2:
        strict_pair_kernel<2, false><<<(unsigned)ctas, threads, 0, stream>>>(
            ac, b, d, ec, scratch, mc, k, n, p, lda, ldb, ldd, lde);
        break;
      default:
        strict_pair_kernel<1, false><<<(unsigned)ctas, threads, 0, stream>>>(
            ac, b, d, ec, scratch, mc, k, n, p, lda, ldb, ldd, lde);
        break;
    }
    ++launches;
    cudaError_t err = cudaGetLastError();
    if (err != cudaSuccess) return err;
  }
  if (info) {
    info->launches = launches;
    info->tile_m = R;
    info->tile_n = threads;
    info->ctas = static_cast<int>((rows_per_launch + R - 1) / R);
    info->set_route("strict_f32_simt_pair_fixed_scratch");
  }
  return cudaSuccess;
}

}  // namespace mcb

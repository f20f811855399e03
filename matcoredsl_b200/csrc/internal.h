// Internal launcher interface between the C-ABI layer (api.cpp) and the
// kernel translation units. Nothing here is exported from libmcb.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include "mcb.h"

// This GPU's side of a head-sharded pair's exchange (peer.cu): one device
// allocation of a header (two step counters: "data" at byte 0, raised by the
// peer once its share of this GPU's rows is in the receive buffer;
// "consumed" at byte 128, raised by the peer once it has read the data this
// GPU wrote into its buffer) and the receive buffer at kHeaderBytes; `remote`
// is the peer's allocation opened through its IPC handle.
struct mcb_peer_exchange {
  static constexpr uint64_t kHeaderBytes = 256;
  int32_t device = -1;
  uint64_t recv_bytes = 0;
  void *local = nullptr;
  void *remote = nullptr;
  uint32_t step = 0;  // calls made so far (both GPUs of the pair call in lockstep)
};

namespace mcb {

struct LaunchInfo {
  int launches = 0;
  int tile_m = 0, tile_n = 0, tile_k = 0, stages = 0, ctas = 0;
  bool stream_k = false;  // the GEMM split K-block ranges of tiles over clusters
  char route[48] = {0};
  void set_route(const char *r) {
    strncpy(route, r, sizeof(route) - 1);
    route[sizeof(route) - 1] = 0;
  }
};

// ---- strict.cu ----------------------------------------------------------------
cudaError_t launch_strict_gemm(const float *a, const float *b, float *c, int64_t m, int64_t k,
                               int64_t n, int64_t lda, int64_t ldb, int64_t ldc, int sms,
                               cudaStream_t stream, LaunchInfo *info);
// Fused pair as two tiled strict GEMMs through a binary32 intermediate
// C_buf [M,N] (row stride N, 16-byte aligned): C = A B, then E = C D.
cudaError_t launch_strict_pair_two_pass(const float *a, const float *b, const float *d, float *e,
                                        float *c_buf, int64_t m, int64_t k, int64_t n, int64_t p,
                                        int64_t lda, int64_t ldb, int64_t ldd, int64_t lde,
                                        int sms, cudaStream_t stream, LaunchInfo *info);
// Floats of global scratch the fused pair needs (0 when the panel fits in
// shared memory).
int64_t strict_pair_scratch_floats(int64_t m, int64_t n, int sms, int smem_limit_bytes);
cudaError_t launch_strict_pair(const float *a, const float *b, const float *d, float *e,
                               float *scratch, int64_t m, int64_t k, int64_t n, int64_t p,
                               int64_t lda, int64_t ldb, int64_t ldd, int64_t lde, int sms,
                               int smem_limit_bytes, cudaStream_t stream, LaunchInfo *info);

// The fused pair with its intermediate panel in a fixed scratch array of
// `scratch_floats` floats (used by the allocation-free entry point).
// *panel_too_large is set (and nothing launched) when one panel row of N
// floats does not fit the array.
cudaError_t launch_strict_pair_fixed_scratch(const float *a, const float *b, const float *d,
                                             float *e, float *scratch, int64_t scratch_floats,
                                             int64_t m, int64_t k, int64_t n, int64_t p,
                                             int64_t lda, int64_t ldb, int64_t ldd, int64_t lde,
                                             int sms, cudaStream_t stream, LaunchInfo *info,
                                             bool *panel_too_large);

// Self-test of the bounded wait of a stream-K owner for another cluster's
// partial (mcb_device_peer_timeout_selftest_v1); see gemm_tc.cu.
cudaError_t launch_gemm_tc_peer_stall_selftest(const void *x, const void *w, void *y, float *part,
                                               int *flags, long long spin_limit, uint32_t *status,
                                               cudaStream_t stream);
// Self-test of the bounded pipeline waits (mcb_device_timeout_selftest_v1):
// one single-SM GEMM tile whose producer issues no loads.
cudaError_t launch_gemm_tc_stall_selftest(const void *x, const void *w, void *y,
                                          long long spin_limit, uint32_t *status,
                                          cudaStream_t stream);

// True while test runtime hooks (mcb_test_set_runtime_hooks_v1) are installed:
// entry points that launch kernels outside the hookable path refuse to run.
bool runtime_hooks_installed();

// ---- epilogue description shared by the GEMM kernels ----------------------------
constexpr int kMaxEpiOps = 8, kMaxEpiBoundaries = 4;
struct Epilogue {
  int bias_mode = 0;  // 0 none, 1 row-broadcast [N], 2 full [M,N]
  int bias_op = 0;    // 0 add, 1 reverse subtract
  int act = 0;        // 0 none, 1 relu, 2 gelu_tanh, 3 exp, 4 sigmoid, 5 tanh
  int bias_bf16 = 0;  // bias element type: bf16 (else f16 when bias_f16, else f32)
  int bias_f16 = 0;
  int bias_aligned16 = 0;  // bias base is 16-byte aligned (vector loads allowed)
  const void *bias = nullptr;
  int64_t ld_bias = 0;
  // General chain (mcb_gemm_epilogue_chain_v1): when n_ops > 0 the fields
  // above are unused and the ops apply in order to the f32 accumulator.
  // Kinds are the MCB_EW_* codes (unary < 32, binary >= 32); a binary op
  // combines the running value with boundary op_bnd[i] ([M,N], row stride
  // ld_bnd, dtype code bnd_dt: 1 f32, 3 bf16, 6 f16), the value on the left
  // when op_pos[i] == 0, on the right when 1.
  int n_ops = 0;
  uint8_t op_kind[kMaxEpiOps] = {};
  uint8_t op_pos[kMaxEpiOps] = {};
  uint8_t op_bnd[kMaxEpiOps] = {};
  uint8_t bnd_dt[kMaxEpiBoundaries] = {};
  const void *bnd[kMaxEpiBoundaries] = {};
  int64_t ld_bnd[kMaxEpiBoundaries] = {};
};

// ---- gemm_tc.cu: tcgen05 bf16 / f16 GEMM + epilogue ------------------------------
// X [M,K] (ld_x), W [K,N] (ld_w, w_transposed=0) or W^T [N,K] (w_transposed=1),
// both bf16 or both f16 (in_f16); Y [M,N] f32, bf16 or f16 (y_kind). Requires
// K, N, ld_x, ld_w multiples of 8 and 16-byte aligned bases (TMA); the caller
// checks.
enum : int { kOutF32 = 0, kOutBf16 = 1, kOutF16 = 2 };
// Device workspace of the stream-K route of the CTA-pair GEMM: arrival
// counters (2 per stream-K tile, zero between launches; every launch leaves
// them zero unless it aborted) and partial-accumulator slots (128x256 f32 per
// cluster, slot 0/1 and CTA rank). Launches that share one workspace must not
// overlap on the GPU.
struct GemmStreamK {
  int *flags = nullptr;  // ready flag per (split tile, CTA rank); 0 between launches
  float *part = nullptr; // tail partials: one 128x256 f32 slot per (cluster, CTA rank)
  int clusters = 0;      // clusters the slots cover
  int max_tiles = 0;     // split tiles the flags cover
};
constexpr int64_t kGemmStreamKSlotFloats = 128 * 256;
cudaError_t launch_gemm_tc_bf16(const void *x, const void *w, void *y, int64_t m, int64_t n,
                                int64_t k, int64_t ld_x, int64_t ld_w, int64_t ld_y,
                                int w_transposed, int y_kind, const Epilogue &epi,
                                uint32_t *status, int sms, cudaStream_t stream, LaunchInfo *info,
                                int in_f16 = 0, const GemmStreamK *sk = nullptr,
                                int no_tma_store = 0);

// Family B chain E = glue(A B) W fused on tcgen05 (chain_tc.cu): bf16 A [M,K],
// B [K,N1], W [N1,N2] (row-major, 16-byte aligned bases and row strides,
// K, N1, N2 multiples of 8), E f32 or bf16 (e_kind); `glue` is a bias +
// activation epilogue over the intermediate (no op chain). The intermediate
// stays in TMEM / shared memory. cudaErrorNotSupported: nothing launched.
cudaError_t launch_chain_tc_bf16(const void *a, const void *b, const void *w, void *e, int64_t m,
                                 int64_t k, int64_t n1, int64_t n2, int64_t lda, int64_t ldb,
                                 int64_t ldw, int64_t lde, int e_kind, const Epilogue &glue,
                                 uint32_t *status, int sms, cudaStream_t stream, LaunchInfo *info);

// Small Family B chains on CUDA cores in one launch, the intermediate in
// shared memory in f32 (16 rows per CTA, N1 <= 1536). dt: operand dtype (1 f32,
// 3 bf16); e_dt: output dtype. cudaErrorNotSupported: nothing launched.
cudaError_t launch_chain_simt_small(const void *a, const void *b, const void *w, void *e, int dt,
                                    int e_dt, int64_t m, int64_t k, int64_t n1, int64_t n2,
                                    int64_t lda, int64_t ldb, int64_t ldw, int64_t lde,
                                    const Epilogue &glue, cudaStream_t stream, LaunchInfo *info);

// ---- simt.cu: CUDA-core fallbacks for shapes/dtypes the tensor-core kernels do not take
// dtype codes: 1 f32, 3 bf16, 6 f16 (as in mcb.h)
cudaError_t launch_gemm_simt(const void *x, int x_dtype, const void *w, int w_dtype, void *y,
                             int y_dtype, int64_t m, int64_t n, int64_t k, int64_t ld_x,
                             int64_t ld_w, int64_t ld_y, int w_transposed, const Epilogue &epi,
                             cudaStream_t stream, LaunchInfo *info);

// Batched rank-2 MSM on CUDA cores (online softmax), any Dqk/Dv <= 256.
struct MsmShape {
  int64_t batch = 1, heads = 1, m = 0, n = 0, dqk = 0, dv = 0;
  // element strides: [batch, head, row] for each tensor (innermost is 1)
  int64_t q_s[3], k_s[3], v_s[3], o_s[3];
};
cudaError_t launch_msm_simt(const void *q, const void *k, const void *v, void *o, int dtype,
                            const MsmShape &s, float scale, cudaStream_t stream,
                            LaunchInfo *info);

// ---- msm_tc.cu: tcgen05 MSM, bf16, Dqk = Dv = 128 ----------------------------------------
cudaError_t launch_msm_tc_bf16(const void *q, const void *k, const void *v, void *o,
                               const MsmShape &s, float scale, uint32_t *status, int sms,
                               cudaStream_t stream, LaunchInfo *info);

// ---- fp8.cu -------------------------------------------------------------------------------
cudaError_t launch_fp8_quantize(const void *x, int x_dtype, uint8_t *q, float *scales,
                                int64_t rows, int64_t cols, int64_t ld_x, int64_t block,
                                int fmt_e5m2, cudaStream_t stream, LaunchInfo *info);
cudaError_t launch_gemm_fp8_tc(const uint8_t *a, int a_e5m2, const float *sa, const uint8_t *bt,
                               int b_e5m2, const float *sbt, void *c, int c_bf16, int64_t m,
                               int64_t n, int64_t k, int64_t block, uint32_t *status, int sms,
                               cudaStream_t stream, LaunchInfo *info);
cudaError_t launch_gemm_fp8_simt(const uint8_t *a, int a_e5m2, const float *sa,
                                 const uint8_t *bt, int b_e5m2, const float *sbt, void *c,
                                 int c_bf16, int64_t m, int64_t n, int64_t k, int64_t block,
                                 cudaStream_t stream, LaunchInfo *info);

// Strict pairs with M*N at least this many elements run as two tiled
// launches through a binary32 C [M,N] in device scratch (api.cpp); the plan
// sizes its workspace by the same rule (plan.cpp).
constexpr int64_t kStrictTwoPassMinElems = 16384;

// ---- typed.cu: int8 and bf16-fma typed GEMMs -------------------------------------------------
cudaError_t launch_transpose_u8(const void *in, void *out, int64_t rows, int64_t cols,
                                int64_t ld_in, cudaStream_t stream);
// b_mn = 1: b is B [K,N] (row stride ldb), read MN-major; b_mn = 0: b is
// Bt [N,K] (row stride ldb), read K-major. Returns cudaErrorNotSupported when
// a stride or base is not 16-byte aligned or k == 0.
// Zero points of a quantized int8 GEMM, C = sum_k (A - za)(B - zb) modulo
// 2^32, applied in the epilogue as C = A.B + k*za*zb - zb*row_sum[m] -
// za*col_sum[n] (an identity in wrapping int32 arithmetic). row_sum is
// needed when zb != 0, col_sum when za != 0 (each 16-byte aligned).
struct I8ZeroPoints {
  int32_t za = 0, zb = 0;
  const int32_t *row_sum = nullptr;  // sum_k A[m,k], M entries
  const int32_t *col_sum = nullptr;  // sum_k B[k,n], N entries
};
cudaError_t launch_gemm_i8_tc(const int8_t *a, int64_t lda, const int8_t *b, int64_t ldb,
                              int b_mn, int32_t *c, int64_t m, int64_t n, int64_t k, int64_t ld_c,
                              const I8ZeroPoints *zp, uint32_t *status, int sms,
                              cudaStream_t stream, LaunchInfo *info);
// The sums I8ZeroPoints needs: row_sum of A [M,K] (when zb != 0) and col_sum
// of B (when za != 0), B given as [K,N] (b_mn = 1, row stride ldb) or as its
// transpose Bt [N,K] (b_mn = 0). Rows must be 16-byte aligned for the
// vector path (other strides use byte loads).
cudaError_t launch_i8_zero_point_sums(const int8_t *a, int64_t lda, const int8_t *b, int64_t ldb,
                                      int b_mn, int64_t m, int64_t n, int64_t k,
                                      const I8ZeroPoints &zp, int32_t *row_sum, int32_t *col_sum,
                                      int sms, cudaStream_t stream, LaunchInfo *info);
cudaError_t launch_gemm_i8_simt(const int8_t *a, const int8_t *b, int32_t *c, int64_t m, int64_t n,
                                int64_t k, int64_t lda, int64_t ldb, int64_t ldc, int32_t za,
                                int32_t zb, cudaStream_t stream, LaunchInfo *info);
cudaError_t launch_gemm_bf16_fma(const void *a, const void *b, float *c, int64_t m, int64_t n,
                                 int64_t k, int64_t lda, int64_t ldb, int64_t ldc,
                                 cudaStream_t stream, LaunchInfo *info);

// ---- region.cu: block_attn_res (reference region op) ---------------------------------------
cudaError_t launch_block_attn_res(const float *blocks, const float *partial, const float *query,
                                  float *out, int64_t rows, int64_t d, int64_t block_stride,
                                  int block_count, int has_partial, float eps, int sms,
                                  cudaStream_t stream, LaunchInfo *info);

// ---- rmsnorm (attention block) -------------------------------------------------------------
// attn_proj2 (optional): a second bf16 partial of the projection, added after attn_proj.
cudaError_t launch_residual_rmsnorm(const void *x, const void *attn_proj, void *y, int64_t rows,
                                    int64_t cols, float eps, cudaStream_t stream,
                                    LaunchInfo *info, const void *attn_proj2 = nullptr);

// ---- peer.cu: flags between the two GPUs of a head-sharded pair -----------------------------
// One thread spins (bounded by `limit` clock64 cycles, nanosleep between
// polls) until the 32-bit step counter at `flag` (this GPU's memory, written
// by the peer) reaches `target`; on timeout it sets kErrTimeoutRemote in
// *status and returns.
cudaError_t launch_peer_wait(const uint32_t *flag, uint32_t target, long long limit,
                             uint32_t *status, cudaStream_t stream);
// One thread makes every earlier write of this stream visible system-wide,
// then stores `value` to `flag` (the peer's memory) with release semantics.
cudaError_t launch_peer_signal(uint32_t *flag, uint32_t value, cudaStream_t stream);

// Tensor-map encoder (driver entry point fetched once through the runtime).
bool encode_tmap_2d(CUtensorMap *map, CUtensorMapDataType dtype, const void *base,
                    uint64_t inner, uint64_t outer, uint64_t row_stride_bytes, uint32_t box_inner,
                    uint32_t box_outer, CUtensorMapSwizzle swizzle);
bool encode_tmap_3d(CUtensorMap *map, CUtensorMapDataType dtype, const void *base,
                    uint64_t d0, uint64_t d1, uint64_t d2, uint64_t stride1_bytes,
                    uint64_t stride2_bytes, uint32_t box0, uint32_t box1, uint32_t box2,
                    CUtensorMapSwizzle swizzle);

}  // namespace mcb

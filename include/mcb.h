/*
 * mcb.h -- C ABI of the B200 (sm_100a) implementation of MatcoreDSL's
 * data-parallel hot path: strict f32 GEMM and fused GEMM pair, bf16 GEMM with
 * a fused epilogue (Family A), matmul-softmax-matmul (Family C), the FP8
 * block-scaled GEMM, and the attention-residual block region.
 *
 * Every entry point is extern "C", noexcept, takes plain pointers and sizes,
 * and reports failure only through its return code. Each declaration names
 * the MatcoreDSL interface (path:line in the MatcoreDSL repository) it
 * replaces.
 *
 * Conventions
 *  - Ownership: the caller owns every buffer. Operands may live in host
 *    memory (MCB_MEMORY_HOST: the library stages them through device buffers
 *    on the caller's stream and synchronises before returning) or in device
 *    memory (MCB_MEMORY_CUDA_DEVICE: the call is asynchronous on the stream
 *    unless MCB_EXEC_SYNC is set). All operands of one call must live in the
 *    same memory space.
 *  - Scratch: an entry point that needs device scratch for intermediates
 *    uses mcb_exec.workspace when it holds enough bytes at a 16-byte aligned
 *    base; otherwise it allocates stream-ordered from a memory pool the
 *    library owns on that device (released on the stream when the call ends;
 *    the pool keeps up to 4 GiB reserved between calls), so device-resident
 *    calls stay asynchronous either way. Only if that allocation fails does
 *    the call fall back to a shared staging buffer and synchronise.
 *  - Layout: dims and strides are in elements, row-major, innermost stride 1.
 *  - Errors: all failures return a status; nothing throws across this
 *    boundary. Device-side pipeline stalls are bounded: a kernel that waits
 *    too long records a bit in the per-device status word and exits, and a
 *    synchronous call then returns MCB_STATUS_DEVICE_TIMEOUT.
 *  - Threading: calls on distinct streams are independent; the only global
 *    state is a lazily created per-device context guarded by a mutex. One
 *    exception: GEMM launches that take the stream-K route share a per-device
 *    workspace, so the library orders each such launch after the previous
 *    one on that device (an event wait when they are on different streams).
 */
#ifndef MCB_H
#define MCB_H

#include <stddef.h>
#include <stdint.h>

#if defined(__cplusplus)
#define MCB_NOEXCEPT noexcept
extern "C" {
#else
#define MCB_NOEXCEPT
#endif

#if defined(_WIN32)
#define MCB_API
#else
#define MCB_API __attribute__((visibility("default")))
#endif

#define MCB_ABI_VERSION_V1 UINT32_C(1)
#define MCB_MAX_RANK 4

/* Status codes. 0-26 keep the numbering of MatcoreDSL's runtime C ABI
 * (compiler/include/matcore/runtime_c.h:77-104); 40+ are device-side codes
 * that mirror closed_host_v1::Code (compiler/include/matcore/detail/
 * region_storage.h:16-21) where the meaning matches. */
typedef int32_t mcb_status;
enum {
  MCB_STATUS_OK = 0,
  MCB_STATUS_INVALID_ARGUMENT = 1,
  MCB_STATUS_ABI_MISMATCH = 2,
  MCB_STATUS_UNSUPPORTED_DTYPE = 3,
  MCB_STATUS_UNSUPPORTED_RANK = 4,
  MCB_STATUS_INVALID_SHAPE = 5,
  MCB_STATUS_UNSUPPORTED_LAYOUT = 6,
  MCB_STATUS_UNSUPPORTED_MEMORY_SPACE = 7,
  MCB_STATUS_MIXED_MEMORY_SPACES = 8,
  MCB_STATUS_OUTPUT_NOT_MUTABLE = 9,
  MCB_STATUS_SHAPE_MISMATCH = 11,
  MCB_STATUS_ALIAS_VIOLATION = 12,
  MCB_STATUS_ARITHMETIC_OVERFLOW = 15,
  MCB_STATUS_INVALID_ALIGNMENT = 16,
  MCB_STATUS_INSUFFICIENT_WORKSPACE = 17,
  MCB_STATUS_UNAVAILABLE_VARIANT = 18,
  MCB_STATUS_ALLOCATION_FAILURE = 40,   /* Code::allocation_failure */
  MCB_STATUS_CANDIDATE_FAILURE = 41,    /* Code::candidate_failure (CUDA error) */
  MCB_STATUS_CANDIDATE_UNAVAILABLE = 42,/* Code::candidate_unavailable (no sm_100 GPU) */
  MCB_STATUS_DEVICE_TIMEOUT = 43,       /* a bounded device-side wait expired */
  MCB_STATUS_STALE_HANDLE = 44          /* device buffer handle freed or unknown */
};

/* Element types; 1-5 keep runtime_c.h:38-46 numbering. */
typedef uint32_t mcb_dtype;
enum {
  MCB_DTYPE_INVALID = 0,
  MCB_DTYPE_F32 = 1,
  MCB_DTYPE_F64 = 2,
  MCB_DTYPE_BF16 = 3,
  MCB_DTYPE_I8 = 4,
  MCB_DTYPE_I32 = 5,
  MCB_DTYPE_F16 = 6,
  MCB_DTYPE_E4M3 = 7, /* OCP float8 e4m3 ("fn": no Inf, max 448) */
  MCB_DTYPE_E5M2 = 8  /* OCP float8 e5m2 (IEEE-style Inf/NaN, max 57344) */
};

typedef uint32_t mcb_memory_space;
enum { MCB_MEMORY_INVALID = 0, MCB_MEMORY_HOST = 1, MCB_MEMORY_CUDA_DEVICE = 2 };

/* Tensor descriptor; mirrors matcore_tensor_desc_v0
 * (compiler/include/matcore/runtime_c.h:107-118) and RuntimeTensorView
 * (include/matcore/kernel_ir.h:274-283). Set abi_version = MCB_ABI_VERSION_V1
 * and struct_size = sizeof(mcb_tensor). */
typedef struct mcb_tensor {
  uint32_t abi_version;
  uint32_t struct_size;
  void *data;
  mcb_dtype dtype;
  uint32_t rank;
  int64_t dims[MCB_MAX_RANK];
  int64_t strides[MCB_MAX_RANK];
  mcb_memory_space memory_space;
  uint32_t reserved0;
  uint64_t reserved[2];
} mcb_tensor;

/* Per-call report: which kernel ran and what it moved. Mirrors the roles of
 * CompilationStats (include/matcore/jit_runner.h:13-21) and CandidateReport
 * (compiler/lib/runtime/closed_host_v1.h:29-44). */
typedef struct mcb_report {
  uint32_t abi_version;
  uint32_t struct_size;
  char route[48];          /* e.g. "tcgen05_bf16_gemm_epilogue" */
  int32_t kernel_launches; /* launches this call issued */
  int32_t tile_m, tile_n, tile_k, stages, ctas;
  float kernel_ms;         /* device time of the compute kernels (MCB_EXEC_TIME) */
  float h2d_ms, d2h_ms;    /* staging copies (MCB_EXEC_TIME, host operands) */
  uint64_t h2d_bytes, d2h_bytes;
  uint32_t device_status;  /* device status word after a synchronous call */
  uint32_t route_flags;    /* MCB_ROUTE_* bits describing how the route ran */
} mcb_report;
/* report->route_flags: the CTA-pair GEMM split the K-block ranges of some
 * tiles over several clusters (stream-K) to fill every SM. */
enum { MCB_ROUTE_STREAM_K = 1u << 0 };

/* Execution context: device, stream and options for one call. */
enum {
  MCB_EXEC_SYNC = 1u << 0, /* synchronise the stream before returning */
  MCB_EXEC_TIME = 1u << 1  /* fill report->kernel_ms / h2d_ms / d2h_ms (implies SYNC) */
};
typedef struct mcb_exec {
  uint32_t abi_version;
  uint32_t struct_size;
  int32_t device;          /* CUDA ordinal, -1 = the calling thread's current device */
  uint32_t flags;
  void *stream;            /* cudaStream_t, NULL = the legacy default stream */
  void *workspace;         /* optional device scratch supplied by the caller */
  uint64_t workspace_bytes;
  mcb_report *report;      /* optional */
  uint64_t reserved[2];
} mcb_exec;

/* ---- library ------------------------------------------------------------ */
MCB_API uint32_t mcb_abi_version(void) MCB_NOEXCEPT;
MCB_API const char *mcb_status_message(mcb_status code) MCB_NOEXCEPT;
/* Reads (and with clear != 0 resets) the device status word of `device`. */
MCB_API mcb_status mcb_device_status(int32_t device, uint32_t *word, int32_t clear) MCB_NOEXCEPT;
/* Self-test of the bounded device waits, the counterpart of the reference
 * adapter's poison domain (compiler/lib/runtime/closed_cuda_candidate_v1.cpp:86-120):
 * runs one tensor-core GEMM tile on `device` whose loads are never issued,
 * so its pipeline wait gives up after `spin_limit_cycles` (10^4..4*10^9
 * clock64 cycles; ordinary launches use ~2 s). Returns
 * MCB_STATUS_DEVICE_TIMEOUT when the kernel returned and reported the stall
 * (bit 0, "producer data never arrived", set in the device status word,
 * which stays set until cleared with mcb_device_status). Synchronises the
 * device; allocates 112 KiB for the call. */
MCB_API mcb_status mcb_device_timeout_selftest_v1(int32_t device,
                                                  uint64_t spin_limit_cycles) MCB_NOEXCEPT;
/* The same for the one wait on another CTA cluster: a stream-K GEMM (two
 * 256x256 tiles, K = 4096, each split over two clusters) whose tail parts
 * never raise their ready flags, so each owner's wait gives up after
 * `spin_limit_cycles` (same range). Returns MCB_STATUS_DEVICE_TIMEOUT when
 * the kernel returned and reported it (bit 5, "another CTA's stream-K partial
 * never arrived", sticky like bit 0). Synchronises the device; allocates
 * about 8.3 MiB for the call. */
MCB_API mcb_status mcb_device_peer_timeout_selftest_v1(int32_t device,
                                                       uint64_t spin_limit_cycles) MCB_NOEXCEPT;
/* Ok when `device` is an sm_100 GPU this build can run on; replaces
 * detail::cudaCandidateAvailable (compiler/lib/runtime/closed_cuda_candidate_v1.h:13). */
MCB_API mcb_status mcb_candidate_available(int32_t device) MCB_NOEXCEPT;

/* ---- strict f32 (bit-exact with the reference's strict leaf) ------------- */
/* C = A*B with a separate binary32 multiply and add per step, increasing k,
 * +0 seed (compiler/lib/runtime/closed_host_v1.cpp:401-415). Replaces
 * detail::cudaGemmCandidate (compiler/lib/runtime/closed_cuda_candidate_v1.h:14). */
MCB_API mcb_status mcb_strict_gemm_f32_v1(const mcb_tensor *c, const mcb_tensor *a,
                                          const mcb_tensor *b, const mcb_exec *exec) MCB_NOEXCEPT;
/* E = (A*B)*D with the intermediate rounded to binary32 and never written to
 * the caller (compiler/lib/mlir/MatcoreCpuFusedGemmCandidate.h:19-31).
 * Replaces detail::cudaFusedPairCandidate
 * (compiler/lib/runtime/closed_cuda_candidate_v1.h:19-20). K may be 0 (E =
 * +0*D, so Inf/NaN in D propagate); N = 0 gives E = +0. */
MCB_API mcb_status mcb_strict_fused_pair_f32_v1(const mcb_tensor *e, const mcb_tensor *a,
                                                const mcb_tensor *b, const mcb_tensor *d,
                                                const mcb_exec *exec) MCB_NOEXCEPT;

/* Allocation-free variant of mcb_strict_fused_pair_f32_v1, for callers that
 * cannot call cudaMalloc: a host framework that owns every byte of device
 * memory through its own pool, a latency-critical path that must not trigger
 * cudaMalloc's implicit device-wide synchronisation, or code that must not
 * fail for lack of memory midway through a run. It has no counterpart in the
 * reference. Same bit-exact result; the intermediate panel lives in a fixed
 * 8 MiB array (2^21 floats) compiled into the library and held on every GPU
 * that loads it until exit. Limits: all operands device-resident
 * (MCB_STATUS_UNSUPPORTED_MEMORY_SPACE otherwise), N <= 2^21
 * (MCB_STATUS_INSUFFICIENT_WORKSPACE otherwise), MCB_EXEC_TIME not accepted.
 * The first call on each device performs a one-time set-up (it looks up the
 * array's device address) and should come before any stream capture. All
 * calls share the array: calls that overlap on the GPU race and must be
 * serialised by the caller. */
MCB_API mcb_status mcb_strict_fused_pair_f32_noalloc_v1(const mcb_tensor *e, const mcb_tensor *a,
                                                        const mcb_tensor *b, const mcb_tensor *d,
                                                        const mcb_exec *exec) MCB_NOEXCEPT;

/* ---- typed isolated GEMMs (bit-exact with the reference's typed references) */
/* C[M,N] int32 = A[M,K] int8 * B[K,N] int8, accumulated modulo 2^32. Runs on
 * tcgen05 (kind::i8) when A's rows and C are 16-byte aligned: B is read in
 * place when its rows are 16-byte aligned, else (K a multiple of 16) it is
 * transposed into device scratch first. Other layouts run on CUDA cores;
 * integer sums are exact either way. Counterpart of
 * cpu_reference_gemm_i8_i32_v1
 * (compiler/lib/runtime/cpu_numeric_reference.h:58-61, .cpp:185-209). */
MCB_API mcb_status mcb_gemm_i8_i32_v1(const mcb_tensor *c, const mcb_tensor *a,
                                      const mcb_tensor *b, const mcb_exec *exec) MCB_NOEXCEPT;
/* Quantized matmul with zero points: C[m,n] = sum_k (A[m,k] - a_zero_point) *
 * (B[k,n] - b_zero_point) in wrapping int32 arithmetic, the legacy int8
 * path's linalg.quantized_matmul (src/mlir_engine.cpp:944-958; the zero
 * point of each operand is its own when its quantization is enabled, else
 * the kernel's global one: the caller passes the resolved values). Same
 * routes as mcb_gemm_i8_i32_v1; on tcgen05 the raw codes are multiplied and
 * the epilogue adds K*za*zb - zb*rowsum(A) - za*colsum(B) (one pre-pass
 * computes the sums into device scratch). Zero points 0 give
 * mcb_gemm_i8_i32_v1's result. */
MCB_API mcb_status mcb_gemm_i8_i32_zp_v1(const mcb_tensor *c, const mcb_tensor *a,
                                         const mcb_tensor *b, int32_t a_zero_point,
                                         int32_t b_zero_point,
                                         const mcb_exec *exec) MCB_NOEXCEPT;
/* C[M,N] f32 = A[M,K] bf16 * B[K,N] bf16 with one f32 fma per k in
 * increasing order from +0 (CUDA cores; bit-exact). Counterpart of
 * cpu_reference_gemm_bf16_f32_v1 (cpu_numeric_reference.h:45-48, .cpp:108-127). */
MCB_API mcb_status mcb_gemm_bf16_f32_fma_v1(const mcb_tensor *c, const mcb_tensor *a,
                                            const mcb_tensor *b,
                                            const mcb_exec *exec) MCB_NOEXCEPT;

/* ---- Family A: GEMM + fused epilogue ------------------------------------ */
enum { MCB_BIAS_NONE = 0, MCB_BIAS_ROW = 1 /* b[N] broadcast over rows */,
       MCB_BIAS_FULL = 2 /* boundary [M,N] */ };
enum { MCB_BIAS_ADD = 0 /* acc + b */, MCB_BIAS_RSUB = 1 /* b - acc */ };
enum { MCB_ACT_NONE = 0, MCB_ACT_RELU = 1, MCB_ACT_GELU_TANH = 2, MCB_ACT_EXP = 3,
       MCB_ACT_SIGMOID = 4, MCB_ACT_TANH = 5 };
typedef struct mcb_epilogue {
  uint32_t abi_version;
  uint32_t struct_size;
  uint32_t bias_mode;
  uint32_t bias_op;
  uint32_t activation;   /* applied after the bias */
  uint32_t reserved0;
  uint64_t reserved[2];
} mcb_epilogue;
/* Y = act(X*W (+|r-) bias). X [M,K], W [K,N] (row-major, "MN-major" B) or,
 * with w given as [N,K] and rank-2 dims {N,K} plus MCB_GEMM_W_TRANSPOSED in
 * flags, W^T. X and W are both bf16, both f16 or both f32 (the reference's
 * matmul signatures, src/mlir_engine.cpp:114-152). 16-bit X/W with 16-byte
 * aligned rows run on tcgen05 tensor cores (kind::f16, bf16 or f16 operand
 * format) with an f32 TMEM accumulator; f32 X/W and unaligned rows run on
 * CUDA cores with f32 FMA accumulation. Output f32 or the inputs' 16-bit
 * type; bias f32, bf16 or f16. GELU is the tanh form of
 * src/fusion_emitter_common.cpp:86-108.
 * Replaces the Family A leaf emitted by FusionMlirEmitter::emitFamilyA
 * (src/fusion_emitter_family_a.cpp:12-244) and reached through compileAndRun
 * (include/matcore/jit_runner.h:23-26).
 * Host-memory operands (without MCB_EXEC_TIME) move in row chunks: W and a
 * row bias first, then each chunk's X rows (and full-bias rows) up, GEMM and
 * Y rows down, overlapped on separate streams; a call that fails part-way may
 * already have written the Y rows of completed chunks. */
enum { MCB_GEMM_W_TRANSPOSED = 1u << 0 };
MCB_API mcb_status mcb_gemm_epilogue_v1(const mcb_tensor *y, const mcb_tensor *x,
                                        const mcb_tensor *w, const mcb_tensor *bias,
                                        const mcb_epilogue *epilogue, uint32_t gemm_flags,
                                        const mcb_exec *exec) MCB_NOEXCEPT;

/* General Family A epilogue chain: Y = op_n(...op_1(X*W)...), the chain
 * FusionMlirEmitter::emitFamilyA accepts (src/fusion_emitter_family_a.cpp:
 * 149-220; op semantics src/fusion_emitter_common.cpp:38-160). Each op is
 * unary, or binary against an exact-shape [M,N] boundary tensor with the
 * running value on the left (value_pos 0: v op b) or right (1: b op v).
 * Up to MCB_EPILOGUE_MAX_OPS ops and MCB_EPILOGUE_MAX_BOUNDARIES boundaries
 * (f32, bf16 or f16, any row stride). Arithmetic is f32 on the accumulator;
 * relu / min / max propagate NaN and order -0 < +0 (arith.maximumf /
 * minimumf). Same kernels and routes as mcb_gemm_epilogue_v1. */
enum {
  MCB_EW_RELU = 1, MCB_EW_EXP = 2, MCB_EW_LOG = 3, MCB_EW_TANH = 4, MCB_EW_SQRT = 5,
  MCB_EW_NEG = 6, MCB_EW_ABS = 7, MCB_EW_SIN = 8, MCB_EW_COS = 9, MCB_EW_RSQRT = 10,
  MCB_EW_SIGMOID = 11, MCB_EW_GELU_TANH = 12,
  MCB_EW_ADD = 32, MCB_EW_SUB = 33, MCB_EW_MUL = 34, MCB_EW_DIV = 35, MCB_EW_MIN = 36,
  MCB_EW_MAX = 37
};
#define MCB_EPILOGUE_MAX_OPS 8
#define MCB_EPILOGUE_MAX_BOUNDARIES 4
typedef struct mcb_epilogue_op {
  uint32_t kind;      /* MCB_EW_* */
  uint32_t value_pos; /* binary: 0 = v op boundary, 1 = boundary op v */
  uint32_t boundary;  /* binary: index into `boundaries` */
  uint32_t reserved;
} mcb_epilogue_op;
MCB_API mcb_status mcb_gemm_epilogue_chain_v1(const mcb_tensor *y, const mcb_tensor *x,
                                              const mcb_tensor *w,
                                              const mcb_tensor *boundaries,
                                              uint32_t num_boundaries,
                                              const mcb_epilogue_op *ops, uint32_t num_ops,
                                              uint32_t gemm_flags,
                                              const mcb_exec *exec) MCB_NOEXCEPT;

/* ---- Family B: two-GEMM chain with elementwise glue ------------------------ */
/* E = glue(A*B) * W where glue is a Family A epilogue (optional boundary
 * [M,N1] or row bias [N1], added or reverse-subtracted, then one activation).
 * A [M,K], B [K,N1], W [N1,N2], E [M,N2]. The glue is fused into the first
 * GEMM's epilogue; the intermediate (bf16 for bf16 operands, f32 for f32) is
 * kept in device scratch (M*N1 elements; see Scratch above) and consumed by
 * the second GEMM. bf16 runs on
 * tcgen05, f32 on CUDA cores. Replaces the leaf emitted by
 * FusionMlirEmitter::emitFamilyB (src/fusion_emitter_family_b.cpp:12-408). */
MCB_API mcb_status mcb_gemm_chain_v1(const mcb_tensor *e, const mcb_tensor *a,
                                     const mcb_tensor *b, const mcb_tensor *boundary,
                                     const mcb_epilogue *glue, const mcb_tensor *w,
                                     const mcb_exec *exec) MCB_NOEXCEPT;

/* ---- Family C: matmul-softmax-matmul -------------------------------------- */
/* O = softmax(scale * Q*K^T) * V per leading index. Q [.., M, Dqk],
 * K [.., N, Dqk], V [.., N, Dv], O [.., M, Dv] with up to two leading
 * (batch, head) dims. scale = 1 gives the reference's unscaled softmax
 * (tests/test_family_c.py:102-113). bf16 with Dqk = Dv = 64 or 128 (any M
 * and N, 16-byte aligned rows) runs the tcgen05 kernels (S and O in TMEM, online
 * softmax, S never in HBM); other shapes and f32 run a CUDA-core
 * online-softmax kernel. Replaces the kernel emitted by
 * FusionMlirEmitter::emitFamilyC (src/fusion_emitter_family_c.cpp:13-596). */
MCB_API mcb_status mcb_msm_v1(const mcb_tensor *o, const mcb_tensor *q, const mcb_tensor *k,
                              const mcb_tensor *v, double scale,
                              const mcb_exec *exec) MCB_NOEXCEPT;

/* ---- FP8 block-scaled GEMM ------------------------------------------------ */
/* Per-(block x block) absmax quantisation of an f32 or bf16 matrix:
 * s = absmax/fmt_max (1 for an all-zero block), q = sat_RNE(x/s). scales is
 * f32 [ceil(rows/block), ceil(cols/block)]. */
MCB_API mcb_status mcb_fp8_quantize_blockwise_v1(const mcb_tensor *q, const mcb_tensor *scales,
                                                 const mcb_tensor *x, int64_t block,
                                                 const mcb_exec *exec) MCB_NOEXCEPT;
/* C = (sa.A) * (sb.B)^T... precisely C[m,n] = sum_k sa[m/b,k/b] A[m,k] *
 * sbt[n/b,k/b] Bt[n,k]: A [M,K] and Bt [N,K] are e4m3/e5m2 codes (K-major),
 * fp32 accumulation, C bf16 or f32. Replaces the throwing
 * runFp8WgmmaPreflight (src/lowering_pipeline.cpp:2531-2572). */
MCB_API mcb_status mcb_gemm_fp8_blockscaled_v1(const mcb_tensor *c, const mcb_tensor *a,
                                               const mcb_tensor *sa, const mcb_tensor *bt,
                                               const mcb_tensor *sbt, int64_t block,
                                               const mcb_exec *exec) MCB_NOEXCEPT;
/* Tile policy of getFp8WgmmaTileConfig / isLegalFp8WgmmaShape
 * (src/fp8_wgmma.cpp:10-24,61-109), kept for callers that query it. */
typedef struct mcb_fp8_tile_config {
  int32_t m_tile, n_tile, k_tile, use_tma;
} mcb_fp8_tile_config;
MCB_API int32_t mcb_fp8_is_legal_shape_v1(int64_t m, int64_t n, int64_t k) MCB_NOEXCEPT;
MCB_API mcb_fp8_tile_config mcb_fp8_tile_config_v1(int64_t m, int64_t n,
                                                   int64_t k) MCB_NOEXCEPT;

/* ---- block_attn_res region op (the reference's region_v1 operator) ------------ */
/* Depth attention over packed block history, f32: for every (b, t), sources
 * = blocks[0..block_count) (+ partial when has_partial); each source row is
 * RMS-normalised over D (eps) and dotted with query; softmax over sources;
 * out = weighted sum of the raw source rows (zeros when there is no source).
 * blocks [MAX_BLOCKS<=32, B, T, D], partial/out [B, T, D], query [D], all
 * dense f32. Replaces the kernel RegionMlirEmitter::emitBlockAttnRes emits
 * (src/region_emitter_block_attn_res.cpp:38-432); argument rules of
 * matcore/frontend.py:1734-1765. */
MCB_API mcb_status mcb_block_attn_res_v1(const mcb_tensor *out, const mcb_tensor *blocks,
                                         const mcb_tensor *partial, const mcb_tensor *query,
                                         int64_t block_count, int32_t has_partial, float eps,
                                         const mcb_exec *exec) MCB_NOEXCEPT;

/* ---- attention-residual block region ------------------------------------------- */
/* Y = RMSNorm(X + Wo * MSM(X Wq, X Wk, X Wv)) with unit gain; X [B,S,D] bf16,
 * W* [D,D] bf16, `heads` heads of D/heads, softmax scale (D/heads)^-0.5.
 * Composed from the kernels above with device-resident intermediates in
 * scratch of mcb_attn_block_workspace_bytes_v1 bytes (see Scratch above). Named after the
 * region path of RegionMlirEmitter (src/region_emitter_block_attn_res.cpp:38-432). */
MCB_API uint64_t mcb_attn_block_workspace_bytes_v1(int64_t batch, int64_t seq,
                                                   int64_t d_model) MCB_NOEXCEPT;
MCB_API mcb_status mcb_attn_block_region_v1(const mcb_tensor *y, const mcb_tensor *x,
                                            const mcb_tensor *wq, const mcb_tensor *wk,
                                            const mcb_tensor *wv, const mcb_tensor *wo,
                                            int64_t heads, float eps,
                                            const mcb_exec *exec) MCB_NOEXCEPT;

/* Head-sharded form of the region, for a batch too small to split over the
 * GPUs (batch x heads sharding; no counterpart in the single-GPU reference).
 * mcb_attn_block_heads_v1 computes one head group's share of the output
 * projection, P = MSM(X Wq_g, X Wk_g, X Wv_g) Wo_g: X [B,S,D] and P [B,S,D]
 * dense bf16; Wq_g, Wk_g, Wv_g [D,Dh] the group's column slices of Wq, Wk,
 * Wv and Wo_g [Dh,D] the matching row slice of Wo, all dense bf16; `heads`
 * heads of Dh/heads, softmax scale (Dh/heads)^-0.5 (the region's, since the
 * head width is the same). Scratch: mcb_attn_block_heads_workspace_bytes_v1.
 * Summing P over the head groups (mcb_reduce_scatter_v1 across GPUs) gives
 * the region's Wo * MSM(...); mcb_residual_rmsnorm_v1 then writes
 * Y = RMSNorm(X + sum P) for any dense [.., D] bf16 rows (D <= 8192), the
 * region's last step. */
MCB_API uint64_t mcb_attn_block_heads_workspace_bytes_v1(int64_t batch, int64_t seq,
                                                         int64_t d_heads) MCB_NOEXCEPT;
MCB_API mcb_status mcb_attn_block_heads_v1(const mcb_tensor *p, const mcb_tensor *x,
                                           const mcb_tensor *wq, const mcb_tensor *wk,
                                           const mcb_tensor *wv, const mcb_tensor *wo,
                                           int64_t heads, const mcb_exec *exec) MCB_NOEXCEPT;
MCB_API mcb_status mcb_residual_rmsnorm_v1(const mcb_tensor *y, const mcb_tensor *x,
                                           const mcb_tensor *p, float eps,
                                           const mcb_exec *exec) MCB_NOEXCEPT;

/* Two head groups on two GPUs with the exchange fused into the output
 * projection (no counterpart in the reference). Each GPU of the pair creates
 * its side with mcb_peer_exchange_create_v1 (a device allocation for
 * `recv_bytes` of received rows plus two step counters) and gets an IPC
 * handle, which the caller passes to the other process out of band; each
 * then calls mcb_peer_exchange_connect_v1 with the other's handle.
 * mcb_attn_block_heads_pair_v1 then computes, on GPU `group` (0 or 1), the
 * group's Q/K/V projections and MSM, and the output projection in two row
 * halves: the other GPU's rows are stored straight into that GPU's receive
 * buffer by the GEMM's epilogue (NVLink stores that overlap the math), the
 * own rows locally; after the other GPU's counter says its share has arrived
 * it writes Y = RMSNorm(X_own + P_own + P_received) for its half of the rows.
 * X [B,S,D] (the pair's batch elements), W* as in mcb_attn_block_heads_v1,
 * Y [B*S/2, D] (rows [group*B*S/2, (group+1)*B*S/2) of X), all dense bf16 in
 * device memory; recv_bytes >= B*S/2 * D * 2. Both GPUs must make the same
 * calls in the same order; waits on the other GPU give up after ~2 s with
 * MCB_STATUS_DEVICE_TIMEOUT (the pair must then be destroyed and recreated).
 * Destroy only after both GPUs have finished their calls. */
typedef struct mcb_peer_exchange mcb_peer_exchange;
typedef struct mcb_ipc_handle {
  char internal[64];
} mcb_ipc_handle;
MCB_API mcb_status mcb_peer_exchange_create_v1(int32_t device, uint64_t recv_bytes,
                                               mcb_peer_exchange **out,
                                               mcb_ipc_handle *handle) MCB_NOEXCEPT;
MCB_API mcb_status mcb_peer_exchange_connect_v1(mcb_peer_exchange *x,
                                                const mcb_ipc_handle *peer) MCB_NOEXCEPT;
MCB_API mcb_status mcb_peer_exchange_destroy_v1(mcb_peer_exchange *x) MCB_NOEXCEPT;
MCB_API mcb_status mcb_attn_block_heads_pair_v1(const mcb_tensor *y, const mcb_tensor *x,
                                                const mcb_tensor *wq, const mcb_tensor *wk,
                                                const mcb_tensor *wv, const mcb_tensor *wo,
                                                int64_t heads, float eps, int32_t group,
                                                mcb_peer_exchange *exchange,
                                                const mcb_exec *exec) MCB_NOEXCEPT;

/* ---- execution plans (shape-locked, optional CUDA-graph replay) ------------ */
/* Mirrors MatcorePlan::create / execute (include/matcore/plan.h:37-107): a
 * plan freezes the operator and the metadata (dtype, rank, dims, strides,
 * memory space) of its tensors; execute rejects tensors that differ. With
 * graph_mode = 1 the first execute captures the operator's launches into a
 * CUDA graph on a stream the plan owns, and later executes replay it; like
 * the reference, replay rejects data-pointer changes
 * (src/jit_runner.cpp:1060-1111). Graph plans need device-resident tensors;
 * ops that need scratch (GEMM_CHAIN, ATTN_BLOCK) get a workspace the plan
 * allocates once at create time. Tensor slots follow each entry point's
 * argument order; an optional slot (bias / boundary) is a tensor with
 * dtype MCB_DTYPE_INVALID. */
enum {
  MCB_PLAN_STRICT_PAIR = 1,   /* e, a, b, d */
  MCB_PLAN_STRICT_GEMM = 2,   /* c, a, b */
  MCB_PLAN_GEMM_EPILOGUE = 3, /* y, x, w, bias */
  MCB_PLAN_GEMM_CHAIN = 4,    /* e, a, b, boundary, w */
  MCB_PLAN_MSM = 5,           /* o, q, k, v */
  MCB_PLAN_FP8_GEMM = 6,      /* c, a, sa, bt, sbt */
  MCB_PLAN_ATTN_BLOCK = 7,    /* y, x, wq, wk, wv, wo */
  MCB_PLAN_GEMM_I8 = 8,       /* c, a, b (zero points from the descriptor) */
  MCB_PLAN_GEMM_EPILOGUE_CHAIN = 9 /* y, x, w, boundaries[num_boundaries] (ops from the
                                      descriptor's chain extension) */
};
#define MCB_PLAN_MAX_TENSORS 8
typedef struct mcb_plan_desc {
  uint32_t abi_version;
  uint32_t struct_size;
  uint32_t op;
  uint32_t graph_mode;
  int32_t device;        /* -1 = current device */
  uint32_t num_tensors;
  mcb_tensor tensors[MCB_PLAN_MAX_TENSORS]; /* templates: metadata is frozen, data ignored */
  mcb_epilogue epilogue; /* GEMM_EPILOGUE, GEMM_CHAIN */
  uint32_t gemm_flags;   /* GEMM_EPILOGUE */
  uint32_t reserved0;
  double scale;          /* MSM */
  int64_t block;         /* FP8_GEMM */
  int64_t heads;         /* ATTN_BLOCK */
  float eps;             /* ATTN_BLOCK */
  uint32_t reserved1;
  int32_t a_zero_point;  /* GEMM_I8 */
  int32_t b_zero_point;  /* GEMM_I8 */
  uint64_t reserved;
  /* Chain extension (GEMM_EPILOGUE_CHAIN; read only when struct_size covers
   * it, so descriptors built against the smaller first layout stay valid):
   * the op list of mcb_gemm_epilogue_chain_v1, copied into the plan, and the
   * number of boundary tensors, which follow y, x, w in `tensors`. */
  uint32_t num_ops;
  uint32_t num_boundaries;
  mcb_epilogue_op ops[MCB_EPILOGUE_MAX_OPS];
} mcb_plan_desc;
/* struct_size of a descriptor without the chain extension. */
#define MCB_PLAN_DESC_BASE_SIZE ((uint32_t)offsetof(mcb_plan_desc, num_ops))
typedef struct mcb_plan mcb_plan;
MCB_API mcb_status mcb_plan_create_v1(const mcb_plan_desc *desc, mcb_plan **out) MCB_NOEXCEPT;
/* Runs the plan on `stream` (cudaStream_t, NULL = legacy default stream);
 * asynchronous with respect to the host. */
MCB_API mcb_status mcb_plan_execute_v1(mcb_plan *plan, const mcb_tensor *tensors,
                                       uint32_t num_tensors, void *stream) MCB_NOEXCEPT;
/* Monotonic id of the plan (stale-handle detection, MatcorePlan::generationId). */
MCB_API uint64_t mcb_plan_generation_v1(const mcb_plan *plan) MCB_NOEXCEPT;
MCB_API mcb_status mcb_plan_destroy_v1(mcb_plan *plan) MCB_NOEXCEPT;

/* ---- multi-GPU shard plan -------------------------------------------------- */
/* How one rank's share of a region is chosen when the path is partitioned
 * across GPUs with no collective on the data path (the reference is
 * single-GPU; this has no counterpart there). ROWS: the M rows of a GEMM
 * (configs 2 and 4), in multiples of `align`. UNITS: independent (batch,
 * head) units of a Family C call (config 3). TOKENS: the B*S tokens of an
 * attention block (config 5), where `group` = S; each rank owns a token range
 * inside one batch element (or whole batch elements) and must also compute
 * K/V for [kv_begin, kv_begin + kv_count), the batch element(s) it reads. */
enum { MCB_SHARD_ROWS = 0, MCB_SHARD_UNITS = 1, MCB_SHARD_TOKENS = 2 };
typedef struct mcb_shard {
  int64_t begin, count;       /* owned rows / units / tokens */
  int64_t kv_begin, kv_count; /* TOKENS: token range whose K/V this rank computes */
} mcb_shard;
MCB_API mcb_status mcb_shard_plan_v1(uint32_t kind, int64_t total, int64_t group, int64_t align,
                                     int32_t world, int32_t rank, mcb_shard *out) MCB_NOEXCEPT;

/* ---- optional output all-gather (NCCL) -------------------------------------- */
/* The path needs no collective: each rank computes its shard. A caller that
 * wants the whole output on every rank gathers the shards with one NCCL
 * all-gather over NVLink / NVSwitch (the optional step of the multi-GPU
 * plan; no counterpart in the single-GPU reference). Rank 0 makes an id with
 * mcb_comm_unique_id_v1 and hands it to the others out of band; every rank
 * then calls mcb_comm_init_v1 (collective, blocking) on its device.
 * mcb_allgather_v1 queues on `stream` (a cudaStream_t) the gather of
 * `bytes_per_rank` bytes from every rank into `recv` in rank order
 * (world * bytes_per_rank bytes; shards of unequal size are padded by the
 * caller); `send` may be this rank's slot of `recv`. NCCL is loaded at run
 * time (the copy already in the process if there is one); without it these
 * return MCB_STATUS_CANDIDATE_UNAVAILABLE. */
typedef struct mcb_comm mcb_comm;
typedef struct mcb_comm_id {
  char internal[128];
} mcb_comm_id;
MCB_API mcb_status mcb_comm_unique_id_v1(mcb_comm_id *out) MCB_NOEXCEPT;
MCB_API mcb_status mcb_comm_init_v1(const mcb_comm_id *id, int32_t world, int32_t rank,
                                    int32_t device, mcb_comm **out) MCB_NOEXCEPT;
MCB_API mcb_status mcb_allgather_v1(mcb_comm *comm, const void *send, void *recv,
                                    uint64_t bytes_per_rank, void *stream) MCB_NOEXCEPT;
/* mcb_reduce_scatter_v1 queues on `stream` the element-wise sum over all
 * ranks of `send` (world * count_per_rank elements of dtype MCB_DTYPE_F32 or
 * MCB_DTYPE_BF16), leaving in `recv` this rank's slot of the sum (elements
 * [rank * count_per_rank, (rank + 1) * count_per_rank)); `recv` may be this
 * rank's slot of `send`. The exchange step of the head-sharded region. */
MCB_API mcb_status mcb_reduce_scatter_v1(mcb_comm *comm, const void *send, void *recv,
                                         uint64_t count_per_rank, int32_t dtype,
                                         void *stream) MCB_NOEXCEPT;
MCB_API mcb_status mcb_comm_destroy_v1(mcb_comm *comm) MCB_NOEXCEPT;

/* ---- device buffers ------------------------------------------------------- */
/* Ownership-tracked device memory; mirrors DeviceBufferHandle and the
 * matcore_device_* functions (include/matcore/device_buffer.h:11-53): a
 * monotonic alloc_id detects stale handles after free and reuse. */
typedef struct mcb_buffer {
  uint64_t ptr;
  uint64_t size_bytes;
  uint64_t alloc_id;
  int32_t device;
  uint32_t reserved0;
} mcb_buffer;
MCB_API mcb_status mcb_device_alloc(int32_t device, uint64_t size_bytes,
                                    mcb_buffer *out) MCB_NOEXCEPT;
MCB_API mcb_status mcb_device_free(mcb_buffer handle) MCB_NOEXCEPT;
MCB_API int32_t mcb_device_is_valid(mcb_buffer handle) MCB_NOEXCEPT;
MCB_API mcb_status mcb_device_upload(mcb_buffer dst, const void *host_src,
                                     uint64_t size_bytes) MCB_NOEXCEPT;
MCB_API mcb_status mcb_device_download(void *host_dst, mcb_buffer src,
                                       uint64_t size_bytes) MCB_NOEXCEPT;
/* Stream-ordered upload / download: queued on `stream` (a cudaStream_t, NULL =
 * the legacy default stream); the call returns at once, and pinned host
 * memory (cudaHostAlloc / cudaHostRegister) lets the copy overlap device work.
 * The host buffer must stay valid until the stream reaches the copy. */
MCB_API mcb_status mcb_device_upload_async(mcb_buffer dst, const void *host_src,
                                           uint64_t size_bytes, void *stream) MCB_NOEXCEPT;
MCB_API mcb_status mcb_device_download_async(void *host_dst, mcb_buffer src,
                                             uint64_t size_bytes, void *stream) MCB_NOEXCEPT;
MCB_API mcb_status mcb_device_zero(mcb_buffer handle) MCB_NOEXCEPT;
MCB_API mcb_status mcb_device_zero_raw_on_stream(void *device_ptr, uint64_t size_bytes,
                                                 void *stream) MCB_NOEXCEPT;

/* ---- test support: host-side fault injection ------------------------------
 * The counterpart of the reference's fake-driver adapter test
 * (compiler/tests/generated_gpu/cuda_adapter_test.cpp): a table of stand-ins
 * for the CUDA runtime calls of the host path (device discovery, staging
 * allocations, host<->device copies, synchronisation) and for kernel
 * launches, so that a test can fail any one of them, on a machine without a
 * GPU. Each stand-in returns 0 for success or a CUDA runtime error code
 * (e.g. 2 = out of memory, 999 = unknown). While a table is installed:
 *  - kernels are not launched: `launch` stands in for each launch, and the
 *    "device" pointers the library hands it are whatever `malloc_device`
 *    returned;
 *  - only the strict GEMM and strict fused pair entry points and the device
 *    status / availability queries run; every other entry point returns
 *    MCB_STATUS_CANDIDATE_UNAVAILABLE;
 *  - MCB_EXEC_TIME is ignored (no events are created).
 * Installing is refused (MCB_STATUS_INVALID_ARGUMENT) once the process has
 * created a real device context; NULL removes the table and forgets the
 * device state created under it. Install and remove from one thread, with
 * no other call in flight. Not for production use. */
typedef struct mcb_hook_launch {
  const char *op;     /* "strict_gemm" or "strict_fused_pair" */
  const void *in[3];  /* A, B and (pair) D */
  void *out;          /* C, or the pair's E */
  void *scratch;      /* the pair's intermediate C when it is in device memory, else NULL */
  int64_t m, k, n, p; /* C = A[m,k] B[k,n]; E = C D[n,p] */
  int64_t ld[4];      /* row strides (elements) of A, B, D and the output */
} mcb_hook_launch;
typedef struct mcb_runtime_hooks {
  uint32_t abi_version; /* MCB_ABI_VERSION_V1 */
  uint32_t struct_size; /* sizeof(mcb_runtime_hooks) */
  int32_t (*get_device_count)(int32_t *count);
  int32_t (*get_device)(int32_t *device);
  int32_t (*set_device)(int32_t device);
  int32_t (*device_info)(int32_t device, int32_t *cc_major, int32_t *cc_minor, int32_t *sms,
                         int32_t *smem_optin_bytes);
  int32_t (*malloc_device)(void **ptr, uint64_t bytes);
  int32_t (*free_device)(void *ptr);
  int32_t (*memset_device)(void *ptr, int32_t value, uint64_t bytes);
  /* kind: 1 host->device, 2 device->host, 3 device->device */
  int32_t (*memcpy_async)(void *dst, const void *src, uint64_t bytes, int32_t kind, void *stream);
  int32_t (*memcpy2d_async)(void *dst, uint64_t dst_pitch, const void *src, uint64_t src_pitch,
                            uint64_t width_bytes, uint64_t rows, int32_t kind, void *stream);
  int32_t (*memcpy_sync)(void *dst, const void *src, uint64_t bytes, int32_t kind);
  int32_t (*stream_synchronize)(void *stream);
  int32_t (*launch)(const mcb_hook_launch *launch);
} mcb_runtime_hooks;
MCB_API mcb_status mcb_test_set_runtime_hooks_v1(const mcb_runtime_hooks *hooks) MCB_NOEXCEPT;

#if defined(__cplusplus)
}
#endif
#endif /* MCB_H */

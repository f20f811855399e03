// Execution plans: shape-locked operator calls with optional CUDA-graph
// capture and replay, the B200 counterpart of MatcorePlan
// (include/matcore/plan.h:37-107, src/jit_runner.cpp:881-1125).
//
// create   freezes the operator, its scalar parameters and every tensor's
//          metadata, initialises the device context and (for ops that need
//          scratch) allocates the plan's own workspace.
// execute  checks the tensors against the frozen metadata, then either calls
//          the operator's C entry point directly or, in graph mode, captures
//          it once on the plan's stream and replays the instantiated graph.
//          Replay requires the same data pointers as the capture.
#include <cuda_runtime.h>

#include <atomic>
#include <cstring>
#include <new>

#include "internal.h"
#include "mcb.h"

struct mcb_plan {
  mcb_plan_desc desc;
  uint64_t generation = 0;
  int device = 0;
  cudaStream_t stream = nullptr;
  cudaEvent_t ev_in = nullptr, ev_out = nullptr;
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
  void *captured[MCB_PLAN_MAX_TENSORS] = {};
  void *workspace = nullptr;
  uint64_t workspace_bytes = 0;
};

namespace {

std::atomic<uint64_t> g_next_generation{1};

bool is_optional_slot(uint32_t op, uint32_t i) {
  return (op == MCB_PLAN_GEMM_EPILOGUE && i == 3) || (op == MCB_PLAN_GEMM_CHAIN && i == 3);
}

uint32_t slots_for(const mcb_plan_desc &d) {
  switch (d.op) {
    case MCB_PLAN_STRICT_PAIR: return 4;
    case MCB_PLAN_STRICT_GEMM: return 3;
    case MCB_PLAN_GEMM_EPILOGUE: return 4;
    case MCB_PLAN_GEMM_CHAIN: return 5;
    case MCB_PLAN_MSM: return 4;
    case MCB_PLAN_FP8_GEMM: return 5;
    case MCB_PLAN_ATTN_BLOCK: return 6;
    case MCB_PLAN_GEMM_I8: return 3;
    case MCB_PLAN_GEMM_EPILOGUE_CHAIN:
      return d.num_boundaries <= MCB_EPILOGUE_MAX_BOUNDARIES ? 3 + d.num_boundaries : 0;
    default: return 0;
  }
}

bool same_meta(const mcb_tensor &a, const mcb_tensor &b) {
  if (a.dtype != b.dtype || a.rank != b.rank || a.memory_space != b.memory_space) return false;
  for (uint32_t i = 0; i < a.rank && i < MCB_MAX_RANK; ++i)
    if (a.dims[i] != b.dims[i] || a.strides[i] != b.strides[i]) return false;
  return true;
}

const mcb_tensor *slot(const mcb_tensor *t, uint32_t op, uint32_t i) {
  if (is_optional_slot(op, i) && t[i].dtype == MCB_DTYPE_INVALID) return nullptr;
  return &t[i];
}

// Calls the operator's entry point with the plan's parameters.
mcb_status run_op(const mcb_plan &p, const mcb_tensor *t, cudaStream_t stream) {
  mcb_exec ex{};
  ex.abi_version = MCB_ABI_VERSION_V1;
  ex.struct_size = sizeof(mcb_exec);
  ex.device = p.device;
  ex.stream = stream;
  ex.workspace = p.workspace;
  ex.workspace_bytes = p.workspace_bytes;
  const uint32_t op = p.desc.op;
  switch (op) {
    case MCB_PLAN_STRICT_PAIR:
      return mcb_strict_fused_pair_f32_v1(&t[0], &t[1], &t[2], &t[3], &ex);
    case MCB_PLAN_STRICT_GEMM:
      return mcb_strict_gemm_f32_v1(&t[0], &t[1], &t[2], &ex);
    case MCB_PLAN_GEMM_EPILOGUE:
      return mcb_gemm_epilogue_v1(&t[0], &t[1], &t[2], slot(t, op, 3), &p.desc.epilogue,
                                  p.desc.gemm_flags, &ex);
    case MCB_PLAN_GEMM_CHAIN:
      return mcb_gemm_chain_v1(&t[0], &t[1], &t[2], slot(t, op, 3), &p.desc.epilogue, &t[4], &ex);
    case MCB_PLAN_MSM:
      return mcb_msm_v1(&t[0], &t[1], &t[2], &t[3], p.desc.scale, &ex);
    case MCB_PLAN_FP8_GEMM:
      return mcb_gemm_fp8_blockscaled_v1(&t[0], &t[1], &t[2], &t[3], &t[4], p.desc.block, &ex);
    case MCB_PLAN_ATTN_BLOCK:
      return mcb_attn_block_region_v1(&t[0], &t[1], &t[2], &t[3], &t[4], &t[5], p.desc.heads,
                                      p.desc.eps, &ex);
    case MCB_PLAN_GEMM_I8:
      return mcb_gemm_i8_i32_zp_v1(&t[0], &t[1], &t[2], p.desc.a_zero_point,
                                   p.desc.b_zero_point, &ex);
    case MCB_PLAN_GEMM_EPILOGUE_CHAIN:
      return mcb_gemm_epilogue_chain_v1(&t[0], &t[1], &t[2],
                                        p.desc.num_boundaries ? &t[3] : nullptr,
                                        p.desc.num_boundaries, p.desc.ops, p.desc.num_ops,
                                        p.desc.gemm_flags, &ex);
    default:
      return MCB_STATUS_INVALID_ARGUMENT;
  }
}

uint64_t workspace_for(const mcb_plan_desc &d) {
  if (d.op == MCB_PLAN_ATTN_BLOCK) {
    const mcb_tensor &x = d.tensors[1];
    return mcb_attn_block_workspace_bytes_v1(x.dims[0], x.dims[1], x.dims[2]);
  }
  if (d.op == MCB_PLAN_GEMM_CHAIN) {
    const mcb_tensor &a = d.tensors[1], &b = d.tensors[2];
    const uint64_t esz = a.dtype == MCB_DTYPE_BF16 ? 2 : 4;
    return static_cast<uint64_t>(a.dims[0]) * ((b.dims[1] + 7) / 8 * 8) * esz;
  }
  if (d.op == MCB_PLAN_GEMM_I8) {
    // B^T, then the zero-point row and column sums (the int8 entry point's
    // scratch layout). The entry point transposes B when its row stride or
    // its base pointer is not 16-byte aligned; the base pointer of a later
    // execute is not known at create time, so B^T is always reserved.
    const mcb_tensor &a = d.tensors[1], &b = d.tensors[2];
    auto up16 = [](uint64_t x) { return (x + 15) & ~uint64_t{15}; };
    const uint64_t m = static_cast<uint64_t>(a.dims[0]), k = static_cast<uint64_t>(a.dims[1]);
    const uint64_t n = static_cast<uint64_t>(b.dims[1]);
    uint64_t bytes = up16(n * k);
    if (d.b_zero_point != 0) bytes += up16(m * 4);
    if (d.a_zero_point != 0) bytes += up16(n * 4);
    return bytes;
  }
  if (d.op == MCB_PLAN_STRICT_PAIR) {
    // Pairs of M*N >= kStrictTwoPassMinElems keep the binary32 C [M,N]
    // between their two launches; smaller ones use a shared-memory panel, or
    // a global panel when 4 rows of N floats exceed 227 KiB. Holding it in
    // the plan's workspace keeps allocations out of a captured graph.
    const mcb_tensor &a = d.tensors[1], &b = d.tensors[2];
    const int64_t m = a.dims[0], n = b.dims[1];
    if (m * n >= mcb::kStrictTwoPassMinElems) return static_cast<uint64_t>(m) * n * 4;
    if (n * 16 <= 227 * 1024) return 0;
    return static_cast<uint64_t>(m + 4) * n * 4;
  }
  return 0;
}

void release(mcb_plan *p) {
  if (!p) return;
  int prev = -1;
  cudaGetDevice(&prev);
  if (prev != p->device) cudaSetDevice(p->device);
  if (p->exec) cudaGraphExecDestroy(p->exec);
  if (p->graph) cudaGraphDestroy(p->graph);
  if (p->ev_in) cudaEventDestroy(p->ev_in);
  if (p->ev_out) cudaEventDestroy(p->ev_out);
  if (p->stream) cudaStreamDestroy(p->stream);
  if (p->workspace) cudaFree(p->workspace);
  if (prev >= 0 && prev != p->device) cudaSetDevice(prev);
  delete p;
}

}  // namespace

extern "C" {

MCB_API mcb_status mcb_plan_create_v1(const mcb_plan_desc *desc, mcb_plan **out) noexcept {
  if (!desc || !out) return MCB_STATUS_INVALID_ARGUMENT;
  *out = nullptr;
  if (desc->abi_version != MCB_ABI_VERSION_V1 || desc->struct_size < MCB_PLAN_DESC_BASE_SIZE)
    return MCB_STATUS_ABI_MISMATCH;
  // The plan keeps its own copy; fields past the caller's struct_size (the
  // chain extension of a descriptor built with the first layout) read as 0.
  mcb_plan_desc d;
  std::memset(&d, 0, sizeof(d));
  std::memcpy(&d, desc, desc->struct_size < sizeof(d) ? desc->struct_size : sizeof(d));
  if (d.op == MCB_PLAN_GEMM_EPILOGUE_CHAIN) {
    if (desc->struct_size < sizeof(mcb_plan_desc)) return MCB_STATUS_ABI_MISMATCH;
    if (d.num_ops == 0 || d.num_ops > MCB_EPILOGUE_MAX_OPS) return MCB_STATUS_INVALID_ARGUMENT;
  }
  const uint32_t n = slots_for(d);
  if (n == 0 || d.num_tensors != n) return MCB_STATUS_INVALID_ARGUMENT;
  for (uint32_t i = 0; i < n; ++i) {
    const mcb_tensor &t = d.tensors[i];
    if (is_optional_slot(d.op, i) && t.dtype == MCB_DTYPE_INVALID) continue;
    if (t.abi_version != MCB_ABI_VERSION_V1 || t.struct_size < sizeof(mcb_tensor))
      return MCB_STATUS_ABI_MISMATCH;
    if (d.graph_mode && t.memory_space != MCB_MEMORY_CUDA_DEVICE)
      return MCB_STATUS_UNSUPPORTED_MEMORY_SPACE;
  }
  int dev = d.device;
  int count = 0;
  if (cudaGetDeviceCount(&count) != cudaSuccess || count == 0) {
    cudaGetLastError();
    return MCB_STATUS_CANDIDATE_UNAVAILABLE;
  }
  if (dev < 0 && cudaGetDevice(&dev) != cudaSuccess) return MCB_STATUS_CANDIDATE_UNAVAILABLE;
  mcb_status s = mcb_candidate_available(dev);  // also creates the device context
  if (s != MCB_STATUS_OK) return s;
  mcb_plan *p = new (std::nothrow) mcb_plan;
  if (!p) return MCB_STATUS_ALLOCATION_FAILURE;
  p->desc = d;
  p->device = dev;
  p->generation = g_next_generation.fetch_add(1);
  int prev = -1;
  cudaGetDevice(&prev);
  if (prev != dev) cudaSetDevice(dev);
  cudaError_t e = cudaSuccess;
  p->workspace_bytes = workspace_for(d);
  if (p->workspace_bytes) e = cudaMalloc(&p->workspace, p->workspace_bytes);
  if (e == cudaSuccess && d.graph_mode) {
    e = cudaStreamCreateWithFlags(&p->stream, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&p->ev_in, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&p->ev_out, cudaEventDisableTiming);
  }
  if (prev >= 0 && prev != dev) cudaSetDevice(prev);
  if (e != cudaSuccess) {
    release(p);
    return e == cudaErrorMemoryAllocation ? MCB_STATUS_ALLOCATION_FAILURE
                                          : MCB_STATUS_CANDIDATE_FAILURE;
  }
  *out = p;
  return MCB_STATUS_OK;
}

MCB_API mcb_status mcb_plan_execute_v1(mcb_plan *p, const mcb_tensor *tensors,
                                       uint32_t num_tensors, void *stream_v) noexcept {
  if (!p || !tensors) return MCB_STATUS_INVALID_ARGUMENT;
  const uint32_t n = slots_for(p->desc);
  if (num_tensors != n) return MCB_STATUS_SHAPE_MISMATCH;
  for (uint32_t i = 0; i < n; ++i)
    if (!same_meta(tensors[i], p->desc.tensors[i])) return MCB_STATUS_SHAPE_MISMATCH;
  cudaStream_t caller = static_cast<cudaStream_t>(stream_v);
  if (!p->desc.graph_mode) return run_op(*p, tensors, caller);

  int prev = -1;
  cudaGetDevice(&prev);
  if (prev != p->device) cudaSetDevice(p->device);
  mcb_status result = MCB_STATUS_OK;
  if (!p->exec) {
    // Capture once on the plan's own stream (thread-local capture mode).
    if (cudaStreamBeginCapture(p->stream, cudaStreamCaptureModeThreadLocal) != cudaSuccess) {
      result = MCB_STATUS_CANDIDATE_FAILURE;
    } else {
      const mcb_status s = run_op(*p, tensors, p->stream);
      cudaGraph_t g = nullptr;
      const cudaError_t ce = cudaStreamEndCapture(p->stream, &g);
      if (s != MCB_STATUS_OK || ce != cudaSuccess) {
        if (g) cudaGraphDestroy(g);
        result = s != MCB_STATUS_OK ? s : MCB_STATUS_CANDIDATE_FAILURE;
      } else if (cudaGraphInstantiate(&p->exec, g, 0) != cudaSuccess) {
        cudaGraphDestroy(g);
        p->exec = nullptr;
        result = MCB_STATUS_CANDIDATE_FAILURE;
      } else {
        p->graph = g;
        for (uint32_t i = 0; i < n; ++i) p->captured[i] = tensors[i].data;
      }
    }
  } else {
    for (uint32_t i = 0; i < n; ++i)
      if (tensors[i].data != p->captured[i]) {
        result = MCB_STATUS_INVALID_ARGUMENT;  // replay cannot follow moved buffers
        break;
      }
  }
  if (result == MCB_STATUS_OK) {
    // Order the replay after the caller's prior work and the caller's later
    // work after the replay.
    cudaError_t e = cudaEventRecord(p->ev_in, caller);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(p->stream, p->ev_in, 0);
    if (e == cudaSuccess) e = cudaGraphLaunch(p->exec, p->stream);
    if (e == cudaSuccess) e = cudaEventRecord(p->ev_out, p->stream);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(caller, p->ev_out, 0);
    if (e != cudaSuccess) result = MCB_STATUS_CANDIDATE_FAILURE;
  }
  if (prev >= 0 && prev != p->device) cudaSetDevice(prev);
  return result;
}

MCB_API uint64_t mcb_plan_generation_v1(const mcb_plan *p) noexcept {
  return p ? p->generation : 0;
}

MCB_API mcb_status mcb_plan_destroy_v1(mcb_plan *p) noexcept {
  if (!p) return MCB_STATUS_INVALID_ARGUMENT;
  release(p);
  return MCB_STATUS_OK;
}

}  // extern "C"

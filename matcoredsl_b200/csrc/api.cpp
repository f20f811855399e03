// C-ABI implementation of include/mcb.h: argument validation, per-device
// context, staging of host-resident operands, dispatch to the kernels, and
// the ownership-tracked device-buffer registry.
//
// Nothing in this file computes results on the CPU: when no sm_100 GPU is
// usable every compute entry point returns MCB_STATUS_CANDIDATE_UNAVAILABLE.
#include "mcb.h"

#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <new>
#include <unordered_map>
#include <vector>

#include "internal.h"

namespace mcb {

// ---- tensor maps --------------------------------------------------------------
namespace {
PFN_cuTensorMapEncodeTiled_v12000 g_encode_tiled = nullptr;
std::once_flag g_encode_once;

PFN_cuTensorMapEncodeTiled_v12000 encoder() {
  std::call_once(g_encode_once, [] {
    void *fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000, cudaEnableDefault,
                                         &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode_tiled = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  return g_encode_tiled;
}
}  // namespace

bool encode_tmap_2d(CUtensorMap *map, CUtensorMapDataType dtype, const void *base,
                    uint64_t inner, uint64_t outer, uint64_t row_stride_bytes, uint32_t box_inner,
                    uint32_t box_outer, CUtensorMapSwizzle swizzle) {
  auto fn = encoder();
  if (!fn) return false;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  return fn(map, dtype, 2, const_cast<void *>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool encode_tmap_3d(CUtensorMap *map, CUtensorMapDataType dtype, const void *base, uint64_t d0,
                    uint64_t d1, uint64_t d2, uint64_t stride1_bytes, uint64_t stride2_bytes,
                    uint32_t box0, uint32_t box1, uint32_t box2, CUtensorMapSwizzle swizzle) {
  auto fn = encoder();
  if (!fn) return false;
  cuuint64_t dims[3] = {d0, d1, d2};
  cuuint64_t strides[2] = {stride1_bytes, stride2_bytes};
  cuuint32_t box[3] = {box0, box1, box2};
  cuuint32_t estr[3] = {1, 1, 1};
  return fn(map, dtype, 3, const_cast<void *>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// 4D bf16 map {d0 (innermost), d1, d2, d3} with byte strides s1..s3, box
// {64, 128, 1, 1} and 128-byte swizzle (the MSM Q/K/V tiles).
bool encode_tmap_4d_bf16(CUtensorMap *map, const void *base, uint64_t d0, uint64_t d1,
                         uint64_t d2, uint64_t d3, uint64_t s1, uint64_t s2, uint64_t s3) {
  auto fn = encoder();
  if (!fn) return false;
  cuuint64_t dims[4] = {d0, d1, d2, d3};
  cuuint64_t strides[3] = {s1, s2, s3};
  cuuint32_t box[4] = {64, 128, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void *>(base), dims, strides,
            box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace mcb

namespace {

using mcb::LaunchInfo;

constexpr int kMaxDevices = 64;
constexpr int kStageSlots = 8;
// Strict pairs with at least this many intermediate elements (M*N) run as two
// tiled GEMMs; smaller ones as one fused kernel (launch-bound either way).

// Lazily created per-device state: SM count, the device status word and the
// grow-only staging buffers used for host-resident operands.
struct DeviceCtx {
  std::mutex mu;
  bool ready = false;
  bool usable = false;  // an sm_100 part
  int sms = 0;
  int smem_optin = 0;
  uint32_t *status = nullptr;
  void *stage[kStageSlots] = {};
  size_t stage_cap[kStageSlots] = {};
  // Row pipeline for host operands: uploads and downloads run on their own
  // streams (separate copy engines, PCIe is full duplex) and are ordered
  // against the compute stream with events from this pool.
  cudaStream_t copy_in = nullptr, copy_out = nullptr;
  std::vector<cudaEvent_t> events;
  // Stream-ordered scratch (kernel intermediates of calls without a large
  // enough workspace): a pool owned by this library, so its retention setting
  // touches no other allocator in the process. Created on first use.
  std::once_flag pool_once;
  cudaMemPool_t pool = nullptr;
  // Stream-K workspace of the CTA-pair GEMM (created on first use): the
  // ready flags and partial slots are shared by every launch on the device, so
  // each stream-K launch is ordered after the previous one (sk_done).
  std::mutex sk_mu;
  bool sk_tried = false;
  mcb::GemmStreamK sk;
  cudaEvent_t sk_done = nullptr;
  cudaStream_t sk_stream = nullptr;
  bool sk_pending = false;
};
// Bytes the scratch pool keeps reserved across synchronisations, so repeated
// calls reuse mapped memory instead of mapping it again.
constexpr uint64_t kPoolKeepBytes = 4ull << 30;
DeviceCtx g_dev[kMaxDevices];

// ---- host runtime calls behind a replaceable table (fault injection) ------------
// mcb_test_set_runtime_hooks_v1 installs stand-ins for the CUDA runtime calls
// of the host path and for kernel launches, so that tests can fail any one of
// them on a machine without a GPU. With no table installed every rt_* helper
// is the CUDA runtime call itself.
mcb_runtime_hooks g_hook_table;
std::atomic<bool> g_hooks_on{false};
std::atomic<bool> g_real_context{false};  // a device context was created through CUDA
const mcb_runtime_hooks *hooks() {
  return g_hooks_on.load(std::memory_order_acquire) ? &g_hook_table : nullptr;
}

cudaError_t rt_get_device_count(int *n) {
  if (const auto *h = hooks()) {
    int32_t v = 0;
    const int32_t e = h->get_device_count(&v);
    *n = v;
    return static_cast<cudaError_t>(e);
  }
  return cudaGetDeviceCount(n);
}
cudaError_t rt_get_device(int *d) {
  if (const auto *h = hooks()) {
    int32_t v = 0;
    const int32_t e = h->get_device(&v);
    *d = v;
    return static_cast<cudaError_t>(e);
  }
  return cudaGetDevice(d);
}
cudaError_t rt_set_device(int d) {
  if (const auto *h = hooks()) return static_cast<cudaError_t>(h->set_device(d));
  return cudaSetDevice(d);
}
cudaError_t rt_malloc(void **p, size_t bytes) {
  if (const auto *h = hooks()) return static_cast<cudaError_t>(h->malloc_device(p, bytes));
  return cudaMalloc(p, bytes);
}
cudaError_t rt_free(void *p) {
  if (const auto *h = hooks()) return static_cast<cudaError_t>(h->free_device(p));
  return cudaFree(p);
}
cudaError_t rt_memset(void *p, int v, size_t bytes) {
  if (const auto *h = hooks()) return static_cast<cudaError_t>(h->memset_device(p, v, bytes));
  return cudaMemset(p, v, bytes);
}
cudaError_t rt_memcpy_async(void *d, const void *s, size_t bytes, cudaMemcpyKind kind,
                            cudaStream_t st) {
  if (const auto *h = hooks())
    return static_cast<cudaError_t>(h->memcpy_async(d, s, bytes, static_cast<int32_t>(kind), st));
  return cudaMemcpyAsync(d, s, bytes, kind, st);
}
cudaError_t rt_memcpy2d_async(void *d, size_t dp, const void *s, size_t sp, size_t w, size_t rows,
                              cudaMemcpyKind kind, cudaStream_t st) {
  if (const auto *h = hooks())
    return static_cast<cudaError_t>(
        h->memcpy2d_async(d, dp, s, sp, w, rows, static_cast<int32_t>(kind), st));
  return cudaMemcpy2DAsync(d, dp, s, sp, w, rows, kind, st);
}
cudaError_t rt_memcpy(void *d, const void *s, size_t bytes, cudaMemcpyKind kind) {
  if (const auto *h = hooks())
    return static_cast<cudaError_t>(h->memcpy_sync(d, s, bytes, static_cast<int32_t>(kind)));
  return cudaMemcpy(d, s, bytes, kind);
}
cudaError_t rt_stream_sync(cudaStream_t st) {
  if (const auto *h = hooks()) return static_cast<cudaError_t>(h->stream_synchronize(st));
  return cudaStreamSynchronize(st);
}

// Restores the caller's current device on scope exit.
struct DeviceGuard {
  int prev = -1;
  bool switched = false;
  bool ok = true;  // `dev` is current (false when the switch failed)
  explicit DeviceGuard(int dev) {
    if (rt_get_device(&prev) != cudaSuccess) {
      ok = false;  // the caller's device could not be restored afterwards
    } else if (prev != dev) {
      switched = rt_set_device(dev) == cudaSuccess;
      ok = switched;
    }
  }
  ~DeviceGuard() {
    if (switched) rt_set_device(prev);
  }
};

mcb_status init_ctx(int dev, DeviceCtx **out) {
  if (dev < 0 || dev >= kMaxDevices) return MCB_STATUS_INVALID_ARGUMENT;
  DeviceCtx &c = g_dev[dev];
  std::lock_guard<std::mutex> lock(c.mu);
  if (!c.ready) {
    int major = 0, minor = 0;
    if (const auto *h = hooks()) {
      int32_t mj = 0, mn = 0, sms = 0, smem = 0;
      if (h->device_info(dev, &mj, &mn, &sms, &smem) != 0) return MCB_STATUS_CANDIDATE_UNAVAILABLE;
      major = mj;
      minor = mn;
      c.sms = sms;
      c.smem_optin = smem;
    } else {
      cudaDeviceProp prop;
      if (cudaGetDeviceProperties(&prop, dev) != cudaSuccess) return MCB_STATUS_CANDIDATE_UNAVAILABLE;
      major = prop.major;
      minor = prop.minor;
      c.sms = prop.multiProcessorCount;
      c.smem_optin = static_cast<int>(prop.sharedMemPerBlockOptin);
    }
    c.usable = major == 10 && minor == 0 && c.sms > 0;
    if (c.usable) {
      DeviceGuard g(dev);
      if (!g.ok) return MCB_STATUS_CANDIDATE_FAILURE;
      if (!hooks()) g_real_context.store(true, std::memory_order_release);
      if (!c.status && rt_malloc(reinterpret_cast<void **>(&c.status), sizeof(uint32_t)) != cudaSuccess)
        return MCB_STATUS_ALLOCATION_FAILURE;
      if (rt_memset(c.status, 0, sizeof(uint32_t)) != cudaSuccess) return MCB_STATUS_CANDIDATE_FAILURE;
    }
    c.ready = true;
  }
  if (!c.usable) return MCB_STATUS_CANDIDATE_UNAVAILABLE;
  *out = &c;
  return MCB_STATUS_OK;
}

mcb_status resolve_device(const mcb_exec *exec, int *dev) {
  int count = 0;
  if (rt_get_device_count(&count) != cudaSuccess || count == 0) {
    if (!hooks()) cudaGetLastError();
    return MCB_STATUS_CANDIDATE_UNAVAILABLE;
  }
  int d = exec ? exec->device : -1;
  if (d < 0 && rt_get_device(&d) != cudaSuccess) return MCB_STATUS_CANDIDATE_UNAVAILABLE;
  if (d >= count) return MCB_STATUS_INVALID_ARGUMENT;
  *dev = d;
  return MCB_STATUS_OK;
}

size_t dtype_size(mcb_dtype t) {
  switch (t) {
    case MCB_DTYPE_F32: case MCB_DTYPE_I32: return 4;
    case MCB_DTYPE_F64: return 8;
    case MCB_DTYPE_BF16: case MCB_DTYPE_F16: return 2;
    case MCB_DTYPE_I8: case MCB_DTYPE_E4M3: case MCB_DTYPE_E5M2: return 1;
    default: return 0;
  }
}

// Structural checks common to every tensor argument.
mcb_status check_tensor(const mcb_tensor *t, uint32_t min_rank, uint32_t max_rank) {
  if (!t) return MCB_STATUS_INVALID_ARGUMENT;
  if (t->abi_version != MCB_ABI_VERSION_V1 || t->struct_size < sizeof(mcb_tensor))
    return MCB_STATUS_ABI_MISMATCH;
  if (t->rank < min_rank || t->rank > max_rank) return MCB_STATUS_UNSUPPORTED_RANK;
  if (dtype_size(t->dtype) == 0) return MCB_STATUS_UNSUPPORTED_DTYPE;
  if (t->memory_space != MCB_MEMORY_HOST && t->memory_space != MCB_MEMORY_CUDA_DEVICE)
    return MCB_STATUS_UNSUPPORTED_MEMORY_SPACE;
  int64_t elems = 1;
  for (uint32_t i = 0; i < t->rank; ++i) {
    if (t->dims[i] < 0) return MCB_STATUS_INVALID_SHAPE;
    if (t->dims[i] != 0 && elems > INT64_MAX / t->dims[i]) return MCB_STATUS_ARITHMETIC_OVERFLOW;
    elems *= t->dims[i];
  }
  if (elems > 0) {
    if (!t->data) return MCB_STATUS_INVALID_ARGUMENT;
    if (t->strides[t->rank - 1] != 1) return MCB_STATUS_UNSUPPORTED_LAYOUT;
    // Any positive strides describe a valid view (e.g. heads interleaved in
    // a packed QKV row). The element sets of different indices must not
    // collide: ordering the dimensions by stride, each stride must step over
    // the whole block spanned by the smaller ones. Extent-1 dims are free.
    int order[MCB_MAX_RANK];
    int nd = 0;
    for (uint32_t i = 0; i < t->rank; ++i) {
      if (t->dims[i] <= 1) continue;
      if (t->strides[i] <= 0) return MCB_STATUS_UNSUPPORTED_LAYOUT;
      order[nd++] = static_cast<int>(i);
    }
    std::sort(order, order + nd, [t](int x, int y) { return t->strides[x] < t->strides[y]; });
    int64_t block = 1;
    for (int j = 0; j < nd; ++j) {
      if (t->strides[order[j]] < block) return MCB_STATUS_UNSUPPORTED_LAYOUT;
      block = t->strides[order[j]] * t->dims[order[j]];
    }
    if (reinterpret_cast<uintptr_t>(t->data) % dtype_size(t->dtype) != 0)
      return MCB_STATUS_INVALID_ALIGNMENT;
  }
  return MCB_STATUS_OK;
}

int64_t numel(const mcb_tensor *t) {
  int64_t e = 1;
  for (uint32_t i = 0; i < t->rank; ++i) e *= t->dims[i];
  return e;
}

// Bytes spanned by a (possibly strided) tensor, from its base pointer.
uint64_t span_bytes(const mcb_tensor *t) {
  if (numel(t) == 0) return 0;
  int64_t last = 0;
  for (uint32_t i = 0; i < t->rank; ++i) last += (t->dims[i] - 1) * t->strides[i];
  return static_cast<uint64_t>(last + 1) * dtype_size(t->dtype);
}

bool overlaps(const mcb_tensor *a, const mcb_tensor *b) {
  if (!a || !b || numel(a) == 0 || numel(b) == 0) return false;
  const uintptr_t a0 = reinterpret_cast<uintptr_t>(a->data), a1 = a0 + span_bytes(a);
  const uintptr_t b0 = reinterpret_cast<uintptr_t>(b->data), b1 = b0 + span_bytes(b);
  return a0 < b1 && b0 < a1;
}

mcb_status check_exec(const mcb_exec *exec) {
  if (!exec) return MCB_STATUS_OK;
  if (exec->abi_version != MCB_ABI_VERSION_V1 || exec->struct_size < sizeof(mcb_exec))
    return MCB_STATUS_ABI_MISMATCH;
  if (exec->report && (exec->report->abi_version != MCB_ABI_VERSION_V1 ||
                       exec->report->struct_size < sizeof(mcb_report)))
    return MCB_STATUS_ABI_MISMATCH;
  return MCB_STATUS_OK;
}

mcb_status from_cuda(cudaError_t e) {
  if (e == cudaSuccess) return MCB_STATUS_OK;
  if (e == cudaErrorMemoryAllocation) return MCB_STATUS_ALLOCATION_FAILURE;
  if (e == cudaErrorNoDevice || e == cudaErrorInsufficientDriver ||
      e == cudaErrorNoKernelImageForDevice)
    return MCB_STATUS_CANDIDATE_UNAVAILABLE;
  return MCB_STATUS_CANDIDATE_FAILURE;
}

// One call: resolves the device, owns the staging of host operands and the
// optional timing, and finishes with the synchronisation/status checks.
class Call {
 public:
  // `hookable`: the operator runs under installed runtime hooks (its kernel
  // launches go through launch_or_hook); others refuse while hooks are on.
  explicit Call(const mcb_exec *exec, bool hookable = false)
      : exec_(exec), hookable_(hookable) {}
  ~Call() {
    release_pooled();
    for (auto &e : events_)
      if (e) cudaEventDestroy(e);
    if (lock_.owns_lock()) lock_.unlock();
    delete guard_;
  }

  mcb_status begin(bool host_operands) {
    mcb_status s = check_exec(exec_);
    if (s) return s;
    if (hooks() && !hookable_) return MCB_STATUS_CANDIDATE_UNAVAILABLE;
    s = resolve_device(exec_, &dev_);
    if (s) return s;
    guard_ = new (std::nothrow) DeviceGuard(dev_);
    if (!guard_) return MCB_STATUS_ALLOCATION_FAILURE;
    if (!guard_->ok) return MCB_STATUS_CANDIDATE_FAILURE;
    s = init_ctx(dev_, &ctx_);
    if (s) return s;
    stream_ = exec_ ? static_cast<cudaStream_t>(exec_->stream) : nullptr;
    host_ = host_operands;
    timed_ = exec_ && (exec_->flags & MCB_EXEC_TIME) && !hooks();
    sync_ = host_ || timed_ || (exec_ && (exec_->flags & MCB_EXEC_SYNC));
    if (host_) lock_ = std::unique_lock<std::mutex>(ctx_->mu);  // staging slots are per device
    if (timed_) {
      for (auto &e : events_)
        if (cudaEventCreate(&e) != cudaSuccess) return MCB_STATUS_CANDIDATE_FAILURE;
      cudaEventRecord(events_[0], stream_);
    }
    return MCB_STATUS_OK;
  }

  // Device pointer for an operand: itself when device-resident, else a
  // staging buffer (uploaded when `upload`).
  mcb_status device_ptr(const mcb_tensor *t, bool upload, void **out) {
    if (!t || numel(t) == 0) {
      *out = t ? t->data : nullptr;
      return MCB_STATUS_OK;
    }
    if (t->memory_space == MCB_MEMORY_CUDA_DEVICE) {
      *out = t->data;
      return MCB_STATUS_OK;
    }
    if (slot_ >= kStageSlots) return MCB_STATUS_INSUFFICIENT_WORKSPACE;
    const size_t bytes = span_bytes(t);
    const int s = slot_++;
    if (ctx_->stage_cap[s] < bytes) {
      if (ctx_->stage[s]) {
        // The old buffer may still be read by queued work: a failed wait
        // leaves it allocated (not freed under a running kernel).
        if (rt_stream_sync(stream_) != cudaSuccess) return MCB_STATUS_CANDIDATE_FAILURE;
        rt_free(ctx_->stage[s]);
        ctx_->stage[s] = nullptr;
        ctx_->stage_cap[s] = 0;
      }
      const size_t cap = std::max<size_t>(bytes, 1 << 20);
      if (rt_malloc(&ctx_->stage[s], cap) != cudaSuccess) {
        ctx_->stage[s] = nullptr;
        return MCB_STATUS_ALLOCATION_FAILURE;
      }
      ctx_->stage_cap[s] = cap;
    }
    *out = ctx_->stage[s];
    if (upload) {
      if (rt_memcpy_async(*out, t->data, bytes, cudaMemcpyHostToDevice, stream_) != cudaSuccess)
        return MCB_STATUS_CANDIDATE_FAILURE;
      h2d_bytes_ += bytes;
    }
    return MCB_STATUS_OK;
  }

  // Device scratch that keeps the call asynchronous: the caller's workspace
  // when it holds `bytes` at a 16-byte aligned base, else a stream-ordered
  // allocation from the library's pool on this device, released on the
  // call's stream when the call finishes. False when neither is available.
  bool stream_scratch(uint64_t bytes, void **out) {
    if (exec_ && exec_->workspace && exec_->workspace_bytes >= bytes &&
        (reinterpret_cast<uintptr_t>(exec_->workspace) & 15u) == 0) {
      *out = exec_->workspace;
      return true;
    }
    if (n_pooled_ == kMaxPooled || hooks()) return false;
    std::call_once(ctx_->pool_once, [this] {
      cudaMemPoolProps props = {};
      props.allocType = cudaMemAllocationTypePinned;
      props.handleTypes = cudaMemHandleTypeNone;
      props.location.type = cudaMemLocationTypeDevice;
      props.location.id = dev_;
      cudaMemPool_t pool = nullptr;
      if (cudaMemPoolCreate(&pool, &props) != cudaSuccess) {
        (void)cudaGetLastError();
        return;
      }
      uint64_t keep = kPoolKeepBytes;
      (void)cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &keep);
      ctx_->pool = pool;
    });
    if (!ctx_->pool) return false;
    void *p = nullptr;
    if (cudaMallocFromPoolAsync(&p, bytes ? bytes : 1, ctx_->pool, stream_) != cudaSuccess) {
      (void)cudaGetLastError();
      return false;
    }
    pooled_[n_pooled_++] = p;
    *out = p;
    return true;
  }

  // Device scratch for a kernel: stream_scratch when it succeeds, else a
  // staging slot. A staging slot is shared by later calls on this device, so
  // using one forces this call to synchronise before return.
  mcb_status scratch(uint64_t bytes, void **out) {
    if (stream_scratch(bytes, out)) return MCB_STATUS_OK;
    if (!lock_.owns_lock()) lock_ = std::unique_lock<std::mutex>(ctx_->mu);
    sync_ = true;
    mcb_tensor tmp{};
    tmp.abi_version = MCB_ABI_VERSION_V1;
    tmp.struct_size = sizeof(mcb_tensor);
    tmp.data = reinterpret_cast<void *>(16);
    tmp.dtype = MCB_DTYPE_I8;
    tmp.rank = 1;
    tmp.dims[0] = static_cast<int64_t>(bytes);
    tmp.strides[0] = 1;
    tmp.memory_space = MCB_MEMORY_HOST;
    return device_ptr(&tmp, false, out);
  }

  void mark_compute_start() {
    if (timed_) cudaEventRecord(events_[1], stream_);
  }
  void mark_compute_end() {
    if (timed_) cudaEventRecord(events_[2], stream_);
  }

  // Copies a staged output back, synchronises and checks the status word.
  mcb_status finish(const mcb_tensor *out, void *dev_out, const LaunchInfo &info,
                    cudaError_t launch_err) {
    if (launch_err != cudaSuccess) return from_cuda(launch_err);
    if (out && host_ && numel(out) > 0 && !output_staged_) {
      if (out->rank == 2) {
        if (copy_rows(out->data, dev_out, out, 0, out->dims[0], cudaMemcpyDeviceToHost,
                      stream_) != cudaSuccess)
          return MCB_STATUS_CANDIDATE_FAILURE;
        d2h_bytes_ += row_bytes(out, 0, out->dims[0]);
      } else {
        const size_t bytes = span_bytes(out);
        if (rt_memcpy_async(out->data, dev_out, bytes, cudaMemcpyDeviceToHost, stream_) !=
            cudaSuccess)
          return MCB_STATUS_CANDIDATE_FAILURE;
        d2h_bytes_ += bytes;
      }
    }
    if (timed_) cudaEventRecord(events_[3], stream_);
    if (release_pooled() != cudaSuccess) return MCB_STATUS_CANDIDATE_FAILURE;
    uint32_t word = 0;
    if (sync_) {
      cudaError_t e = rt_stream_sync(stream_);
      if (e != cudaSuccess) return from_cuda(e);
      if (rt_memcpy(&word, ctx_->status, sizeof(word), cudaMemcpyDeviceToHost) != cudaSuccess)
        return MCB_STATUS_CANDIDATE_FAILURE;
    }
    if (exec_ && exec_->report) {
      mcb_report *r = exec_->report;
      std::memcpy(r->route, info.route, sizeof(r->route));
      r->kernel_launches = info.launches;
      r->tile_m = info.tile_m;
      r->tile_n = info.tile_n;
      r->tile_k = info.tile_k;
      r->stages = info.stages;
      r->ctas = info.ctas;
      r->h2d_bytes = h2d_bytes_;
      r->d2h_bytes = d2h_bytes_;
      r->device_status = word;
      r->route_flags = info.stream_k ? MCB_ROUTE_STREAM_K : 0u;
      r->kernel_ms = r->h2d_ms = r->d2h_ms = 0.0f;
      if (timed_) {
        cudaEventElapsedTime(&r->h2d_ms, events_[0], events_[1]);
        cudaEventElapsedTime(&r->kernel_ms, events_[1], events_[2]);
        cudaEventElapsedTime(&r->d2h_ms, events_[2], events_[3]);
      }
    }
    if (word != 0) return MCB_STATUS_DEVICE_TIMEOUT;
    return MCB_STATUS_OK;
  }

  // Row pipeline for a row-splittable operator whose operands are in host
  // memory: rows [0, m) are processed in chunks of `chunk_rows`. For each
  // chunk the rows of every `row_inputs` tensor are uploaded on the copy-in
  // stream, `launch(r0, r1)` runs on the call's stream once they have landed,
  // and the chunk's rows of `out` are downloaded on the copy-out stream, so the
  // upload of chunk c+1, the kernels of chunk c and the download of chunk c-1
  // overlap. Row-chunked tensors are rank 2 with unit column stride; their
  // staging buffers (`dev`) have the host tensor's strides. Only the output's
  // own columns are written back (host padding between rows is left alone).
  struct RowOperand {
    const mcb_tensor *t;
    void *dev;
  };
  // `whole_inputs` (operands every chunk reads in full, e.g. the weights) are
  // uploaded first on the copy-in stream, so they arrive at full PCIe
  // bandwidth and the first chunk's kernels and download start early.
  template <typename Launch>
  mcb_status run_row_pipeline(int64_t m, int64_t chunk_rows, const RowOperand *whole_inputs,
                              int n_whole, const RowOperand *row_inputs, int n_inputs,
                              RowOperand out, Launch &&launch, cudaError_t *launch_err) {
    *launch_err = cudaSuccess;
    const int64_t nchunks = (m + chunk_rows - 1) / chunk_rows;
    mcb_status s = pipeline_resources(static_cast<int>(2 * nchunks + 2));
    if (s) return s;
    cudaEvent_t *ev = ctx_->events.data();
    cudaStream_t cin = ctx_->copy_in, cout = ctx_->copy_out;
    // Uploads start after the caller's earlier work on its stream.
    if (cudaEventRecord(ev[0], stream_) != cudaSuccess ||
        cudaStreamWaitEvent(cin, ev[0], 0) != cudaSuccess)
      return MCB_STATUS_CANDIDATE_FAILURE;
    s = MCB_STATUS_OK;
    for (int i = 0; i < n_whole && !s; ++i) {
      const mcb_tensor *t = whole_inputs[i].t;
      if (!t || numel(t) == 0) continue;
      const uint64_t bytes = span_bytes(t);
      if (cudaMemcpyAsync(whole_inputs[i].dev, t->data, bytes, cudaMemcpyHostToDevice, cin) !=
          cudaSuccess)
        s = MCB_STATUS_CANDIDATE_FAILURE;
      else
        h2d_bytes_ += bytes;
    }
    for (int64_t c = 0; c < nchunks && !s; ++c) {
      const int64_t r0 = c * chunk_rows, r1 = std::min(m, r0 + chunk_rows);
      cudaEvent_t in_done = ev[2 + 2 * c], out_ready = ev[3 + 2 * c];
      for (int i = 0; i < n_inputs && !s; ++i) {
        if (copy_rows(row_inputs[i].dev, row_inputs[i].t->data, row_inputs[i].t, r0, r1,
                      cudaMemcpyHostToDevice, cin) != cudaSuccess)
          s = MCB_STATUS_CANDIDATE_FAILURE;
        else
          h2d_bytes_ += row_bytes(row_inputs[i].t, r0, r1);
      }
      if (s) break;
      if (cudaEventRecord(in_done, cin) != cudaSuccess ||
          cudaStreamWaitEvent(stream_, in_done, 0) != cudaSuccess) {
        s = MCB_STATUS_CANDIDATE_FAILURE;
        break;
      }
      *launch_err = launch(r0, r1);
      if (*launch_err != cudaSuccess) break;
      if (cudaEventRecord(out_ready, stream_) != cudaSuccess ||
          cudaStreamWaitEvent(cout, out_ready, 0) != cudaSuccess ||
          copy_rows(out.t->data, out.dev, out.t, r0, r1, cudaMemcpyDeviceToHost, cout) !=
              cudaSuccess) {
        s = MCB_STATUS_CANDIDATE_FAILURE;
        break;
      }
      d2h_bytes_ += row_bytes(out.t, r0, r1);
    }
    // The call's stream (synchronised by finish) waits for the last download;
    // on any failure every stream is drained before the staging slots can be
    // reused.
    if (cudaEventRecord(ev[1], cout) != cudaSuccess ||
        cudaStreamWaitEvent(stream_, ev[1], 0) != cudaSuccess)
      s = s ? s : MCB_STATUS_CANDIDATE_FAILURE;
    if (s || *launch_err != cudaSuccess) {
      cudaStreamSynchronize(cin);
      cudaStreamSynchronize(cout);
      cudaStreamSynchronize(stream_);
    }
    output_staged_ = true;
    return s;
  }

  bool host_operands() const { return host_; }
  bool timed() const { return timed_; }
  DeviceCtx *ctx() const { return ctx_; }
  cudaStream_t stream() const { return stream_; }
  int sms() const { return ctx_->sms; }
  const mcb_exec *exec() const { return exec_; }

  // Runs `launch(sk)` with the device's stream-K workspace (nullptr when it
  // cannot be used: runtime hooks installed, the stream is being captured,
  // or the workspace could not be created), ordered after the previous
  // stream-K launch on this device when that was on another stream.
  // `launch` reports through `info->stream_k` whether it used the workspace.
  template <typename Launch>
  cudaError_t with_stream_k(LaunchInfo *info, Launch &&launch) {
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    if (hooks() || cudaStreamIsCapturing(stream_, &cs) != cudaSuccess ||
        cs != cudaStreamCaptureStatusNone) {
      (void)cudaGetLastError();
      return launch(static_cast<const mcb::GemmStreamK *>(nullptr));
    }
    std::lock_guard<std::mutex> lock(ctx_->sk_mu);
    if (!ctx_->sk_tried) {
      ctx_->sk_tried = true;
      mcb::GemmStreamK w;
      w.clusters = std::max(1, ctx_->sms / 2);
      w.max_tiles = 2 * w.clusters;
      // One tail partial per CTA: two 128x256 f32 slots per cluster.
      const size_t part_bytes = static_cast<size_t>(w.clusters) * 2 *
                                static_cast<size_t>(mcb::kGemmStreamKSlotFloats) * sizeof(float);
      const size_t flag_bytes = static_cast<size_t>(w.max_tiles) * 2 * sizeof(int);
      if (cudaMalloc(reinterpret_cast<void **>(&w.part), part_bytes) == cudaSuccess &&
          cudaMalloc(reinterpret_cast<void **>(&w.flags), flag_bytes) == cudaSuccess &&
          cudaMemset(w.flags, 0, flag_bytes) == cudaSuccess &&
          cudaEventCreateWithFlags(&ctx_->sk_done, cudaEventDisableTiming) == cudaSuccess) {
        ctx_->sk = w;
      } else {
        (void)cudaGetLastError();
        if (w.part) cudaFree(w.part);
        if (w.flags) cudaFree(w.flags);
      }
    }
    if (!ctx_->sk.flags) return launch(static_cast<const mcb::GemmStreamK *>(nullptr));
    if (ctx_->sk_pending && ctx_->sk_stream != stream_ &&
        cudaStreamWaitEvent(stream_, ctx_->sk_done, 0) != cudaSuccess)
      return cudaErrorUnknown;
    const cudaError_t err = launch(static_cast<const mcb::GemmStreamK *>(&ctx_->sk));
    if (err == cudaSuccess && info->stream_k) {
      if (cudaEventRecord(ctx_->sk_done, stream_) != cudaSuccess) return cudaErrorUnknown;
      ctx_->sk_stream = stream_;
      ctx_->sk_pending = true;
    }
    return err;
  }

  // A kernel launch, or under installed runtime hooks the hook standing in
  // for it (`desc` says what the launch would compute).
  template <typename Launch>
  cudaError_t launch_or_hook(const mcb_hook_launch &desc, Launch &&launch) {
    if (const auto *h = hooks()) return static_cast<cudaError_t>(h->launch(&desc));
    return launch();
  }

 private:
  // Returns this call's pool allocations to the pool, in stream order after
  // everything the call enqueued.
  cudaError_t release_pooled() {
    cudaError_t err = cudaSuccess;
    for (int i = 0; i < n_pooled_; ++i) {
      const cudaError_t e = cudaFreeAsync(pooled_[i], stream_);
      if (err == cudaSuccess) err = e;
    }
    n_pooled_ = 0;
    return err;
  }
  // Bytes of rows [r0, r1) of a rank-2 tensor, its own columns only.
  static uint64_t row_bytes(const mcb_tensor *t, int64_t r0, int64_t r1) {
    return static_cast<uint64_t>(r1 - r0) * static_cast<uint64_t>(t->dims[1]) *
           dtype_size(t->dtype);
  }
  // Copies rows [r0, r1) of a rank-2 tensor between host memory and its
  // staging buffer (same strides on both sides): one linear copy when the
  // rows are packed, else a pitched copy of the tensor's own columns.
  static cudaError_t copy_rows(void *dst, const void *src, const mcb_tensor *t, int64_t r0,
                               int64_t r1, cudaMemcpyKind kind, cudaStream_t stream) {
    const size_t es = dtype_size(t->dtype);
    const size_t pitch = static_cast<size_t>(t->strides[0]) * es;
    const size_t width = static_cast<size_t>(t->dims[1]) * es;
    const size_t off = static_cast<size_t>(r0) * pitch;
    const size_t rows = static_cast<size_t>(r1 - r0);
    if (rows == 0 || width == 0) return cudaSuccess;
    char *d = static_cast<char *>(dst) + off;
    const char *s = static_cast<const char *>(src) + off;
    if (pitch == width || rows == 1) return rt_memcpy_async(d, s, rows * width, kind, stream);
    return rt_memcpy2d_async(d, pitch, s, pitch, width, rows, kind, stream);
  }
  // Copy streams and at least `n` events of the device's row pipeline
  // (created once; the device mutex is held for host-operand calls).
  mcb_status pipeline_resources(int n) {
    if (!ctx_->copy_in &&
        cudaStreamCreateWithFlags(&ctx_->copy_in, cudaStreamNonBlocking) != cudaSuccess)
      return MCB_STATUS_CANDIDATE_FAILURE;
    if (!ctx_->copy_out &&
        cudaStreamCreateWithFlags(&ctx_->copy_out, cudaStreamNonBlocking) != cudaSuccess)
      return MCB_STATUS_CANDIDATE_FAILURE;
    while (static_cast<int>(ctx_->events.size()) < n) {
      cudaEvent_t e;
      if (cudaEventCreateWithFlags(&e, cudaEventDisableTiming) != cudaSuccess)
        return MCB_STATUS_CANDIDATE_FAILURE;
      ctx_->events.push_back(e);
    }
    return MCB_STATUS_OK;
  }

  const mcb_exec *exec_;
  bool hookable_ = false;
  bool output_staged_ = false;
  int dev_ = -1;
  DeviceGuard *guard_ = nullptr;
  DeviceCtx *ctx_ = nullptr;
  cudaStream_t stream_ = nullptr;
  bool host_ = false, timed_ = false, sync_ = false;
  std::unique_lock<std::mutex> lock_;
  cudaEvent_t events_[4] = {};
  int slot_ = 0;
  static constexpr int kMaxPooled = 4;
  void *pooled_[kMaxPooled] = {};
  int n_pooled_ = 0;
  uint64_t h2d_bytes_ = 0, d2h_bytes_ = 0;
};

// All operands of one call must share one memory space.
mcb_status same_space(std::initializer_list<const mcb_tensor *> ts, bool *host) {
  int space = 0;
  for (const mcb_tensor *t : ts) {
    if (!t) continue;
    if (space == 0) space = static_cast<int>(t->memory_space);
    else if (space != static_cast<int>(t->memory_space)) return MCB_STATUS_MIXED_MEMORY_SPACES;
  }
  *host = space == MCB_MEMORY_HOST;
  return MCB_STATUS_OK;
}

mcb_status guarded(mcb_status (*fn)(void *), void *arg) noexcept {
  try {
    return fn(arg);
  } catch (const std::bad_alloc &) {
    return MCB_STATUS_ALLOCATION_FAILURE;
  } catch (...) {
    return MCB_STATUS_CANDIDATE_FAILURE;
  }
}

// ---- strict ---------------------------------------------------------------------
mcb_status strict_gemm_impl(const mcb_tensor *c, const mcb_tensor *a, const mcb_tensor *b,
                            const mcb_exec *exec) {
  mcb_status s;
  if ((s = check_tensor(a, 2, 2)) || (s = check_tensor(b, 2, 2)) || (s = check_tensor(c, 2, 2)))
    return s;
  if (a->dtype != MCB_DTYPE_F32 || b->dtype != MCB_DTYPE_F32 || c->dtype != MCB_DTYPE_F32)
    return MCB_STATUS_UNSUPPORTED_DTYPE;
  const int64_t m = a->dims[0], k = a->dims[1], n = b->dims[1];
  if (b->dims[0] != k || c->dims[0] != m || c->dims[1] != n) return MCB_STATUS_SHAPE_MISMATCH;
  if (overlaps(c, a) || overlaps(c, b)) return MCB_STATUS_ALIAS_VIOLATION;
  bool host = false;
  if ((s = same_space({a, b, c}, &host))) return s;
  Call call(exec, /*hookable=*/true);
  if ((s = call.begin(host))) return s;
  void *da, *db, *dc;
  if ((s = call.device_ptr(a, true, &da)) || (s = call.device_ptr(b, true, &db)) ||
      (s = call.device_ptr(c, false, &dc)))
    return s;
  LaunchInfo info;
  call.mark_compute_start();
  mcb_hook_launch desc{"strict_gemm", {da, db, nullptr}, dc, nullptr, m, k, n, 0,
                       {a->strides[0], b->strides[0], 0, c->strides[0]}};
  cudaError_t e = call.launch_or_hook(desc, [&] {
    return mcb::launch_strict_gemm(static_cast<const float *>(da), static_cast<const float *>(db),
                                   static_cast<float *>(dc), m, k, n, a->strides[0],
                                   b->strides[0], c->strides[0], call.sms(), call.stream(), &info);
  });
  call.mark_compute_end();
  return call.finish(c, dc, info, e);
}

mcb_status strict_pair_impl(const mcb_tensor *e, const mcb_tensor *a, const mcb_tensor *b,
                            const mcb_tensor *d, const mcb_exec *exec) {
  mcb_status s;
  if ((s = check_tensor(a, 2, 2)) || (s = check_tensor(b, 2, 2)) || (s = check_tensor(d, 2, 2)) ||
      (s = check_tensor(e, 2, 2)))
    return s;
  if (a->dtype != MCB_DTYPE_F32 || b->dtype != MCB_DTYPE_F32 || d->dtype != MCB_DTYPE_F32 ||
      e->dtype != MCB_DTYPE_F32)
    return MCB_STATUS_UNSUPPORTED_DTYPE;
  const int64_t m = a->dims[0], k = a->dims[1], n = b->dims[1], p = d->dims[1];
  if (b->dims[0] != k || d->dims[0] != n || e->dims[0] != m || e->dims[1] != p)
    return MCB_STATUS_SHAPE_MISMATCH;
  if (overlaps(e, a) || overlaps(e, b) || overlaps(e, d)) return MCB_STATUS_ALIAS_VIOLATION;
  bool host = false;
  if ((s = same_space({a, b, d, e}, &host))) return s;
  Call call(exec, /*hookable=*/true);
  if ((s = call.begin(host))) return s;
  void *da, *db, *dd, *de;
  if ((s = call.device_ptr(a, true, &da)) || (s = call.device_ptr(b, true, &db)) ||
      (s = call.device_ptr(d, true, &dd)) || (s = call.device_ptr(e, false, &de)))
    return s;
  // Two tiled strict GEMMs through a binary32 C [M,N] in device memory: the
  // caller's workspace when it holds C, else a stream-ordered allocation, so
  // the call stays asynchronous. Small problems, and any allocation failure,
  // take the single fused kernel below.
  if (m > 0 && n > 0 && p > 0 && m * n >= mcb::kStrictTwoPassMinElems) {
    const uint64_t cbytes = static_cast<uint64_t>(m) * static_cast<uint64_t>(n) * 4;
    void *cbuf = nullptr;
    if (call.stream_scratch(cbytes, &cbuf)) {
      LaunchInfo info;
      call.mark_compute_start();
      mcb_hook_launch desc{"strict_fused_pair", {da, db, dd}, de, cbuf, m, k, n, p,
                           {k ? a->strides[0] : 0, b->strides[0], d->strides[0], e->strides[0]}};
      cudaError_t err = call.launch_or_hook(desc, [&] {
        return mcb::launch_strict_pair_two_pass(
            static_cast<const float *>(da), static_cast<const float *>(db),
            static_cast<const float *>(dd), static_cast<float *>(de), static_cast<float *>(cbuf),
            m, k, n, p, k ? a->strides[0] : 0, b->strides[0], d->strides[0], e->strides[0],
            call.sms(), call.stream(), &info);
      });
      call.mark_compute_end();
      return call.finish(e, de, info, err);
    }
  }
  // The intermediate panel lives in shared memory when it fits; otherwise it
  // needs scratch, taken from the caller's workspace or a staging slot.
  const int smem_limit = call.ctx()->smem_optin;
  const int64_t scratch_floats = mcb::strict_pair_scratch_floats(m, n, call.sms(), smem_limit);
  void *scratch = nullptr;
  if (scratch_floats > 0 &&
      (s = call.scratch(static_cast<uint64_t>(scratch_floats) * 4, &scratch)))
    return s;
  LaunchInfo info;
  call.mark_compute_start();
  mcb_hook_launch desc{"strict_fused_pair", {da, db, dd}, de, scratch, m, k, n, p,
                       {k ? a->strides[0] : 0, n ? b->strides[0] : 0, p ? d->strides[0] : 0,
                        e->strides[0]}};
  cudaError_t err = call.launch_or_hook(desc, [&] {
    return mcb::launch_strict_pair(
        static_cast<const float *>(da), static_cast<const float *>(db),
        static_cast<const float *>(dd), static_cast<float *>(de), static_cast<float *>(scratch), m,
        k, n, p, k ? a->strides[0] : 0, n ? b->strides[0] : 0, p ? d->strides[0] : 0,
        e->strides[0], call.sms(), smem_limit, call.stream(), &info);
  });
  call.mark_compute_end();
  return call.finish(e, de, info, err);
}

// ---- Family A -------------------------------------------------------------------------
// Row-chunk size for the host-operand pipeline of a row-splittable operator:
// a multiple of 256 rows holding about 8 MiB of the row operand `x`, at most
// 64 chunks; 0 (no pipeline) when `m` gives fewer than two chunks.
int64_t pipeline_chunk_rows(int64_t m, const mcb_tensor *x) {
  constexpr int64_t kChunkBytes = 8 << 20, kAlign = 256, kMaxChunks = 64;
  const int64_t row_bytes = std::max<int64_t>(1, x->strides[0]) *
                            static_cast<int64_t>(dtype_size(x->dtype));
  int64_t rows = (kChunkBytes / row_bytes + kAlign - 1) / kAlign * kAlign;
  rows = std::max(rows, kAlign);
  const int64_t min_rows = ((m + kMaxChunks - 1) / kMaxChunks + kAlign - 1) / kAlign * kAlign;
  rows = std::max(rows, min_rows);
  return m >= 2 * rows ? rows : 0;
}

// `ops` (num_ops > 0): the general epilogue chain of mcb_gemm_epilogue_chain_v1
// instead of bias + activation; `bnds` are its [M,N] boundary tensors.
mcb_status gemm_epilogue_impl(const mcb_tensor *y, const mcb_tensor *x, const mcb_tensor *w,
                              const mcb_tensor *bias, const mcb_epilogue *epi,
                              uint32_t gemm_flags, const mcb_exec *exec,
                              const mcb_tensor *bnds = nullptr, uint32_t num_bnds = 0,
                              const mcb_epilogue_op *ops = nullptr, uint32_t num_ops = 0) {
  mcb_status s;
  if ((s = check_tensor(x, 2, 2)) || (s = check_tensor(w, 2, 2)) || (s = check_tensor(y, 2, 2)))
    return s;
  mcb::Epilogue ep;
  if (epi) {
    if (epi->abi_version != MCB_ABI_VERSION_V1 || epi->struct_size < sizeof(mcb_epilogue))
      return MCB_STATUS_ABI_MISMATCH;
    if (epi->bias_mode > MCB_BIAS_FULL || epi->bias_op > MCB_BIAS_RSUB ||
        epi->activation > MCB_ACT_TANH)
      return MCB_STATUS_INVALID_ARGUMENT;
    ep.bias_mode = static_cast<int>(epi->bias_mode);
    ep.bias_op = static_cast<int>(epi->bias_op);
    ep.act = static_cast<int>(epi->activation);
  }
  const bool wt = (gemm_flags & MCB_GEMM_W_TRANSPOSED) != 0;
  const int64_t m = x->dims[0], k = x->dims[1];
  const int64_t n = wt ? w->dims[0] : w->dims[1];
  if ((wt ? w->dims[1] : w->dims[0]) != k || y->dims[0] != m || y->dims[1] != n)
    return MCB_STATUS_SHAPE_MISMATCH;
  // X and W: both bf16, both f16 or both f32 (the reference's matmul
  // signatures, src/mlir_engine.cpp:114-152); Y f32 or the inputs' 16-bit
  // type; a bias f32 or 16-bit.
  const bool in_bf16 = x->dtype == MCB_DTYPE_BF16 && w->dtype == MCB_DTYPE_BF16;
  const bool in_f16 = x->dtype == MCB_DTYPE_F16 && w->dtype == MCB_DTYPE_F16;
  const bool in_f32 = x->dtype == MCB_DTYPE_F32 && w->dtype == MCB_DTYPE_F32;
  if (!in_bf16 && !in_f16 && !in_f32) return MCB_STATUS_UNSUPPORTED_DTYPE;
  if (y->dtype != MCB_DTYPE_F32 && y->dtype != (in_f16 ? MCB_DTYPE_F16 : MCB_DTYPE_BF16))
    return MCB_STATUS_UNSUPPORTED_DTYPE;
  if (ep.bias_mode != MCB_BIAS_NONE) {
    if ((s = check_tensor(bias, 1, 2))) return s;
    if (bias->dtype != MCB_DTYPE_BF16 && bias->dtype != MCB_DTYPE_F32 &&
        bias->dtype != MCB_DTYPE_F16)
      return MCB_STATUS_UNSUPPORTED_DTYPE;
    if (ep.bias_mode == MCB_BIAS_ROW &&
        !(numel(bias) == n && (bias->rank == 1 || bias->dims[0] == 1)))
      return MCB_STATUS_SHAPE_MISMATCH;
    if (ep.bias_mode == MCB_BIAS_FULL &&
        !(bias->rank == 2 && bias->dims[0] == m && bias->dims[1] == n))
      return MCB_STATUS_SHAPE_MISMATCH;
    ep.bias_bf16 = bias->dtype == MCB_DTYPE_BF16;
    ep.bias_f16 = bias->dtype == MCB_DTYPE_F16;
    ep.ld_bias = bias->rank == 2 ? bias->strides[0] : n;
  }
  // General chain: validate the ops and boundaries (exact [M,N] tensors, as
  // src/fusion_emitter_family_a.cpp:186-200 requires).
  const mcb_tensor *bt[mcb::kMaxEpiBoundaries] = {};
  if (num_ops > 0) {
    if (!ops || num_ops > mcb::kMaxEpiOps || num_bnds > mcb::kMaxEpiBoundaries ||
        (num_bnds > 0 && !bnds) || ep.bias_mode != MCB_BIAS_NONE || ep.act != MCB_ACT_NONE)
      return MCB_STATUS_INVALID_ARGUMENT;
    for (uint32_t i = 0; i < num_bnds; ++i) {
      const mcb_tensor *b = &bnds[i];
      if ((s = check_tensor(b, 2, 2))) return s;
      if (b->dtype != MCB_DTYPE_F32 && b->dtype != MCB_DTYPE_BF16 && b->dtype != MCB_DTYPE_F16)
        return MCB_STATUS_UNSUPPORTED_DTYPE;
      if (b->dims[0] != m || b->dims[1] != n) return MCB_STATUS_SHAPE_MISMATCH;
      if (overlaps(y, b)) return MCB_STATUS_ALIAS_VIOLATION;
      bt[i] = b;
      ep.bnd_dt[i] = static_cast<uint8_t>(b->dtype);
      ep.ld_bnd[i] = b->strides[0];
    }
    for (uint32_t o = 0; o < num_ops; ++o) {
      const uint32_t kind = ops[o].kind;
      const bool unary = kind >= MCB_EW_RELU && kind <= MCB_EW_GELU_TANH;
      const bool binary = kind >= MCB_EW_ADD && kind <= MCB_EW_MAX;
      if (!unary && !binary) return MCB_STATUS_INVALID_ARGUMENT;
      if (binary && (ops[o].boundary >= num_bnds || ops[o].value_pos > 1))
        return MCB_STATUS_INVALID_ARGUMENT;
      ep.op_kind[o] = static_cast<uint8_t>(kind);
      ep.op_pos[o] = static_cast<uint8_t>(binary ? ops[o].value_pos : 0);
      ep.op_bnd[o] = static_cast<uint8_t>(binary ? ops[o].boundary : 0);
    }
    ep.n_ops = static_cast<int>(num_ops);
  }
  if (overlaps(y, x) || overlaps(y, w) || (ep.bias_mode && overlaps(y, bias)))
    return MCB_STATUS_ALIAS_VIOLATION;
  bool host = false;
  if ((s = same_space({x, w, y, ep.bias_mode ? bias : nullptr, bt[0], bt[1], bt[2], bt[3]},
                      &host)))
    return s;
  Call call(exec);
  if ((s = call.begin(host))) return s;
  // Host operands (untimed calls): X, a full bias and Y move in row chunks of
  // about 8 MiB of X so that uploads, GEMMs and downloads overlap (W and a
  // row bias are uploaded whole, ahead of the first chunk).
  // (Chain boundaries are staged whole, so such calls do not pipeline.)
  const int64_t chunk_rows =
      host && !call.timed() && num_bnds == 0 ? pipeline_chunk_rows(m, x) : 0;
  const bool full_bias = ep.bias_mode == MCB_BIAS_FULL;
  void *dx, *dw, *dy, *db = nullptr;
  const bool serial = chunk_rows == 0;
  if ((s = call.device_ptr(x, serial, &dx)) || (s = call.device_ptr(w, serial, &dw)) ||
      (s = call.device_ptr(y, false, &dy)))
    return s;
  if (ep.bias_mode && (s = call.device_ptr(bias, serial, &db))) return s;
  for (uint32_t i = 0; i < num_bnds; ++i) {
    void *d = nullptr;
    if ((s = call.device_ptr(bt[i], true, &d))) return s;
    ep.bnd[i] = d;
  }
  ep.bias = db;
  ep.bias_aligned16 = (reinterpret_cast<uintptr_t>(db) & 15u) == 0;
  LaunchInfo info;
  cudaError_t err = cudaSuccess;
  const int64_t ld_x = x->strides[0], ld_w = w->strides[0], ld_y = y->strides[0];
  // Tensor-core eligibility: TMA wants 16-byte aligned bases and row strides.
  // Row chunks start at multiples of 256 rows, so they keep the alignment.
  const bool tma_ok = (in_bf16 || in_f16) && k > 0 && (k % 8 == 0) && (ld_x % 8 == 0) &&
                      (ld_w % 8 == 0) && (wt || n % 8 == 0) &&
                      (reinterpret_cast<uintptr_t>(dx) % 16 == 0) &&
                      (reinterpret_cast<uintptr_t>(dw) % 16 == 0) &&
                      (reinterpret_cast<uintptr_t>(dy) % 16 == 0) &&
                      (ld_y % (y->dtype == MCB_DTYPE_F32 ? 4 : 8) == 0);
  const int y_kind = y->dtype == MCB_DTYPE_F32   ? mcb::kOutF32
                     : y->dtype == MCB_DTYPE_F16 ? mcb::kOutF16
                                                 : mcb::kOutBf16;
  const size_t xs = dtype_size(x->dtype), ys = dtype_size(y->dtype);
  const size_t bs = ep.bias_mode ? dtype_size(bias->dtype) : 0;
  auto launch_rows = [&](int64_t r0, int64_t r1) -> cudaError_t {
    const void *xr = static_cast<const char *>(dx) + r0 * ld_x * xs;
    void *yr = static_cast<char *>(dy) + r0 * ld_y * ys;
    mcb::Epilogue e = ep;
    if (full_bias) {
      e.bias = static_cast<const char *>(db) + r0 * ep.ld_bias * bs;
      e.bias_aligned16 = (reinterpret_cast<uintptr_t>(e.bias) & 15u) == 0;
    }
    for (uint32_t i = 0; i < num_bnds; ++i)
      e.bnd[i] = static_cast<const char *>(ep.bnd[i]) + r0 * ep.ld_bnd[i] * dtype_size(bt[i]->dtype);
    if (tma_ok)
      return mcb::launch_gemm_tc_bf16(xr, dw, yr, r1 - r0, n, k, ld_x, ld_w, ld_y, wt ? 1 : 0,
                                      y_kind, e, call.ctx()->status, call.sms(), call.stream(),
                                      &info, in_f16 ? 1 : 0);
    return mcb::launch_gemm_simt(xr, static_cast<int>(x->dtype), dw, static_cast<int>(w->dtype),
                                 yr, static_cast<int>(y->dtype), r1 - r0, n, k, ld_x, ld_w, ld_y,
                                 wt ? 1 : 0, e, call.stream(), &info);
  };
  call.mark_compute_start();
  if (chunk_rows) {
    const Call::RowOperand whole[2] = {{w, dw}, {ep.bias_mode ? bias : nullptr, db}};
    const Call::RowOperand ins[2] = {{x, dx}, {bias, db}};
    int launches = 0;
    s = call.run_row_pipeline(
        m, chunk_rows, whole, full_bias ? 1 : 2, ins, full_bias ? 2 : 1, Call::RowOperand{y, dy},
        [&](int64_t r0, int64_t r1) {
          ++launches;
          return launch_rows(r0, r1);
        },
        &err);
    if (s) return s;
    info.launches = launches;
  } else if (tma_ok) {
    err = call.with_stream_k(&info, [&](const mcb::GemmStreamK *sk) {
      return mcb::launch_gemm_tc_bf16(dx, dw, dy, m, n, k, ld_x, ld_w, ld_y, wt ? 1 : 0, y_kind,
                                      ep, call.ctx()->status, call.sms(), call.stream(), &info,
                                      in_f16 ? 1 : 0, sk);
    });
  } else {
    err = launch_rows(0, m);
  }
  call.mark_compute_end();
  return call.finish(y, dy, info, err);
}

// ---- typed GEMMs --------------------------------------------------------------------------
mcb_status typed_gemm_impl(const mcb_tensor *c, const mcb_tensor *a, const mcb_tensor *b,
                           const mcb_exec *exec, bool int8, int32_t za = 0, int32_t zb = 0) {
  mcb_status s;
  if ((s = check_tensor(a, 2, 2)) || (s = check_tensor(b, 2, 2)) || (s = check_tensor(c, 2, 2)))
    return s;
  const mcb_dtype in_t = int8 ? MCB_DTYPE_I8 : MCB_DTYPE_BF16;
  const mcb_dtype out_t = int8 ? MCB_DTYPE_I32 : MCB_DTYPE_F32;
  if (a->dtype != in_t || b->dtype != in_t || c->dtype != out_t) return MCB_STATUS_UNSUPPORTED_DTYPE;
  const int64_t m = a->dims[0], k = a->dims[1], n = b->dims[1];
  if (b->dims[0] != k || c->dims[0] != m || c->dims[1] != n) return MCB_STATUS_SHAPE_MISMATCH;
  if (overlaps(c, a) || overlaps(c, b)) return MCB_STATUS_ALIAS_VIOLATION;
  bool host = false;
  if ((s = same_space({a, b, c}, &host))) return s;
  Call call(exec);
  if ((s = call.begin(host))) return s;
  void *da, *db, *dc;
  if ((s = call.device_ptr(a, true, &da)) || (s = call.device_ptr(b, true, &db)) ||
      (s = call.device_ptr(c, false, &dc)))
    return s;
  LaunchInfo info;
  cudaError_t err = cudaErrorNotSupported;
  call.mark_compute_start();
  if (!int8) {
    err = mcb::launch_gemm_bf16_fma(da, db, static_cast<float *>(dc), m, n, k, a->strides[0],
                                    b->strides[0], c->strides[0], call.stream(), &info);
  } else {
    const int64_t lda = a->strides[0], ldb = b->strides[0];
    const bool tc = k > 0 && lda % 16 == 0 && (reinterpret_cast<uintptr_t>(da) % 16 == 0) &&
                    c->strides[0] % 4 == 0 && (reinterpret_cast<uintptr_t>(dc) % 16 == 0);
    const bool b_direct = ldb % 16 == 0 && (reinterpret_cast<uintptr_t>(db) % 16 == 0);
    if (tc && (b_direct || k % 16 == 0)) {
      // B [K,N] is read MN-major in place when its rows are 16-byte aligned;
      // otherwise it is first transposed into a dense B^T [N,K] (row stride
      // K). Zero points add a pre-pass for the row sums of A and column
      // sums of B. One scratch block: [B^T][row sums][column sums], each
      // part 16-byte aligned.
      auto up16 = [](uint64_t x) { return (x + 15) & ~uint64_t{15}; };
      const uint64_t bt_bytes =
          b_direct ? 0 : up16(static_cast<uint64_t>(n) * static_cast<uint64_t>(k));
      const uint64_t rs_bytes = zb != 0 ? up16(static_cast<uint64_t>(m) * 4) : 0;
      const uint64_t cs_bytes = za != 0 ? up16(static_cast<uint64_t>(n) * 4) : 0;
      uint8_t *scr = nullptr;
      if (bt_bytes + rs_bytes + cs_bytes > 0) {
        void *p = nullptr;
        if ((s = call.scratch(bt_bytes + rs_bytes + cs_bytes, &p))) return s;
        scr = static_cast<uint8_t *>(p);
      }
      const int8_t *bop = static_cast<const int8_t *>(db);
      int64_t ld_bop = ldb;
      int b_mn = 1;
      err = cudaSuccess;
      if (!b_direct) {
        err = mcb::launch_transpose_u8(db, scr, k, n, ldb, call.stream());
        info.launches = 1;
        bop = reinterpret_cast<const int8_t *>(scr);
        ld_bop = k;
        b_mn = 0;
      }
      mcb::I8ZeroPoints zpv;
      zpv.za = za;
      zpv.zb = zb;
      zpv.row_sum = rs_bytes ? reinterpret_cast<int32_t *>(scr + bt_bytes) : nullptr;
      zpv.col_sum = cs_bytes ? reinterpret_cast<int32_t *>(scr + bt_bytes + rs_bytes) : nullptr;
      const bool zp_on = za != 0 || zb != 0;
      if (err == cudaSuccess && zp_on)
        err = mcb::launch_i8_zero_point_sums(
            static_cast<const int8_t *>(da), lda, bop, ld_bop, b_mn, m, n, k, zpv,
            const_cast<int32_t *>(zpv.row_sum), const_cast<int32_t *>(zpv.col_sum), call.sms(),
            call.stream(), &info);
      if (err == cudaSuccess)
        err = mcb::launch_gemm_i8_tc(static_cast<const int8_t *>(da), lda, bop, ld_bop, b_mn,
                                     static_cast<int32_t *>(dc), m, n, k, c->strides[0],
                                     zp_on ? &zpv : nullptr, call.ctx()->status, call.sms(),
                                     call.stream(), &info);
    }
    if (err == cudaErrorNotSupported) {
      info.launches = 0;
      err = mcb::launch_gemm_i8_simt(static_cast<const int8_t *>(da),
                                     static_cast<const int8_t *>(db), static_cast<int32_t *>(dc),
                                     m, n, k, a->strides[0], b->strides[0], c->strides[0], za, zb,
                                     call.stream(), &info);
    }
  }
  call.mark_compute_end();
  return call.finish(c, dc, info, err);
}

// ---- Family B -----------------------------------------------------------------------------
// One GEMM launch on whichever kernel the operands allow (tcgen05 for
// TMA-compatible bf16, CUDA cores otherwise).
cudaError_t launch_gemm_any(const void *x, int x_dt, const void *w, int w_dt, void *y, int y_dt,
                            int64_t m, int64_t n, int64_t k, int64_t ld_x, int64_t ld_w,
                            int64_t ld_y, const mcb::Epilogue &ep, Call &call, LaunchInfo *info) {
  const bool bf16 = x_dt == MCB_DTYPE_BF16 && w_dt == MCB_DTYPE_BF16;
  const bool tma_ok = bf16 && k > 0 && k % 8 == 0 && n % 8 == 0 && ld_x % 8 == 0 &&
                      ld_w % 8 == 0 && (reinterpret_cast<uintptr_t>(x) % 16 == 0) &&
                      (reinterpret_cast<uintptr_t>(w) % 16 == 0) &&
                      (reinterpret_cast<uintptr_t>(y) % 16 == 0) &&
                      ld_y % (y_dt == MCB_DTYPE_BF16 ? 8 : 4) == 0;
  if (tma_ok)
    return mcb::launch_gemm_tc_bf16(x, w, y, m, n, k, ld_x, ld_w, ld_y, 0,
                                    y_dt == MCB_DTYPE_BF16 ? 1 : 0, ep, call.ctx()->status,
                                    call.sms(), call.stream(), info);
  return mcb::launch_gemm_simt(x, x_dt, w, w_dt, y, y_dt, m, n, k, ld_x, ld_w, ld_y, 0, ep,
                               call.stream(), info);
}

mcb_status chain_impl(const mcb_tensor *e, const mcb_tensor *a, const mcb_tensor *b,
                      const mcb_tensor *boundary, const mcb_epilogue *glue, const mcb_tensor *w,
                      const mcb_exec *exec) {
  mcb_status s;
  if ((s = check_tensor(a, 2, 2)) || (s = check_tensor(b, 2, 2)) || (s = check_tensor(w, 2, 2)) ||
      (s = check_tensor(e, 2, 2)))
    return s;
  const int dt = static_cast<int>(a->dtype);
  if ((dt != MCB_DTYPE_BF16 && dt != MCB_DTYPE_F32) || b->dtype != a->dtype ||
      w->dtype != a->dtype || (e->dtype != MCB_DTYPE_BF16 && e->dtype != MCB_DTYPE_F32))
    return MCB_STATUS_UNSUPPORTED_DTYPE;
  const int64_t m = a->dims[0], k = a->dims[1], n1 = b->dims[1], n2 = w->dims[1];
  if (b->dims[0] != k || w->dims[0] != n1 || e->dims[0] != m || e->dims[1] != n2)
    return MCB_STATUS_SHAPE_MISMATCH;
  mcb::Epilogue ep;
  if (glue) {
    if (glue->abi_version != MCB_ABI_VERSION_V1 || glue->struct_size < sizeof(mcb_epilogue))
      return MCB_STATUS_ABI_MISMATCH;
    if (glue->bias_mode > MCB_BIAS_FULL || glue->bias_op > MCB_BIAS_RSUB ||
        glue->activation > MCB_ACT_TANH)
      return MCB_STATUS_INVALID_ARGUMENT;
    ep.bias_mode = static_cast<int>(glue->bias_mode);
    ep.bias_op = static_cast<int>(glue->bias_op);
    ep.act = static_cast<int>(glue->activation);
  }
  if (ep.bias_mode != MCB_BIAS_NONE) {
    if ((s = check_tensor(boundary, 1, 2))) return s;
    if (boundary->dtype != MCB_DTYPE_BF16 && boundary->dtype != MCB_DTYPE_F32)
      return MCB_STATUS_UNSUPPORTED_DTYPE;
    if (ep.bias_mode == MCB_BIAS_ROW && numel(boundary) != n1) return MCB_STATUS_SHAPE_MISMATCH;
    if (ep.bias_mode == MCB_BIAS_FULL &&
        !(boundary->rank == 2 && boundary->dims[0] == m && boundary->dims[1] == n1))
      return MCB_STATUS_SHAPE_MISMATCH;
    ep.bias_bf16 = boundary->dtype == MCB_DTYPE_BF16;
    ep.ld_bias = boundary->rank == 2 ? boundary->strides[0] : n1;
  }
  for (const mcb_tensor *t : {a, b, w}) if (overlaps(e, t)) return MCB_STATUS_ALIAS_VIOLATION;
  if (ep.bias_mode && overlaps(e, boundary)) return MCB_STATUS_ALIAS_VIOLATION;
  bool host = false;
  if ((s = same_space({a, b, w, e, ep.bias_mode ? boundary : nullptr}, &host))) return s;
  Call call(exec);
  if ((s = call.begin(host))) return s;
  void *da, *db, *dw, *de, *dbnd = nullptr, *mid = nullptr;
  if ((s = call.device_ptr(a, true, &da)) || (s = call.device_ptr(b, true, &db)) ||
      (s = call.device_ptr(w, true, &dw)) || (s = call.device_ptr(e, false, &de)))
    return s;
  if (ep.bias_mode && (s = call.device_ptr(boundary, true, &dbnd))) return s;
  ep.bias = dbnd;
  ep.bias_aligned16 = (reinterpret_cast<uintptr_t>(dbnd) & 15u) == 0;
  // bf16 operands with TMA-compatible rows: one fused tensor-core kernel, the
  // intermediate kept on chip (TMEM and shared memory), no scratch, where it
  // is the faster route (measured, back to back, B200):
  //  - tiny problems (M*K*N1 <= 2^25), where the second launch and the
  //    intermediate's round trip dominate (256x512x256x64: 23.7 vs 30.1 us);
  //  - K <= 256 with at least 8192 rows and E at most 256 wide, where the
  //    intermediate outweighs A (16384x256x4096x64: 103.8 vs 114.0 us).
  // The fused kernel re-reads A once per 128 intermediate columns and runs
  // one unit per 128 rows, so elsewhere the two GEMMs below win
  // (16384x4096x4096x256: 927 vs 424 us; 1024x1024x1024x256: 92 vs 29 us).
  const bool small_chain = m * k * n1 <= (int64_t{1} << 25) && n2 <= 512;
  const bool thin_chain = k <= 256 && m >= 8192 && n2 <= 256;
  auto al16 = [](const void *ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; };
  // MCB_CHAIN_FUSED (read per call): 0 = always two GEMMs, 2 = fused at any
  // size (A/B measurement); unset = the rule above.
  const char *fused_env = getenv("MCB_CHAIN_FUSED");
  const int fused_mode = fused_env ? atoi(fused_env) : 1;
  if (fused_mode != 0 && (small_chain || thin_chain || fused_mode == 2) && dt == MCB_DTYPE_BF16 && k > 0 && n1 > 0 && k % 8 == 0 &&
      n1 % 8 == 0 && n2 % 8 == 0 &&
      a->strides[0] % 8 == 0 && b->strides[0] % 8 == 0 && w->strides[0] % 8 == 0 && al16(da) &&
      al16(db) && al16(dw)) {
    LaunchInfo info;
    call.mark_compute_start();
    const cudaError_t err = mcb::launch_chain_tc_bf16(
        da, db, dw, de, m, k, n1, n2, a->strides[0], b->strides[0], w->strides[0], e->strides[0],
        e->dtype == MCB_DTYPE_BF16 ? mcb::kOutBf16 : mcb::kOutF32, ep, call.ctx()->status,
        call.sms(), call.stream(), &info);
    if (err != cudaErrorNotSupported) {
      call.mark_compute_end();
      return call.finish(e, de, info, err);
    }
  }
  // Small f32 chains (the reference's Family B test dtype): one CUDA-core
  // launch, the f32 intermediate in shared memory.
  if (dt == MCB_DTYPE_F32 && small_chain && m * n1 * k <= (int64_t{1} << 27)) {
    LaunchInfo info;
    call.mark_compute_start();
    const cudaError_t err = mcb::launch_chain_simt_small(
        da, db, dw, de, dt, static_cast<int>(e->dtype), m, k, n1, n2, a->strides[0],
        b->strides[0], w->strides[0], e->strides[0], ep, call.stream(), &info);
    if (err != cudaErrorNotSupported) {
      call.mark_compute_end();
      return call.finish(e, de, info, err);
    }
  }
  const int64_t ld_mid = (n1 + 7) / 8 * 8;  // 16-byte rows for the second GEMM's TMA
  const size_t esz = dt == MCB_DTYPE_BF16 ? 2 : 4;
  if ((s = call.scratch(static_cast<uint64_t>(m) * ld_mid * esz, &mid))) return s;
  LaunchInfo i1, i2;
  call.mark_compute_start();
  cudaError_t err = launch_gemm_any(da, dt, db, dt, mid, dt, m, n1, k, a->strides[0], b->strides[0],
                                    ld_mid, ep, call, &i1);
  mcb::Epilogue none;
  if (err == cudaSuccess)
    err = launch_gemm_any(mid, dt, dw, dt, de, static_cast<int>(e->dtype), m, n2, n1, ld_mid,
                          w->strides[0], e->strides[0], none, call, &i2);
  call.mark_compute_end();
  LaunchInfo info = i2;
  info.launches = i1.launches + i2.launches;
  char route[48];
  std::snprintf(route, sizeof(route), "chain:%s", i1.route);
  info.set_route(route);
  return call.finish(e, de, info, err);
}

// ---- Family C -----------------------------------------------------------------------------
constexpr bool kHaveMsmTc = true;

mcb_status msm_impl(const mcb_tensor *o, const mcb_tensor *q, const mcb_tensor *k,
                    const mcb_tensor *v, double scale, const mcb_exec *exec) {
  mcb_status s;
  if ((s = check_tensor(q, 2, 4)) || (s = check_tensor(k, 2, 4)) || (s = check_tensor(v, 2, 4)) ||
      (s = check_tensor(o, 2, 4)))
    return s;
  const uint32_t r = q->rank;
  if (k->rank != r || v->rank != r || o->rank != r) return MCB_STATUS_SHAPE_MISMATCH;
  if (q->dtype != k->dtype || q->dtype != v->dtype || q->dtype != o->dtype)
    return MCB_STATUS_UNSUPPORTED_DTYPE;
  if (q->dtype != MCB_DTYPE_BF16 && q->dtype != MCB_DTYPE_F32) return MCB_STATUS_UNSUPPORTED_DTYPE;
  mcb::MsmShape sh;
  sh.m = q->dims[r - 2];
  sh.dqk = q->dims[r - 1];
  sh.n = k->dims[r - 2];
  sh.dv = v->dims[r - 1];
  if (k->dims[r - 1] != sh.dqk || v->dims[r - 2] != sh.n || o->dims[r - 2] != sh.m ||
      o->dims[r - 1] != sh.dv)
    return MCB_STATUS_SHAPE_MISMATCH;
  for (uint32_t i = 0; i + 2 < r; ++i)
    if (k->dims[i] != q->dims[i] || v->dims[i] != q->dims[i] || o->dims[i] != q->dims[i])
      return MCB_STATUS_SHAPE_MISMATCH;
  sh.batch = r == 4 ? q->dims[0] : 1;
  sh.heads = r >= 3 ? q->dims[r - 3] : 1;
  auto fill = [&](const mcb_tensor *t, int64_t *st) {
    st[0] = r == 4 ? t->strides[0] : 0;
    st[1] = r >= 3 ? t->strides[r - 3] : 0;
    st[2] = t->strides[r - 2];
  };
  fill(q, sh.q_s);
  fill(k, sh.k_s);
  fill(v, sh.v_s);
  fill(o, sh.o_s);
  if (sh.n == 0) return MCB_STATUS_INVALID_SHAPE;  // softmax over zero keys is undefined
  // The kernels compute in f32: a scale that is not finite there is rejected.
  if (!std::isfinite(scale) || !std::isfinite(static_cast<float>(scale)))
    return MCB_STATUS_INVALID_ARGUMENT;
  if (overlaps(o, q) || overlaps(o, k) || overlaps(o, v)) return MCB_STATUS_ALIAS_VIOLATION;
  bool host = false;
  if ((s = same_space({q, k, v, o}, &host))) return s;
  Call call(exec);
  if ((s = call.begin(host))) return s;
  void *dq, *dk, *dv, *dout;
  if ((s = call.device_ptr(q, true, &dq)) || (s = call.device_ptr(k, true, &dk)) ||
      (s = call.device_ptr(v, true, &dv)) || (s = call.device_ptr(o, false, &dout)))
    return s;
  LaunchInfo info;
  cudaError_t err;
  call.mark_compute_start();
  // Any M and N: a partial last query block and key tile are handled in the
  // kernels (zero-filled loads, masked keys, skipped rows).
  const bool tc_ok = kHaveMsmTc && q->dtype == MCB_DTYPE_BF16 && sh.dqk == sh.dv &&
                     (sh.dqk == 64 || sh.dqk == 128) &&
                     sh.m < (int64_t{1} << 31) && sh.n < (int64_t{1} << 31) &&
                     sh.q_s[2] % 8 == 0 && sh.k_s[2] % 8 == 0 && sh.v_s[2] % 8 == 0 &&
                     sh.o_s[2] % 8 == 0 && sh.q_s[0] % 8 == 0 && sh.q_s[1] % 8 == 0 &&
                     sh.k_s[0] % 8 == 0 && sh.k_s[1] % 8 == 0 && sh.v_s[0] % 8 == 0 &&
                     sh.v_s[1] % 8 == 0 && (reinterpret_cast<uintptr_t>(dq) % 16 == 0) &&
                     (reinterpret_cast<uintptr_t>(dk) % 16 == 0) &&
                     (reinterpret_cast<uintptr_t>(dv) % 16 == 0) &&
                     (reinterpret_cast<uintptr_t>(dout) % 16 == 0);
  err = cudaErrorNotSupported;
  if (tc_ok)
    err = mcb::launch_msm_tc_bf16(dq, dk, dv, dout, sh, static_cast<float>(scale),
                                  call.ctx()->status, call.sms(), call.stream(), &info);
  if (err == cudaErrorNotSupported) {
    if (sh.dqk > 256 || sh.dv > 256) return MCB_STATUS_UNAVAILABLE_VARIANT;
    err = mcb::launch_msm_simt(dq, dk, dv, dout, static_cast<int>(q->dtype), sh,
                               static_cast<float>(scale), call.stream(), &info);
  }
  call.mark_compute_end();
  return call.finish(o, dout, info, err);
}

// ---- FP8 ---------------------------------------------------------------------------------
bool is_fp8(mcb_dtype t) { return t == MCB_DTYPE_E4M3 || t == MCB_DTYPE_E5M2; }

// Dense row-major rank-2 tensor of the given shape.
bool dense2(const mcb_tensor *t, int64_t rows, int64_t cols) {
  return t->rank == 2 && t->dims[0] == rows && t->dims[1] == cols &&
         (rows <= 1 || t->strides[0] == cols) && t->strides[1] == 1;
}

mcb_status fp8_quantize_impl(const mcb_tensor *q, const mcb_tensor *scales, const mcb_tensor *x,
                             int64_t block, const mcb_exec *exec) {
  mcb_status s;
  if ((s = check_tensor(x, 2, 2)) || (s = check_tensor(q, 2, 2)) ||
      (s = check_tensor(scales, 2, 2)))
    return s;
  if (block <= 0) return MCB_STATUS_INVALID_ARGUMENT;
  if (x->dtype != MCB_DTYPE_F32 && x->dtype != MCB_DTYPE_BF16) return MCB_STATUS_UNSUPPORTED_DTYPE;
  if (!is_fp8(q->dtype) || scales->dtype != MCB_DTYPE_F32) return MCB_STATUS_UNSUPPORTED_DTYPE;
  const int64_t rows = x->dims[0], cols = x->dims[1];
  if (!dense2(q, rows, cols)) return MCB_STATUS_SHAPE_MISMATCH;
  if (!dense2(scales, (rows + block - 1) / block, (cols + block - 1) / block))
    return MCB_STATUS_SHAPE_MISMATCH;
  if (overlaps(q, x) || overlaps(scales, x) || overlaps(q, scales))
    return MCB_STATUS_ALIAS_VIOLATION;
  bool host = false;
  if ((s = same_space({x, q, scales}, &host))) return s;
  Call call(exec);
  if ((s = call.begin(host))) return s;
  void *dx, *dq, *ds;
  if ((s = call.device_ptr(x, true, &dx)) || (s = call.device_ptr(q, false, &dq)) ||
      (s = call.device_ptr(scales, false, &ds)))
    return s;
  LaunchInfo info;
  call.mark_compute_start();
  cudaError_t err = mcb::launch_fp8_quantize(
      dx, static_cast<int>(x->dtype), static_cast<uint8_t *>(dq), static_cast<float *>(ds), rows,
      cols, x->strides[0], block, q->dtype == MCB_DTYPE_E5M2, call.stream(), &info);
  call.mark_compute_end();
  if (err != cudaSuccess) return from_cuda(err);
  // Both outputs come back for host callers.
  if (host && numel(scales) > 0) {
    if (cudaMemcpyAsync(scales->data, ds, span_bytes(scales), cudaMemcpyDeviceToHost,
                        call.stream()) != cudaSuccess)
      return MCB_STATUS_CANDIDATE_FAILURE;
  }
  return call.finish(q, dq, info, cudaSuccess);
}

mcb_status gemm_fp8_impl(const mcb_tensor *c, const mcb_tensor *a, const mcb_tensor *sa,
                         const mcb_tensor *bt, const mcb_tensor *sbt, int64_t block,
                         const mcb_exec *exec) {
  mcb_status s;
  if ((s = check_tensor(a, 2, 2)) || (s = check_tensor(bt, 2, 2)) || (s = check_tensor(sa, 2, 2)) ||
      (s = check_tensor(sbt, 2, 2)) || (s = check_tensor(c, 2, 2)))
    return s;
  if (block <= 0) return MCB_STATUS_INVALID_ARGUMENT;
  if (!is_fp8(a->dtype) || !is_fp8(bt->dtype)) return MCB_STATUS_UNSUPPORTED_DTYPE;
  if (sa->dtype != MCB_DTYPE_F32 || sbt->dtype != MCB_DTYPE_F32) return MCB_STATUS_UNSUPPORTED_DTYPE;
  if (c->dtype != MCB_DTYPE_BF16 && c->dtype != MCB_DTYPE_F32) return MCB_STATUS_UNSUPPORTED_DTYPE;
  const int64_t m = a->dims[0], k = a->dims[1], n = bt->dims[0];
  const int64_t kbs = (k + block - 1) / block;
  if (!dense2(a, m, k) || !dense2(bt, n, k) || !dense2(c, m, n) ||
      !dense2(sa, (m + block - 1) / block, kbs) || !dense2(sbt, (n + block - 1) / block, kbs))
    return MCB_STATUS_SHAPE_MISMATCH;
  if (overlaps(c, a) || overlaps(c, bt) || overlaps(c, sa) || overlaps(c, sbt))
    return MCB_STATUS_ALIAS_VIOLATION;
  bool host = false;
  if ((s = same_space({a, bt, sa, sbt, c}, &host))) return s;
  Call call(exec);
  if ((s = call.begin(host))) return s;
  void *da, *db, *dsa, *dsb, *dc;
  if ((s = call.device_ptr(a, true, &da)) || (s = call.device_ptr(bt, true, &db)) ||
      (s = call.device_ptr(sa, true, &dsa)) || (s = call.device_ptr(sbt, true, &dsb)) ||
      (s = call.device_ptr(c, false, &dc)))
    return s;
  LaunchInfo info;
  call.mark_compute_start();
  const int ae5 = a->dtype == MCB_DTYPE_E5M2, be5 = bt->dtype == MCB_DTYPE_E5M2;
  const int cbf = c->dtype == MCB_DTYPE_BF16;
  cudaError_t err = cudaErrorNotSupported;
  const bool aligned = (reinterpret_cast<uintptr_t>(da) % 16 == 0) &&
                       (reinterpret_cast<uintptr_t>(db) % 16 == 0) &&
                       (reinterpret_cast<uintptr_t>(dc) % 16 == 0) && (n % 8 == 0);
  if (aligned && k > 0)
    err = mcb::launch_gemm_fp8_tc(static_cast<const uint8_t *>(da), ae5,
                                  static_cast<const float *>(dsa), static_cast<const uint8_t *>(db),
                                  be5, static_cast<const float *>(dsb), dc, cbf, m, n, k, block,
                                  call.ctx()->status, call.sms(), call.stream(), &info);
  if (err == cudaErrorNotSupported)
    err = mcb::launch_gemm_fp8_simt(static_cast<const uint8_t *>(da), ae5,
                                    static_cast<const float *>(dsa),
                                    static_cast<const uint8_t *>(db), be5,
                                    static_cast<const float *>(dsb), dc, cbf, m, n, k, block,
                                    call.stream(), &info);
  call.mark_compute_end();
  return call.finish(c, dc, info, err);
}

// ---- block_attn_res ------------------------------------------------------------------------
mcb_status block_attn_res_impl(const mcb_tensor *out, const mcb_tensor *blocks,
                               const mcb_tensor *partial, const mcb_tensor *query,
                               int64_t block_count, int32_t has_partial, float eps,
                               const mcb_exec *exec) {
  mcb_status s;
  if ((s = check_tensor(blocks, 4, 4)) || (s = check_tensor(partial, 3, 3)) ||
      (s = check_tensor(query, 1, 1)) || (s = check_tensor(out, 3, 3)))
    return s;
  for (const mcb_tensor *t : {blocks, partial, query, out})
    if (t->dtype != MCB_DTYPE_F32) return MCB_STATUS_UNSUPPORTED_DTYPE;
  const int64_t maxb = blocks->dims[0], B = blocks->dims[1], T = blocks->dims[2],
                D = blocks->dims[3];
  if (maxb < 1 || maxb > 32) return MCB_STATUS_INVALID_SHAPE;          // MAX_BLOCKS in [1, 32]
  if (block_count < 0 || block_count > maxb) return MCB_STATUS_INVALID_ARGUMENT;
  if (!(eps > 0.0f)) return MCB_STATUS_INVALID_ARGUMENT;               // eps must be positive
  auto dense = [](const mcb_tensor *t) {
    int64_t st = 1;
    for (int i = static_cast<int>(t->rank) - 1; i >= 0; --i) {
      if (t->dims[i] > 1 && t->strides[i] != st) return false;
      st *= t->dims[i];
    }
    return true;
  };
  for (const mcb_tensor *t : {blocks, partial, query, out})
    if (!dense(t)) return MCB_STATUS_UNSUPPORTED_LAYOUT;
  for (const mcb_tensor *t : {partial, out})
    if (t->dims[0] != B || t->dims[1] != T || t->dims[2] != D) return MCB_STATUS_SHAPE_MISMATCH;
  if (query->dims[0] != D) return MCB_STATUS_SHAPE_MISMATCH;
  for (const mcb_tensor *t : {blocks, partial, query})
    if (overlaps(out, t)) return MCB_STATUS_ALIAS_VIOLATION;
  bool host = false;
  if ((s = same_space({blocks, partial, query, out}, &host))) return s;
  Call call(exec);
  if ((s = call.begin(host))) return s;
  void *db, *dp, *dq, *dout;
  if ((s = call.device_ptr(blocks, true, &db)) || (s = call.device_ptr(partial, true, &dp)) ||
      (s = call.device_ptr(query, true, &dq)) || (s = call.device_ptr(out, false, &dout)))
    return s;
  LaunchInfo info;
  call.mark_compute_start();
  cudaError_t err = mcb::launch_block_attn_res(
      static_cast<const float *>(db), static_cast<const float *>(dp),
      static_cast<const float *>(dq), static_cast<float *>(dout), B * T, D, B * T * D,
      static_cast<int>(block_count), has_partial ? 1 : 0, eps, call.sms(), call.stream(), &info);
  call.mark_compute_end();
  return call.finish(out, dout, info, err);
}

// ---- attention-residual block region ------------------------------------------------------
uint64_t attn_workspace_bytes(int64_t batch, int64_t seq, int64_t d) {
  // Q, K, V, O and the output projection: five [B*S, D] bf16 buffers.
  const uint64_t one = static_cast<uint64_t>(batch) * seq * d * 2;
  return 5 * ((one + 255) / 256 * 256);
}

mcb_status attn_block_impl(const mcb_tensor *y, const mcb_tensor *x, const mcb_tensor *wq,
                           const mcb_tensor *wk, const mcb_tensor *wv, const mcb_tensor *wo,
                           int64_t heads, float eps, const mcb_exec *exec) {
  mcb_status s;
  if ((s = check_tensor(x, 3, 3)) || (s = check_tensor(y, 3, 3)) || (s = check_tensor(wq, 2, 2)) ||
      (s = check_tensor(wk, 2, 2)) || (s = check_tensor(wv, 2, 2)) || (s = check_tensor(wo, 2, 2)))
    return s;
  for (const mcb_tensor *t : {x, y, wq, wk, wv, wo})
    if (t->dtype != MCB_DTYPE_BF16) return MCB_STATUS_UNSUPPORTED_DTYPE;
  const int64_t B = x->dims[0], S = x->dims[1], D = x->dims[2];
  if (heads <= 0 || D % heads != 0) return MCB_STATUS_INVALID_ARGUMENT;
  if (!(eps >= 0.0f)) return MCB_STATUS_INVALID_ARGUMENT;
  const int64_t hd = D / heads, M = B * S;
  auto dense3 = [&](const mcb_tensor *t) {
    return t->dims[0] == B && t->dims[1] == S && t->dims[2] == D && t->strides[2] == 1 &&
           (S <= 1 || t->strides[1] == D) && (B <= 1 || t->strides[0] == S * D);
  };
  if (!dense3(x) || !dense3(y)) return MCB_STATUS_SHAPE_MISMATCH;
  for (const mcb_tensor *w : {wq, wk, wv, wo})
    if (!dense2(w, D, D)) return MCB_STATUS_SHAPE_MISMATCH;
  if (S == 0) return MCB_STATUS_INVALID_SHAPE;
  for (const mcb_tensor *t : {x, wq, wk, wv, wo})
    if (overlaps(y, t)) return MCB_STATUS_ALIAS_VIOLATION;
  bool host = false;
  if ((s = same_space({x, y, wq, wk, wv, wo}, &host))) return s;
  Call call(exec);
  if ((s = call.begin(host))) return s;
  void *dx, *dq, *dk, *dv, *dwo, *dy;
  if ((s = call.device_ptr(x, true, &dx)) || (s = call.device_ptr(wq, true, &dq)) ||
      (s = call.device_ptr(wk, true, &dk)) || (s = call.device_ptr(wv, true, &dv)) ||
      (s = call.device_ptr(wo, true, &dwo)) || (s = call.device_ptr(y, false, &dy)))
    return s;
  void *ws = nullptr;
  const uint64_t ws_bytes = attn_workspace_bytes(B, S, D);
  if ((s = call.scratch(ws_bytes, &ws))) return s;
  const uint64_t one = ws_bytes / 5;
  uint8_t *base = static_cast<uint8_t *>(ws);
  void *Q = base, *K = base + one, *V = base + 2 * one, *O = base + 3 * one, *P = base + 4 * one;

  LaunchInfo info, step;
  cudaError_t err = cudaSuccess;
  mcb::Epilogue none;
  const bool tc_gemm = D % 8 == 0 && (reinterpret_cast<uintptr_t>(dx) % 16 == 0) &&
                       (reinterpret_cast<uintptr_t>(ws) % 16 == 0);
  auto gemm = [&](const void *a, const void *w, void *out) {
    if (tc_gemm && (reinterpret_cast<uintptr_t>(w) % 16 == 0))
      return mcb::launch_gemm_tc_bf16(a, w, out, M, D, D, D, D, D, 0, 1, none, call.ctx()->status,
                                      call.sms(), call.stream(), &step);
    return mcb::launch_gemm_simt(a, MCB_DTYPE_BF16, w, MCB_DTYPE_BF16, out, MCB_DTYPE_BF16, M, D,
                                 D, D, D, D, 0, none, call.stream(), &step);
  };
  call.mark_compute_start();
  int launches = 0;
  for (auto [w, out] : {std::pair<void *, void *>{dq, Q}, {dk, K}, {dv, V}}) {
    if ((err = gemm(dx, w, out)) != cudaSuccess) break;
    launches += step.launches;
  }
  if (err == cudaSuccess) {
    // Q/K/V/O are [B, S, D] = [B, S, H, hd]; the MSM reads them as the
    // strided head-major view [B, H, S, hd] (no transpose pass).
    mcb::MsmShape sh;
    sh.batch = B;
    sh.heads = heads;
    sh.m = sh.n = S;
    sh.dqk = sh.dv = hd;
    const int64_t st[3] = {S * D, hd, D};
    for (int i = 0; i < 3; ++i) sh.q_s[i] = sh.k_s[i] = sh.v_s[i] = sh.o_s[i] = st[i];
    const float scale = 1.0f / std::sqrt(static_cast<float>(hd));
    err = cudaErrorNotSupported;
    if ((hd == 64 || hd == 128) && D % 8 == 0)
      err = mcb::launch_msm_tc_bf16(Q, K, V, O, sh, scale, call.ctx()->status, call.sms(),
                                    call.stream(), &step);
    if (err == cudaErrorNotSupported) {
      err = hd <= 256 ? mcb::launch_msm_simt(Q, K, V, O, MCB_DTYPE_BF16, sh, scale, call.stream(),
                                             &step)
                      : cudaErrorNotSupported;
    }
    launches += step.launches;
  }
  if (err == cudaSuccess) {
    err = gemm(O, dwo, P);
    launches += step.launches;
  }
  if (err == cudaSuccess) {
    step.launches = 0;
    err = mcb::launch_residual_rmsnorm(dx, P, dy, M, D, eps, call.stream(), &step);
    launches += step.launches;
  }
  call.mark_compute_end();
  if (err == cudaErrorNotSupported) return MCB_STATUS_UNAVAILABLE_VARIANT;
  info.launches = launches;
  info.tile_m = 128;
  info.tile_n = 256;
  info.ctas = call.sms();
  info.set_route("attn_block_region");
  return call.finish(y, dy, info, err);
}

// ---- head-sharded attention block (the region split over GPUs by heads) --------------------
// One head group's share of the region's output projection,
//   P = MSM(X Wq_g, X Wk_g, X Wv_g) Wo_g,
// with Wq_g / Wk_g / Wv_g the group's [D, Dh] column slices and Wo_g the
// matching [Dh, D] row slice. The sum of P over all head groups is the
// region's Wo * MSM(...); residual_rmsnorm_impl then finishes the block.
uint64_t attn_heads_workspace_bytes(int64_t rows, int64_t dh) {
  // Q, K, V and O of the group: four [rows, Dh] bf16 buffers.
  const uint64_t one = static_cast<uint64_t>(rows) * dh * 2;
  return 4 * ((one + 255) / 256 * 256);
}

mcb_status attn_heads_impl(const mcb_tensor *p, const mcb_tensor *x, const mcb_tensor *wq,
                           const mcb_tensor *wk, const mcb_tensor *wv, const mcb_tensor *wo,
                           int64_t heads, const mcb_exec *exec) {
  mcb_status s;
  if ((s = check_tensor(x, 3, 3)) || (s = check_tensor(p, 3, 3)) || (s = check_tensor(wq, 2, 2)) ||
      (s = check_tensor(wk, 2, 2)) || (s = check_tensor(wv, 2, 2)) || (s = check_tensor(wo, 2, 2)))
    return s;
  for (const mcb_tensor *t : {x, p, wq, wk, wv, wo})
    if (t->dtype != MCB_DTYPE_BF16) return MCB_STATUS_UNSUPPORTED_DTYPE;
  const int64_t B = x->dims[0], S = x->dims[1], D = x->dims[2], Dh = wq->dims[1];
  if (heads <= 0 || Dh <= 0 || Dh % heads != 0) return MCB_STATUS_INVALID_ARGUMENT;
  const int64_t hd = Dh / heads, M = B * S;
  auto dense3 = [&](const mcb_tensor *t) {
    return t->dims[0] == B && t->dims[1] == S && t->dims[2] == D && t->strides[2] == 1 &&
           (S <= 1 || t->strides[1] == D) && (B <= 1 || t->strides[0] == S * D);
  };
  if (!dense3(x) || !dense3(p)) return MCB_STATUS_SHAPE_MISMATCH;
  for (const mcb_tensor *w : {wq, wk, wv})
    if (!dense2(w, D, Dh)) return MCB_STATUS_SHAPE_MISMATCH;
  if (!dense2(wo, Dh, D)) return MCB_STATUS_SHAPE_MISMATCH;
  if (S == 0) return MCB_STATUS_INVALID_SHAPE;
  for (const mcb_tensor *t : {x, wq, wk, wv, wo})
    if (overlaps(p, t)) return MCB_STATUS_ALIAS_VIOLATION;
  bool host = false;
  if ((s = same_space({x, p, wq, wk, wv, wo}, &host))) return s;
  Call call(exec);
  if ((s = call.begin(host))) return s;
  void *dx, *dq, *dk, *dv, *dwo, *dp;
  if ((s = call.device_ptr(x, true, &dx)) || (s = call.device_ptr(wq, true, &dq)) ||
      (s = call.device_ptr(wk, true, &dk)) || (s = call.device_ptr(wv, true, &dv)) ||
      (s = call.device_ptr(wo, true, &dwo)) || (s = call.device_ptr(p, false, &dp)))
    return s;
  void *ws = nullptr;
  const uint64_t ws_bytes = attn_heads_workspace_bytes(M, Dh);
  if ((s = call.scratch(ws_bytes, &ws))) return s;
  const uint64_t one = ws_bytes / 4;
  uint8_t *base = static_cast<uint8_t *>(ws);
  void *Q = base, *K = base + one, *V = base + 2 * one, *O = base + 3 * one;

  LaunchInfo info, step;
  cudaError_t err = cudaSuccess;
  mcb::Epilogue none;
  // [M, k] x [k, n] -> [M, n], all dense bf16 rows.
  auto gemm = [&](const void *a, const void *w, void *out, int64_t n, int64_t k) {
    const bool tc = k % 8 == 0 && n % 8 == 0 &&
                    ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(w) |
                      reinterpret_cast<uintptr_t>(out)) & 15u) == 0;
    if (tc)
      return mcb::launch_gemm_tc_bf16(a, w, out, M, n, k, k, n, n, 0, 1, none, call.ctx()->status,
                                      call.sms(), call.stream(), &step);
    return mcb::launch_gemm_simt(a, MCB_DTYPE_BF16, w, MCB_DTYPE_BF16, out, MCB_DTYPE_BF16, M, n,
                                 k, k, n, n, 0, none, call.stream(), &step);
  };
  call.mark_compute_start();
  int launches = 0;
  for (auto [w, out] : {std::pair<void *, void *>{dq, Q}, {dk, K}, {dv, V}}) {
    step.launches = 0;
    if ((err = gemm(dx, w, out, Dh, D)) != cudaSuccess) break;
    launches += step.launches;
  }
  if (err == cudaSuccess) {
    // Q/K/V/O are [B, S, Dh] = [B, S, heads, hd], read as [B, heads, S, hd].
    mcb::MsmShape sh;
    sh.batch = B;
    sh.heads = heads;
    sh.m = sh.n = S;
    sh.dqk = sh.dv = hd;
    const int64_t st[3] = {S * Dh, hd, Dh};
    for (int i = 0; i < 3; ++i) sh.q_s[i] = sh.k_s[i] = sh.v_s[i] = sh.o_s[i] = st[i];
    const float scale = 1.0f / std::sqrt(static_cast<float>(hd));
    step.launches = 0;
    err = cudaErrorNotSupported;
    if ((hd == 64 || hd == 128) && Dh % 8 == 0)
      err = mcb::launch_msm_tc_bf16(Q, K, V, O, sh, scale, call.ctx()->status, call.sms(),
                                    call.stream(), &step);
    if (err == cudaErrorNotSupported)
      err = hd <= 256 ? mcb::launch_msm_simt(Q, K, V, O, MCB_DTYPE_BF16, sh, scale, call.stream(),
                                             &step)
                      : cudaErrorNotSupported;
    launches += step.launches;
  }
  if (err == cudaSuccess) {
    step.launches = 0;
    err = gemm(O, dwo, dp, D, Dh);
    launches += step.launches;
  }
  call.mark_compute_end();
  if (err == cudaErrorNotSupported) return MCB_STATUS_UNAVAILABLE_VARIANT;
  info.launches = launches;
  info.tile_m = 128;
  info.tile_n = 256;
  info.ctas = call.sms();
  info.set_route("attn_block_heads");
  return call.finish(p, dp, info, err);
}

// Y = RMSNorm(X + P) over the last dimension (unit gain), the region's last
// step, for X / P / Y of the same dense bf16 shape (rank 2 or 3).
mcb_status residual_rmsnorm_impl(const mcb_tensor *y, const mcb_tensor *x, const mcb_tensor *pp,
                                 float eps, const mcb_exec *exec) {
  mcb_status s;
  if ((s = check_tensor(x, 2, 3)) || (s = check_tensor(y, 2, 3)) || (s = check_tensor(pp, 2, 3)))
    return s;
  for (const mcb_tensor *t : {x, y, pp})
    if (t->dtype != MCB_DTYPE_BF16) return MCB_STATUS_UNSUPPORTED_DTYPE;
  if (!(eps >= 0.0f)) return MCB_STATUS_INVALID_ARGUMENT;
  const int r = x->rank;
  const int64_t D = x->dims[r - 1];
  int64_t rows = 1;
  for (int i = 0; i < r - 1; ++i) rows *= x->dims[i];
  auto dense_like_x = [&](const mcb_tensor *t) {
    if (t->rank != r) return false;
    int64_t stride = 1;
    for (int i = r - 1; i >= 0; --i) {
      if (t->dims[i] != x->dims[i]) return false;
      if (t->dims[i] > 1 && t->strides[i] != stride) return false;
      stride *= t->dims[i];
    }
    return true;
  };
  if (!dense_like_x(x) || !dense_like_x(y) || !dense_like_x(pp)) return MCB_STATUS_SHAPE_MISMATCH;
  if (rows == 0 || D == 0) return MCB_STATUS_OK;
  for (const mcb_tensor *t : {x, pp})
    if (overlaps(y, t)) return MCB_STATUS_ALIAS_VIOLATION;
  bool host = false;
  if ((s = same_space({x, y, pp}, &host))) return s;
  Call call(exec);
  if ((s = call.begin(host))) return s;
  void *dx, *dp, *dy;
  if ((s = call.device_ptr(x, true, &dx)) || (s = call.device_ptr(pp, true, &dp)) ||
      (s = call.device_ptr(y, false, &dy)))
    return s;
  LaunchInfo info;
  call.mark_compute_start();
  cudaError_t err = mcb::launch_residual_rmsnorm(dx, dp, dy, rows, D, eps, call.stream(), &info);
  call.mark_compute_end();
  if (err == cudaErrorNotSupported) return MCB_STATUS_UNAVAILABLE_VARIANT;
  info.tile_m = 1;
  info.tile_n = 256;
  info.ctas = static_cast<int>(std::min<int64_t>(rows, 0x7fffffff));
  info.set_route("residual_rmsnorm");
  return call.finish(y, dy, info, err);
}

// Two head groups on two GPUs, the exchange fused into the output projection
// (peer.cu holds the exchange object and the counter kernels). Step s of GPU
// g (both GPUs run the same steps):
//   projections and MSM of the group (local);
//   wait until the peer has consumed what this GPU wrote at step s-1;
//   GEMM of the peer's rows of O_g Wo_g, stored into the peer's receive
//   buffer by the epilogue (plain stores: no TMA touches the peer);
//   raise the peer's "data" counter to s;
//   GEMM of the own rows into scratch;
//   wait for this GPU's "data" counter to reach s;
//   Y = RMSNorm(X_own + P_own + P_received);
//   raise the peer's "consumed" counter to s.
// The waits on the other GPU's counters give up after ~2 s (clock64 cycles
// at ~1.9 GHz), as the pipeline waits of the GEMM kernels do.
constexpr long long kSpinTimeoutCyclesHost = 4000000000LL;

mcb_status attn_heads_pair_impl(const mcb_tensor *y, const mcb_tensor *x, const mcb_tensor *wq,
                                const mcb_tensor *wk, const mcb_tensor *wv, const mcb_tensor *wo,
                                int64_t heads, float eps, int32_t group, mcb_peer_exchange *xch,
                                const mcb_exec *exec) {
  mcb_status s;
  if ((s = check_tensor(x, 3, 3)) || (s = check_tensor(y, 2, 2)) || (s = check_tensor(wq, 2, 2)) ||
      (s = check_tensor(wk, 2, 2)) || (s = check_tensor(wv, 2, 2)) || (s = check_tensor(wo, 2, 2)))
    return s;
  for (const mcb_tensor *t : {x, y, wq, wk, wv, wo})
    if (t->dtype != MCB_DTYPE_BF16) return MCB_STATUS_UNSUPPORTED_DTYPE;
  if (!xch || !xch->local || !xch->remote || (group != 0 && group != 1))
    return MCB_STATUS_INVALID_ARGUMENT;
  if (!(eps >= 0.0f)) return MCB_STATUS_INVALID_ARGUMENT;
  const int64_t B = x->dims[0], S = x->dims[1], D = x->dims[2], Dh = wq->dims[1];
  if (heads <= 0 || Dh <= 0 || Dh % heads != 0) return MCB_STATUS_INVALID_ARGUMENT;
  const int64_t hd = Dh / heads, M = B * S;
  if (S == 0 || M % 2 != 0) return MCB_STATUS_INVALID_SHAPE;
  const int64_t R = M / 2;
  if (!(x->dims[0] == B && x->strides[2] == 1 && (S <= 1 || x->strides[1] == D) &&
        (B <= 1 || x->strides[0] == S * D)))
    return MCB_STATUS_SHAPE_MISMATCH;
  if (!dense2(y, R, D)) return MCB_STATUS_SHAPE_MISMATCH;
  for (const mcb_tensor *w : {wq, wk, wv})
    if (!dense2(w, D, Dh)) return MCB_STATUS_SHAPE_MISMATCH;
  if (!dense2(wo, Dh, D)) return MCB_STATUS_SHAPE_MISMATCH;
  if (static_cast<uint64_t>(R) * static_cast<uint64_t>(D) * 2 > xch->recv_bytes)
    return MCB_STATUS_INSUFFICIENT_WORKSPACE;
  for (const mcb_tensor *t : {x, wq, wk, wv, wo})
    if (overlaps(y, t)) return MCB_STATUS_ALIAS_VIOLATION;
  bool host = false;
  if ((s = same_space({x, y, wq, wk, wv, wo}, &host))) return s;
  if (host) return MCB_STATUS_UNSUPPORTED_MEMORY_SPACE;
  Call call(exec);
  if ((s = call.begin(host))) return s;
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev != xch->device) return MCB_STATUS_INVALID_ARGUMENT;
  void *dx, *dq, *dk, *dv, *dwo, *dy;
  if ((s = call.device_ptr(x, true, &dx)) || (s = call.device_ptr(wq, true, &dq)) ||
      (s = call.device_ptr(wk, true, &dk)) || (s = call.device_ptr(wv, true, &dv)) ||
      (s = call.device_ptr(wo, true, &dwo)) || (s = call.device_ptr(y, false, &dy)))
    return s;
  void *ws = nullptr;
  const uint64_t qkvo = attn_heads_workspace_bytes(M, Dh);
  const uint64_t pown = (static_cast<uint64_t>(R) * D * 2 + 255) / 256 * 256;
  if ((s = call.scratch(qkvo + pown, &ws))) return s;
  const uint64_t one = qkvo / 4;
  uint8_t *base = static_cast<uint8_t *>(ws);
  void *Q = base, *K = base + one, *V = base + 2 * one, *O = base + 3 * one, *P = base + qkvo;
  uint8_t *loc = static_cast<uint8_t *>(xch->local), *rem = static_cast<uint8_t *>(xch->remote);
  uint32_t *data_local = reinterpret_cast<uint32_t *>(loc);
  uint32_t *consumed_local = reinterpret_cast<uint32_t *>(loc + 128);
  uint32_t *data_remote = reinterpret_cast<uint32_t *>(rem);
  uint32_t *consumed_remote = reinterpret_cast<uint32_t *>(rem + 128);
  void *recv_local = loc + mcb_peer_exchange::kHeaderBytes;
  void *recv_remote = rem + mcb_peer_exchange::kHeaderBytes;

  LaunchInfo info, step;
  cudaError_t err = cudaSuccess;
  mcb::Epilogue none;
  auto gemm = [&](const void *a, const void *w, void *out, int64_t m, int64_t n, int64_t k,
                  int no_tma_store) {
    const bool tc = k % 8 == 0 && n % 8 == 0 &&
                    ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(w) |
                      reinterpret_cast<uintptr_t>(out)) & 15u) == 0;
    if (tc)
      return mcb::launch_gemm_tc_bf16(a, w, out, m, n, k, k, n, n, 0, 1, none, call.ctx()->status,
                                      call.sms(), call.stream(), &step, 0, nullptr, no_tma_store);
    return mcb::launch_gemm_simt(a, MCB_DTYPE_BF16, w, MCB_DTYPE_BF16, out, MCB_DTYPE_BF16, m, n,
                                 k, k, n, n, 0, none, call.stream(), &step);
  };
  const uint32_t st = ++xch->step;
  uint32_t *status = call.ctx()->status;
  call.mark_compute_start();
  int launches = 0;
  for (auto [w, out] : {std::pair<void *, void *>{dq, Q}, {dk, K}, {dv, V}}) {
    step.launches = 0;
    if ((err = gemm(dx, w, out, M, Dh, D, 0)) != cudaSuccess) break;
    launches += step.launches;
  }
  if (err == cudaSuccess) {
    mcb::MsmShape sh;
    sh.batch = B;
    sh.heads = heads;
    sh.m = sh.n = S;
    sh.dqk = sh.dv = hd;
    const int64_t stv[3] = {S * Dh, hd, Dh};
    for (int i = 0; i < 3; ++i) sh.q_s[i] = sh.k_s[i] = sh.v_s[i] = sh.o_s[i] = stv[i];
    const float scale = 1.0f / std::sqrt(static_cast<float>(hd));
    step.launches = 0;
    err = cudaErrorNotSupported;
    if ((hd == 64 || hd == 128) && Dh % 8 == 0)
      err = mcb::launch_msm_tc_bf16(Q, K, V, O, sh, scale, status, call.sms(), call.stream(), &step);
    if (err == cudaErrorNotSupported)
      err = hd <= 256 ? mcb::launch_msm_simt(Q, K, V, O, MCB_DTYPE_BF16, sh, scale, call.stream(),
                                             &step)
                      : cudaErrorNotSupported;
    launches += step.launches;
  }
  const int peer = 1 - group;
  const uint8_t *o_rows = static_cast<const uint8_t *>(O);
  if (err == cudaSuccess)
    err = mcb::launch_peer_wait(consumed_local, st - 1, kSpinTimeoutCyclesHost, status,
                                call.stream());
  if (err == cudaSuccess) {
    step.launches = 0;
    err = gemm(o_rows + static_cast<uint64_t>(peer) * R * Dh * 2, dwo, recv_remote, R, D, Dh, 1);
    launches += step.launches;
  }
  if (err == cudaSuccess) err = mcb::launch_peer_signal(data_remote, st, call.stream());
  if (err == cudaSuccess) {
    step.launches = 0;
    err = gemm(o_rows + static_cast<uint64_t>(group) * R * Dh * 2, dwo, P, R, D, Dh, 0);
    launches += step.launches;
  }
  if (err == cudaSuccess)
    err = mcb::launch_peer_wait(data_local, st, kSpinTimeoutCyclesHost, status, call.stream());
  if (err == cudaSuccess) {
    step.launches = 0;
    err = mcb::launch_residual_rmsnorm(static_cast<const uint8_t *>(dx) +
                                           static_cast<uint64_t>(group) * R * D * 2,
                                       P, dy, R, D, eps, call.stream(), &step, recv_local);
    launches += step.launches;
  }
  if (err == cudaSuccess) err = mcb::launch_peer_signal(consumed_remote, st, call.stream());
  launches += 4;  // the two waits and two signals
  call.mark_compute_end();
  if (err == cudaErrorNotSupported) return MCB_STATUS_UNAVAILABLE_VARIANT;
  info.launches = launches;
  info.tile_m = 128;
  info.tile_n = 256;
  info.ctas = call.sms();
  info.set_route("attn_block_heads_pair_p2p");
  return call.finish(y, dy, info, err);
}

// ---- device buffers ------------------------------------------------------------------------
std::mutex g_buf_mu;
std::unordered_map<uint64_t, mcb_buffer> g_bufs;  // ptr -> live handle
std::atomic<uint64_t> g_next_alloc_id{1};

bool live(const mcb_buffer &h) {
  auto it = g_bufs.find(h.ptr);
  return it != g_bufs.end() && it->second.alloc_id == h.alloc_id &&
         it->second.size_bytes == h.size_bytes && it->second.device == h.device;
}

}  // namespace

// =====================================================================================
extern "C" {

MCB_API uint32_t mcb_abi_version(void) noexcept { return MCB_ABI_VERSION_V1; }

MCB_API const char *mcb_status_message(mcb_status code) noexcept {
  switch (code) {
    case MCB_STATUS_OK: return "ok";
    case MCB_STATUS_INVALID_ARGUMENT: return "invalid argument";
    case MCB_STATUS_ABI_MISMATCH: return "ABI version or struct size mismatch";
    case MCB_STATUS_UNSUPPORTED_DTYPE: return "unsupported dtype";
    case MCB_STATUS_UNSUPPORTED_RANK: return "unsupported rank";
    case MCB_STATUS_INVALID_SHAPE: return "invalid shape";
    case MCB_STATUS_UNSUPPORTED_LAYOUT: return "unsupported layout (innermost stride must be 1)";
    case MCB_STATUS_UNSUPPORTED_MEMORY_SPACE: return "unsupported memory space";
    case MCB_STATUS_MIXED_MEMORY_SPACES: return "operands live in different memory spaces";
    case MCB_STATUS_OUTPUT_NOT_MUTABLE: return "output not mutable";
    case MCB_STATUS_SHAPE_MISMATCH: return "shape mismatch";
    case MCB_STATUS_ALIAS_VIOLATION: return "output overlaps an input";
    case MCB_STATUS_ARITHMETIC_OVERFLOW: return "extent overflow";
    case MCB_STATUS_INVALID_ALIGNMENT: return "invalid alignment";
    case MCB_STATUS_INSUFFICIENT_WORKSPACE: return "insufficient workspace";
    case MCB_STATUS_UNAVAILABLE_VARIANT: return "no kernel variant for this shape/dtype";
    case MCB_STATUS_ALLOCATION_FAILURE: return "device allocation failed";
    case MCB_STATUS_CANDIDATE_FAILURE: return "CUDA error during execution";
    case MCB_STATUS_CANDIDATE_UNAVAILABLE: return "no usable sm_100 GPU";
    case MCB_STATUS_DEVICE_TIMEOUT: return "a device-side wait timed out (see mcb_device_status)";
    case MCB_STATUS_STALE_HANDLE: return "stale or unknown device buffer handle";
    default: return "unknown status";
  }
}

MCB_API mcb_status mcb_device_status(int32_t device, uint32_t *word, int32_t clear) noexcept {
  if (!word) return MCB_STATUS_INVALID_ARGUMENT;
  mcb_exec ex{};
  ex.abi_version = MCB_ABI_VERSION_V1;
  ex.struct_size = sizeof(ex);
  ex.device = device;
  int dev;
  mcb_status s = resolve_device(&ex, &dev);
  if (s) return s;
  DeviceGuard g(dev);
  if (!g.ok) return MCB_STATUS_CANDIDATE_FAILURE;
  DeviceCtx *c;
  if ((s = init_ctx(dev, &c))) return s;
  if (rt_memcpy(word, c->status, 4, cudaMemcpyDeviceToHost) != cudaSuccess)
    return MCB_STATUS_CANDIDATE_FAILURE;
  if (clear && rt_memset(c->status, 0, 4) != cudaSuccess) return MCB_STATUS_CANDIDATE_FAILURE;
  if (clear && *word != 0 && !hooks()) {
    // A stream-K launch that aborted may have left ready flags raised.
    std::lock_guard<std::mutex> lock(c->sk_mu);
    if (c->sk.flags && cudaMemset(c->sk.flags, 0, static_cast<size_t>(c->sk.max_tiles) * 2 *
                                                  sizeof(int)) != cudaSuccess)
      return MCB_STATUS_CANDIDATE_FAILURE;
  }
  return MCB_STATUS_OK;
}

MCB_API mcb_status mcb_device_timeout_selftest_v1(int32_t device,
                                                  uint64_t spin_limit_cycles) noexcept {
  if (spin_limit_cycles < 10000 || spin_limit_cycles > 4000000000ull)
    return MCB_STATUS_INVALID_ARGUMENT;
  if (hooks()) return MCB_STATUS_CANDIDATE_UNAVAILABLE;
  mcb_exec ex{};
  ex.abi_version = MCB_ABI_VERSION_V1;
  ex.struct_size = sizeof(ex);
  ex.device = device;
  int dev;
  mcb_status s = resolve_device(&ex, &dev);
  if (s) return s;
  DeviceGuard g(dev);
  if (!g.ok) return MCB_STATUS_CANDIDATE_FAILURE;
  DeviceCtx *c;
  if ((s = init_ctx(dev, &c))) return s;
  // X 128x64, W 64x256 and Y 128x256 bf16 in one allocation (never read or
  // written by the stalled kernel, but its tensor maps must be valid).
  void *buf = nullptr;
  const size_t xb = 128 * 64 * 2, wb = 64 * 256 * 2, yb = 128 * 256 * 2;
  if (cudaMalloc(&buf, xb + wb + yb) != cudaSuccess) {
    cudaGetLastError();
    return MCB_STATUS_ALLOCATION_FAILURE;
  }
  uint8_t *base = static_cast<uint8_t *>(buf);
  cudaError_t err = mcb::launch_gemm_tc_stall_selftest(base, base + xb, base + xb + wb,
                                                       static_cast<long long>(spin_limit_cycles),
                                                       c->status, nullptr);
  if (err == cudaSuccess) err = cudaDeviceSynchronize();
  cudaFree(buf);
  if (err != cudaSuccess) {
    cudaGetLastError();
    return MCB_STATUS_CANDIDATE_FAILURE;
  }
  uint32_t word = 0;
  if (cudaMemcpy(&word, c->status, 4, cudaMemcpyDeviceToHost) != cudaSuccess)
    return MCB_STATUS_CANDIDATE_FAILURE;
  // The stalled wait must have been reported; the word stays set (sticky)
  // until the caller clears it with mcb_device_status.
  constexpr uint32_t kTimeoutFullBit = 1u;  // kErrTimeoutFull of the device status word
  return (word & kTimeoutFullBit) ? MCB_STATUS_DEVICE_TIMEOUT : MCB_STATUS_CANDIDATE_FAILURE;
}

MCB_API mcb_status mcb_device_peer_timeout_selftest_v1(int32_t device,
                                                       uint64_t spin_limit_cycles) noexcept {
  if (spin_limit_cycles < 10000 || spin_limit_cycles > 4000000000ull)
    return MCB_STATUS_INVALID_ARGUMENT;
  if (hooks()) return MCB_STATUS_CANDIDATE_UNAVAILABLE;
  mcb_exec ex{};
  ex.abi_version = MCB_ABI_VERSION_V1;
  ex.struct_size = sizeof(ex);
  ex.device = device;
  int dev;
  mcb_status s = resolve_device(&ex, &dev);
  if (s) return s;
  DeviceGuard g(dev);
  if (!g.ok) return MCB_STATUS_CANDIDATE_FAILURE;
  DeviceCtx *c;
  if ((s = init_ctx(dev, &c))) return s;
  // X 256x4096, W 4096x512, Y 256x512 bf16, the partial slots of four
  // clusters (two CTAs each) and four zeroed flags in one allocation.
  void *buf = nullptr;
  const size_t xb = 256 * 4096 * 2, wb = 4096 * 512 * 2, yb = 256 * 512 * 2;
  const size_t pb = 4 * 2 * static_cast<size_t>(mcb::kGemmStreamKSlotFloats) * 4, fb = 256;
  if (cudaMalloc(&buf, xb + wb + yb + pb + fb) != cudaSuccess) {
    cudaGetLastError();
    return MCB_STATUS_ALLOCATION_FAILURE;
  }
  uint8_t *base = static_cast<uint8_t *>(buf);
  int *flags = reinterpret_cast<int *>(base + xb + wb + yb + pb);
  cudaError_t err = cudaMemset(flags, 0, fb);
  if (err == cudaSuccess)
    err = mcb::launch_gemm_tc_peer_stall_selftest(
        base, base + xb, base + xb + wb, reinterpret_cast<float *>(base + xb + wb + yb), flags,
        static_cast<long long>(spin_limit_cycles), c->status, nullptr);
  if (err == cudaSuccess) err = cudaDeviceSynchronize();
  cudaFree(buf);
  if (err != cudaSuccess) {
    cudaGetLastError();
    return MCB_STATUS_CANDIDATE_FAILURE;
  }
  uint32_t word = 0;
  if (cudaMemcpy(&word, c->status, 4, cudaMemcpyDeviceToHost) != cudaSuccess)
    return MCB_STATUS_CANDIDATE_FAILURE;
  // The stalled wait must have been reported; the word stays set (sticky)
  // until the caller clears it with mcb_device_status.
  constexpr uint32_t kTimeoutPeerBit = 1u << 5;  // kErrTimeoutPeer of the device status word
  return (word & kTimeoutPeerBit) ? MCB_STATUS_DEVICE_TIMEOUT : MCB_STATUS_CANDIDATE_FAILURE;
}

MCB_API mcb_status mcb_test_set_runtime_hooks_v1(const mcb_runtime_hooks *h) noexcept {
  if (!h) {
    if (g_hooks_on.exchange(false, std::memory_order_acq_rel)) {
      // Forget the device state created under the table (its pointers came
      // from the stand-ins; nothing is freed through CUDA).
      for (DeviceCtx &c : g_dev) {
        std::lock_guard<std::mutex> lock(c.mu);
        c.ready = c.usable = false;
        c.status = nullptr;
        for (int i = 0; i < kStageSlots; ++i) {
          c.stage[i] = nullptr;
          c.stage_cap[i] = 0;
        }
      }
    }
    return MCB_STATUS_OK;
  }
  if (h->abi_version != MCB_ABI_VERSION_V1 || h->struct_size < sizeof(mcb_runtime_hooks))
    return MCB_STATUS_ABI_MISMATCH;
  if (!h->get_device_count || !h->get_device || !h->set_device || !h->device_info ||
      !h->malloc_device || !h->free_device || !h->memset_device || !h->memcpy_async ||
      !h->memcpy2d_async || !h->memcpy_sync || !h->stream_synchronize || !h->launch)
    return MCB_STATUS_INVALID_ARGUMENT;
  if (g_real_context.load(std::memory_order_acquire) || g_hooks_on.load()) return MCB_STATUS_INVALID_ARGUMENT;
  g_hook_table = *h;
  g_hooks_on.store(true, std::memory_order_release);
  return MCB_STATUS_OK;
}

MCB_API mcb_status mcb_candidate_available(int32_t device) noexcept {
  mcb_exec ex{};
  ex.abi_version = MCB_ABI_VERSION_V1;
  ex.struct_size = sizeof(ex);
  ex.device = device;
  int dev;
  mcb_status s = resolve_device(&ex, &dev);
  if (s) return s;
  DeviceCtx *c;
  return init_ctx(dev, &c);
}

MCB_API mcb_status mcb_strict_gemm_f32_v1(const mcb_tensor *c, const mcb_tensor *a,
                                          const mcb_tensor *b, const mcb_exec *exec) noexcept {
  try {
    return strict_gemm_impl(c, a, b, exec);
  } catch (...) {
    return MCB_STATUS_CANDIDATE_FAILURE;
  }
}

MCB_API mcb_status mcb_strict_fused_pair_f32_v1(const mcb_tensor *e, const mcb_tensor *a,
                                                const mcb_tensor *b, const mcb_tensor *d,
                                                const mcb_exec *exec) noexcept {
  try {
    return strict_pair_impl(e, a, b, d, exec);
  } catch (...) {
    return MCB_STATUS_CANDIDATE_FAILURE;
  }
}

MCB_API mcb_status mcb_gemm_epilogue_v1(const mcb_tensor *y, const mcb_tensor *x,
                                        const mcb_tensor *w, const mcb_tensor *bias,
                                        const mcb_epilogue *epilogue, uint32_t gemm_flags,
                                        const mcb_exec *exec) noexcept {
  try {
    return gemm_epilogue_impl(y, x, w, bias, epilogue, gemm_flags, exec);
  } catch (...) {
    return MCB_STATUS_CANDIDATE_FAILURE;
  }
}

MCB_API mcb_status mcb_gemm_epilogue_chain_v1(const mcb_tensor *y, const mcb_tensor *x,
                                              const mcb_tensor *w,
                                              const mcb_tensor *boundaries,
                                              uint32_t num_boundaries,
                                              const mcb_epilogue_op *ops, uint32_t num_ops,
                                              uint32_t gemm_flags,
                                              const mcb_exec *exec) noexcept {
  try {
    if (num_ops == 0 || !ops) return MCB_STATUS_INVALID_ARGUMENT;
    return gemm_epilogue_impl(y, x, w, nullptr, nullptr, gemm_flags, exec, boundaries,
                              num_boundaries, ops, num_ops);
  } catch (...) {
    return MCB_STATUS_CANDIDATE_FAILURE;
  }
}

MCB_API mcb_status mcb_gemm_i8_i32_v1(const mcb_tensor *c, const mcb_tensor *a,
                                      const mcb_tensor *b, const mcb_exec *exec) noexcept {
  try {
    return typed_gemm_impl(c, a, b, exec, true);
  } catch (...) {
    return MCB_STATUS_CANDIDATE_FAILURE;
  }
}

MCB_API mcb_status mcb_gemm_i8_i32_zp_v1(const mcb_tensor *c, const mcb_tensor *a,
                                         const mcb_tensor *b, int32_t a_zero_point,
                                         int32_t b_zero_point, const mcb_exec *exec) noexcept {
  try {
    return typed_gemm_impl(c, a, b, exec, true, a_zero_point, b_zero_point);
  } catch (...) {
    return MCB_STATUS_CANDIDATE_FAILURE;
  }
}

MCB_API mcb_status mcb_gemm_bf16_f32_fma_v1(const mcb_tensor *c, const mcb_tensor *a,
                                            const mcb_tensor *b, const mcb_exec *exec) noexcept {
  try {
    return typed_gemm_impl(c, a, b, exec, false);
  } catch (...) {
    return MCB_STATUS_CANDIDATE_FAILURE;
  }
}

MCB_API mcb_status mcb_gemm_chain_v1(const mcb_tensor *e, const mcb_tensor *a,
                                     const mcb_tensor *b, const mcb_tensor *boundary,
                                     const mcb_epilogue *glue, const mcb_tensor *w,
                                     const mcb_exec *exec) noexcept {
  try {
    return chain_impl(e, a, b, boundary, glue, w, exec);
  } catch (...) {
    return MCB_STATUS_CANDIDATE_FAILURE;
  }
}

MCB_API mcb_status mcb_msm_v1(const mcb_tensor *o, const mcb_tensor *q, const mcb_tensor *k,
                              const mcb_tensor *v, double scale, const mcb_exec *exec) noexcept {
  try {
    return msm_impl(o, q, k, v, scale, exec);
  } catch (...) {
    return MCB_STATUS_CANDIDATE_FAILURE;
  }
}

MCB_API int32_t mcb_fp8_is_legal_shape_v1(int64_t m, int64_t n, int64_t k) noexcept {
  // Shape rule of isLegalFp8WgmmaShapeImpl (src/fp8_wgmma.cpp:10-24).
  if (m <= 0 || n <= 0 || k <= 0) return 0;
  if (m % 64 != 0 || k % 32 != 0) return 0;
  if (n < 8 || n > 256 || n % 8 != 0) return 0;
  return 1;
}

MCB_API mcb_fp8_tile_config mcb_fp8_tile_config_v1(int64_t m, int64_t n, int64_t k) noexcept {
  // Tile policy of getFp8WgmmaTileConfig (src/fp8_wgmma.cpp:30-57,85-109).
  mcb_fp8_tile_config c{64, 128, 32, 0};
  if (m <= 0 || n <= 0 || k <= 0) return c;
  c.m_tile = (m >= 128 && m % 128 == 0) ? 128 : 64;
  if (n >= 128 && n % 128 == 0) {
    c.n_tile = 128;
  } else {
    int best = 0;
    for (int cand = 8; cand <= 256 && cand <= n; cand += 8)
      if (n % cand == 0) best = cand;
    if (best > 0) {
      c.n_tile = best;
    } else {
      const int64_t clamped = std::min<int64_t>(256, std::max<int64_t>(8, n));
      c.n_tile = static_cast<int32_t>((clamped + 7) / 8 * 8);
    }
  }
  c.k_tile = 32;
  c.use_tma = mcb_fp8_is_legal_shape_v1(m, n, k) && m * n * k >= int64_t{64} * 64 * 32;
  return c;
}

MCB_API mcb_status mcb_fp8_quantize_blockwise_v1(const mcb_tensor *q, const mcb_tensor *scales,
                                                 const mcb_tensor *x, int64_t block,
                                                 const mcb_exec *exec) noexcept {
  try {
    return fp8_quantize_impl(q, scales, x, block, exec);
  } catch (...) {
    return MCB_STATUS_CANDIDATE_FAILURE;
  }
}

MCB_API mcb_status mcb_gemm_fp8_blockscaled_v1(const mcb_tensor *c, const mcb_tensor *a,
                                               const mcb_tensor *sa, const mcb_tensor *bt,
                                               const mcb_tensor *sbt, int64_t block,
                                               const mcb_exec *exec) noexcept {
  try {
    return gemm_fp8_impl(c, a, sa, bt, sbt, block, exec);
  } catch (...) {
    return MCB_STATUS_CANDIDATE_FAILURE;
  }
}

MCB_API mcb_status mcb_block_attn_res_v1(const mcb_tensor *out, const mcb_tensor *blocks,
                                         const mcb_tensor *partial, const mcb_tensor *query,
                                         int64_t block_count, int32_t has_partial, float eps,
                                         const mcb_exec *exec) noexcept {
  try {
    return block_attn_res_impl(out, blocks, partial, query, block_count, has_partial, eps, exec);
  } catch (...) {
    return MCB_STATUS_CANDIDATE_FAILURE;
  }
}

MCB_API uint64_t mcb_attn_block_workspace_bytes_v1(int64_t batch, int64_t seq,
                                                   int64_t d_model) noexcept {
  if (batch < 0 || seq < 0 || d_model < 0) return 0;
  return attn_workspace_bytes(batch, seq, d_model);
}

MCB_API mcb_status mcb_attn_block_region_v1(const mcb_tensor *y, const mcb_tensor *x,
                                            const mcb_tensor *wq, const mcb_tensor *wk,
                                            const mcb_tensor *wv, const mcb_tensor *wo,
                                            int64_t heads, float eps,
                                            const mcb_exec *exec) noexcept {
  try {
    return attn_block_impl(y, x, wq, wk, wv, wo, heads, eps, exec);
  } catch (...) {
    return MCB_STATUS_CANDIDATE_FAILURE;
  }
}

MCB_API uint64_t mcb_attn_block_heads_workspace_bytes_v1(int64_t batch, int64_t seq,
                                                         int64_t d_heads) noexcept {
  if (batch < 0 || seq < 0 || d_heads < 0) return 0;
  return attn_heads_workspace_bytes(batch * seq, d_heads);
}

MCB_API mcb_status mcb_attn_block_heads_v1(const mcb_tensor *p, const mcb_tensor *x,
                                           const mcb_tensor *wq, const mcb_tensor *wk,
                                           const mcb_tensor *wv, const mcb_tensor *wo,
                                           int64_t heads, const mcb_exec *exec) noexcept {
  try {
    return attn_heads_impl(p, x, wq, wk, wv, wo, heads, exec);
  } catch (...) {
    return MCB_STATUS_CANDIDATE_FAILURE;
  }
}

MCB_API mcb_status mcb_residual_rmsnorm_v1(const mcb_tensor *y, const mcb_tensor *x,
                                           const mcb_tensor *p, float eps,
                                           const mcb_exec *exec) noexcept {
  try {
    return residual_rmsnorm_impl(y, x, p, eps, exec);
  } catch (...) {
    return MCB_STATUS_CANDIDATE_FAILURE;
  }
}

MCB_API mcb_status mcb_attn_block_heads_pair_v1(const mcb_tensor *y, const mcb_tensor *x,
                                                const mcb_tensor *wq, const mcb_tensor *wk,
                                                const mcb_tensor *wv, const mcb_tensor *wo,
                                                int64_t heads, float eps, int32_t group,
                                                mcb_peer_exchange *exchange,
                                                const mcb_exec *exec) noexcept {
  try {
    return attn_heads_pair_impl(y, x, wq, wk, wv, wo, heads, eps, group, exchange, exec);
  } catch (...) {
    return MCB_STATUS_CANDIDATE_FAILURE;
  }
}

MCB_API mcb_status mcb_shard_plan_v1(uint32_t kind, int64_t total, int64_t group, int64_t align,
                                     int32_t world, int32_t rank, mcb_shard *out) noexcept {
  if (!out || world <= 0 || rank < 0 || rank >= world || total < 0)
    return MCB_STATUS_INVALID_ARGUMENT;
  if (align <= 0) align = 1;
  *out = mcb_shard{0, 0, 0, 0};
  // Balanced split of `n` items in chunks of `a` (last chunk may be short):
  // rank r owns chunks [r*c/w, (r+1)*c/w).
  auto split = [](int64_t n, int64_t a, int32_t w, int32_t r, int64_t &b, int64_t &cnt) {
    const int64_t chunks = (n + a - 1) / a;
    const int64_t c0 = chunks * r / w, c1 = chunks * (r + 1) / w;
    b = std::min(n, c0 * a);
    cnt = std::min(n, c1 * a) - b;
  };
  switch (kind) {
    case MCB_SHARD_ROWS:
    case MCB_SHARD_UNITS:
      split(total, kind == MCB_SHARD_UNITS ? 1 : align, world, rank, out->begin, out->count);
      out->kv_begin = out->begin;
      out->kv_count = out->count;
      return MCB_STATUS_OK;
    case MCB_SHARD_TOKENS: {
      if (group <= 0 || total % group != 0) return MCB_STATUS_INVALID_SHAPE;
      const int64_t batches = total / group;
      if (world >= batches) {
        if (batches == 0 || world % batches != 0) return MCB_STATUS_INVALID_ARGUMENT;
        const int32_t per = static_cast<int32_t>(world / batches);
        const int64_t b = rank / per;
        int64_t tb, tc;
        split(group, align, per, rank % per, tb, tc);
        out->begin = b * group + tb;
        out->count = tc;
        out->kv_begin = b * group;
        out->kv_count = group;
      } else {
        if (batches % world != 0) return MCB_STATUS_INVALID_ARGUMENT;
        const int64_t per = batches / world;
        out->begin = out->kv_begin = rank * per * group;
        out->count = out->kv_count = per * group;
      }
      return MCB_STATUS_OK;
    }
    default:
      return MCB_STATUS_INVALID_ARGUMENT;
  }
}

MCB_API mcb_status mcb_device_alloc(int32_t device, uint64_t size_bytes, mcb_buffer *out) noexcept {
  if (!out) return MCB_STATUS_INVALID_ARGUMENT;
  mcb_exec ex{};
  ex.abi_version = MCB_ABI_VERSION_V1;
  ex.struct_size = sizeof(ex);
  ex.device = device;
  int dev;
  mcb_status s = resolve_device(&ex, &dev);
  if (s) return s;
  DeviceGuard g(dev);
  if (!g.ok) return MCB_STATUS_CANDIDATE_FAILURE;
  void *p = nullptr;
  if (cudaMalloc(&p, size_bytes ? size_bytes : 1) != cudaSuccess) {
    cudaGetLastError();
    return MCB_STATUS_ALLOCATION_FAILURE;
  }
  mcb_buffer h{};
  h.ptr = reinterpret_cast<uint64_t>(p);
  h.size_bytes = size_bytes;
  h.alloc_id = g_next_alloc_id.fetch_add(1);
  h.device = dev;
  try {
    std::lock_guard<std::mutex> lock(g_buf_mu);
    g_bufs[h.ptr] = h;
  } catch (...) {
    cudaFree(p);
    return MCB_STATUS_ALLOCATION_FAILURE;
  }
  *out = h;
  return MCB_STATUS_OK;
}

MCB_API mcb_status mcb_device_free(mcb_buffer handle) noexcept {
  std::lock_guard<std::mutex> lock(g_buf_mu);
  if (!live(handle)) return MCB_STATUS_STALE_HANDLE;
  DeviceGuard g(handle.device);
  g_bufs.erase(handle.ptr);
  return from_cuda(cudaFree(reinterpret_cast<void *>(handle.ptr)));
}

MCB_API int32_t mcb_device_is_valid(mcb_buffer handle) noexcept {
  std::lock_guard<std::mutex> lock(g_buf_mu);
  return live(handle) ? 1 : 0;
}

MCB_API mcb_status mcb_device_upload(mcb_buffer dst, const void *host_src,
                                     uint64_t size_bytes) noexcept {
  {
    std::lock_guard<std::mutex> lock(g_buf_mu);
    if (!live(dst)) return MCB_STATUS_STALE_HANDLE;
  }
  if (size_bytes > dst.size_bytes) return MCB_STATUS_ARITHMETIC_OVERFLOW;
  if (size_bytes && !host_src) return MCB_STATUS_INVALID_ARGUMENT;
  DeviceGuard g(dst.device);
  return from_cuda(cudaMemcpy(reinterpret_cast<void *>(dst.ptr), host_src, size_bytes,
                              cudaMemcpyHostToDevice));
}

MCB_API mcb_status mcb_device_download(void *host_dst, mcb_buffer src,
                                       uint64_t size_bytes) noexcept {
  {
    std::lock_guard<std::mutex> lock(g_buf_mu);
    if (!live(src)) return MCB_STATUS_STALE_HANDLE;
  }
  if (size_bytes > src.size_bytes) return MCB_STATUS_ARITHMETIC_OVERFLOW;
  if (size_bytes && !host_dst) return MCB_STATUS_INVALID_ARGUMENT;
  DeviceGuard g(src.device);
  return from_cuda(cudaMemcpy(host_dst, reinterpret_cast<void *>(src.ptr), size_bytes,
                              cudaMemcpyDeviceToHost));
}

// Stream-ordered forms: the copy is queued on `stream` (NULL = the legacy
// default stream) and the call returns at once; with pinned host memory the
// transfer overlaps other work on the device.
MCB_API mcb_status mcb_device_upload_async(mcb_buffer dst, const void *host_src,
                                           uint64_t size_bytes, void *stream) noexcept {
  {
    std::lock_guard<std::mutex> lock(g_buf_mu);
    if (!live(dst)) return MCB_STATUS_STALE_HANDLE;
  }
  if (size_bytes > dst.size_bytes) return MCB_STATUS_ARITHMETIC_OVERFLOW;
  if (size_bytes && !host_src) return MCB_STATUS_INVALID_ARGUMENT;
  DeviceGuard g(dst.device);
  return from_cuda(cudaMemcpyAsync(reinterpret_cast<void *>(dst.ptr), host_src, size_bytes,
                                   cudaMemcpyHostToDevice, static_cast<cudaStream_t>(stream)));
}

MCB_API mcb_status mcb_device_download_async(void *host_dst, mcb_buffer src, uint64_t size_bytes,
                                             void *stream) noexcept {
  {
    std::lock_guard<std::mutex> lock(g_buf_mu);
    if (!live(src)) return MCB_STATUS_STALE_HANDLE;
  }
  if (size_bytes > src.size_bytes) return MCB_STATUS_ARITHMETIC_OVERFLOW;
  if (size_bytes && !host_dst) return MCB_STATUS_INVALID_ARGUMENT;
  DeviceGuard g(src.device);
  return from_cuda(cudaMemcpyAsync(host_dst, reinterpret_cast<void *>(src.ptr), size_bytes,
                                   cudaMemcpyDeviceToHost, static_cast<cudaStream_t>(stream)));
}

MCB_API mcb_status mcb_device_zero(mcb_buffer handle) noexcept {
  {
    std::lock_guard<std::mutex> lock(g_buf_mu);
    if (!live(handle)) return MCB_STATUS_STALE_HANDLE;
  }
  DeviceGuard g(handle.device);
  return from_cuda(cudaMemset(reinterpret_cast<void *>(handle.ptr), 0, handle.size_bytes));
}

MCB_API mcb_status mcb_device_zero_raw_on_stream(void *device_ptr, uint64_t size_bytes,
                                                 void *stream) noexcept {
  if (size_bytes && !device_ptr) return MCB_STATUS_INVALID_ARGUMENT;
  return from_cuda(
      cudaMemsetAsync(device_ptr, 0, size_bytes, static_cast<cudaStream_t>(stream)));
}

}  // extern "C"

namespace mcb {
bool runtime_hooks_installed() { return hooks() != nullptr; }
}  // namespace mcb

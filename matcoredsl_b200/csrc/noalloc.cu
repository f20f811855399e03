// Allocation-free variant of the strict fused pair E = (A*B)*D.
//
// Who needs it: some callers cannot call cudaMalloc. A host framework that
// owns every byte of device memory through its own pool and forbids
// allocations behind its back is one. Another is code on a latency-critical
// path, where cudaMalloc's implicit device-wide synchronisation would stall
// other streams. A third is code that must not fail for lack of memory
// partway through a sequence of calls. mcb_strict_fused_pair_f32_v1 may
// allocate: its first use of a device creates a status word, it stages host
// operands, and it takes scratch for the intermediate panel when the panel
// does not fit in shared memory. This entry point computes the same
// bit-exact result but allocates nothing. Its intermediate panel lives in a
// fixed array compiled into this library (kStaticScratchFloats floats, 8 MiB,
// held on every GPU that loads the library until the process exits).
//
// Set-up: the first call on each device, with that device current, looks up
// the array's device address with cudaGetSymbolAddress (the array's name in
// host code is only a host-side stand-in) and the device's SM count. Make
// that first call before any stream capture.
//
// Sharing: every call uses the same array, and the array keeps whatever the
// last call left in it. Nothing needs clearing, because each panel row is
// fully written before it is read. Calls that overlap on the GPU (different
// streams, or different host threads, on the same device) race on the array
// and must be serialised by the caller.
#include <cuda_runtime.h>

#include <mutex>

#include "internal.h"
#include "mcb.h"

namespace {

constexpr int64_t kStaticScratchFloats = int64_t{1} << 21;  // 8 MiB per GPU

static __device__ __align__(256) float g_pair_panel_scratch[kStaticScratchFloats];

constexpr int kMaxDevices = 64;
struct StaticScratchDevice {
  std::once_flag once;
  cudaError_t setup_error = cudaSuccess;
  float *scratch = nullptr;  // device address of g_pair_panel_scratch
  int sms = 0;
  bool sm100 = false;
};
StaticScratchDevice g_static_dev[kMaxDevices];

// Runs with `dev` current.
void setup_device(StaticScratchDevice &s, int dev) {
  int major = 0, minor = 0;
  cudaError_t e = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&s.sms, cudaDevAttrMultiProcessorCount, dev);
  if (e == cudaSuccess) {
    void *ptr = nullptr;
    e = cudaGetSymbolAddress(&ptr, g_pair_panel_scratch);
    if (e == cudaSuccess) s.scratch = static_cast<float *>(ptr);
  }
  s.sm100 = major == 10 && minor == 0;
  s.setup_error = e;
}

bool dense_f32_device(const mcb_tensor *t) {
  return t && t->abi_version == MCB_ABI_VERSION_V1 && t->struct_size >= sizeof(mcb_tensor) &&
         t->rank == 2 && t->dtype == MCB_DTYPE_F32;
}

bool layout_ok(const mcb_tensor *t) {
  if (t->dims[0] < 0 || t->dims[1] < 0) return false;
  if (t->dims[0] == 0 || t->dims[1] == 0) return true;
  if (!t->data || t->strides[1] != 1) return false;
  if (t->dims[0] > 1 && t->strides[0] < t->dims[1]) return false;
  return reinterpret_cast<uintptr_t>(t->data) % alignof(float) == 0;
}

uint64_t span(const mcb_tensor *t) {
  if (t->dims[0] == 0 || t->dims[1] == 0) return 0;
  return static_cast<uint64_t>((t->dims[0] - 1) * t->strides[0] + t->dims[1]) * sizeof(float);
}

bool overlap(const mcb_tensor *x, const mcb_tensor *y) {
  const uint64_t sx = span(x), sy = span(y);
  if (!sx || !sy) return false;
  const uintptr_t x0 = reinterpret_cast<uintptr_t>(x->data), y0 = reinterpret_cast<uintptr_t>(y->data);
  return x0 < y0 + sy && y0 < x0 + sx;
}

}  // namespace

extern "C" MCB_API mcb_status mcb_strict_fused_pair_f32_noalloc_v1(
    const mcb_tensor *e, const mcb_tensor *a, const mcb_tensor *b, const mcb_tensor *d,
    const mcb_exec *exec) noexcept {
  if (!dense_f32_device(e) || !dense_f32_device(a) || !dense_f32_device(b) ||
      !dense_f32_device(d))
    return (e && a && b && d) ? MCB_STATUS_UNSUPPORTED_DTYPE : MCB_STATUS_INVALID_ARGUMENT;
  if (exec && (exec->abi_version != MCB_ABI_VERSION_V1 || exec->struct_size < sizeof(mcb_exec)))
    return MCB_STATUS_ABI_MISMATCH;
  if (exec && exec->report &&
      (exec->report->abi_version != MCB_ABI_VERSION_V1 ||
       exec->report->struct_size < sizeof(mcb_report)))
    return MCB_STATUS_ABI_MISMATCH;
  // Timing needs CUDA events, which this entry point does not create.
  if (exec && (exec->flags & MCB_EXEC_TIME)) return MCB_STATUS_INVALID_ARGUMENT;
  for (const mcb_tensor *t : {e, a, b, d}) {
    if (t->memory_space != MCB_MEMORY_CUDA_DEVICE) return MCB_STATUS_UNSUPPORTED_MEMORY_SPACE;
    if (!layout_ok(t)) return MCB_STATUS_UNSUPPORTED_LAYOUT;
  }
  const int64_t m = a->dims[0], k = a->dims[1], n = b->dims[1], p = d->dims[1];
  if (b->dims[0] != k || d->dims[0] != n || e->dims[0] != m || e->dims[1] != p)
    return MCB_STATUS_SHAPE_MISMATCH;
  if (overlap(e, a) || overlap(e, b) || overlap(e, d)) return MCB_STATUS_ALIAS_VIOLATION;
  // One panel row of N floats must fit in the fixed array.
  if (m > 0 && p > 0 && n > kStaticScratchFloats) return MCB_STATUS_INSUFFICIENT_WORKSPACE;
  if (mcb::runtime_hooks_installed()) return MCB_STATUS_CANDIDATE_UNAVAILABLE;

  int count = 0;
  if (cudaGetDeviceCount(&count) != cudaSuccess || count == 0) {
    cudaGetLastError();
    return MCB_STATUS_CANDIDATE_UNAVAILABLE;
  }
  int prev = -1;
  if (cudaGetDevice(&prev) != cudaSuccess) return MCB_STATUS_CANDIDATE_UNAVAILABLE;
  const int dev = (exec && exec->device >= 0) ? exec->device : prev;
  if (dev >= count || dev >= kMaxDevices) return MCB_STATUS_INVALID_ARGUMENT;
  const bool switched = dev != prev;
  if (switched && cudaSetDevice(dev) != cudaSuccess) return MCB_STATUS_CANDIDATE_FAILURE;
  struct Restore {
    bool on;
    int dev;
    ~Restore() {
      if (on) cudaSetDevice(dev);
    }
  } restore{switched, prev};

  StaticScratchDevice &s = g_static_dev[dev];
  std::call_once(s.once, [&] { setup_device(s, dev); });
  if (s.setup_error != cudaSuccess || !s.scratch) return MCB_STATUS_CANDIDATE_FAILURE;
  if (!s.sm100) return MCB_STATUS_CANDIDATE_UNAVAILABLE;

  cudaStream_t stream = exec ? static_cast<cudaStream_t>(exec->stream) : nullptr;
  mcb::LaunchInfo info;
  bool panel_too_large = false;
  // An error left unread by the caller's earlier runtime calls must not be
  // reported as this call's launch failure.
  cudaGetLastError();
  cudaError_t err = mcb::launch_strict_pair_fixed_scratch(
      static_cast<const float *>(a->data), static_cast<const float *>(b->data),
      static_cast<const float *>(d->data), static_cast<float *>(e->data), s.scratch,
      kStaticScratchFloats, m, k, n, p, k ? a->strides[0] : 0, n ? b->strides[0] : 0,
      p ? d->strides[0] : 0, e->strides[0], s.sms, stream, &info, &panel_too_large);
  if (panel_too_large) return MCB_STATUS_INSUFFICIENT_WORKSPACE;
  if (err == cudaSuccess && exec && (exec->flags & MCB_EXEC_SYNC))
    err = cudaStreamSynchronize(stream);
  if (exec && exec->report) {
    mcb_report *r = exec->report;
    for (size_t i = 0; i < sizeof(r->route); ++i) r->route[i] = info.route[i];
    r->kernel_launches = info.launches;
    r->tile_m = info.tile_m;
    r->tile_n = info.tile_n;
    r->tile_k = 0;
    r->stages = 0;
    r->ctas = info.ctas;
    r->kernel_ms = r->h2d_ms = r->d2h_ms = 0.0f;
    r->h2d_bytes = r->d2h_bytes = 0;
    r->device_status = 0;
  }
  return err == cudaSuccess ? MCB_STATUS_OK : MCB_STATUS_CANDIDATE_FAILURE;
}

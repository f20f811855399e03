// Pairwise exchange between the two GPUs of a head-sharded attention block
// (mcb_peer_exchange_*_v1; used by mcb_attn_block_heads_pair_v1 in api.cpp).
//
// Each GPU owns one allocation: two 32-bit step counters and a receive
// buffer. The other GPU's output-projection GEMM stores its share of this
// GPU's rows straight into the receive buffer over NVLink (plain stores from
// its epilogue, so the transfer overlaps its math tile by tile), then raises
// the "data" counter here; this GPU raises the peer's "consumed" counter once
// its residual + RMSNorm has read the buffer, before the peer may overwrite
// it. The allocation is shared through a CUDA IPC handle that the caller
// passes between the two processes. No kernel loads another GPU's memory
// with TMA: remote traffic is the GEMM's plain stores and the two counters.
// Every wait on a counter is one thread with a clock64 limit that records
// kErrTimeoutRemote and returns. The reference is single-GPU: none of this
// has a counterpart there.
#include <cuda_runtime.h>

#include <new>

#include "common.cuh"
#include "internal.h"
#include "mcb.h"

namespace mcb {
namespace {

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t *p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(uint32_t *p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__global__ void peer_wait_kernel(const uint32_t *flag, uint32_t target, long long limit,
                                 uint32_t *status) {
  const long long t0 = clock64();
  // Counters only grow; the signed difference keeps the test valid across
  // the 32-bit wrap.
  while (static_cast<int32_t>(ld_acquire_sys(flag) - target) < 0) {
    if (clock64() - t0 > limit) {
      atomicOr(status, kErrTimeoutRemote);
      return;
    }
    __nanosleep(128);
  }
}

__global__ void peer_signal_kernel(uint32_t *flag, uint32_t value) {
  __threadfence_system();
  st_release_sys(flag, value);
}

}  // namespace

cudaError_t launch_peer_wait(const uint32_t *flag, uint32_t target, long long limit,
                             uint32_t *status, cudaStream_t stream) {
  peer_wait_kernel<<<1, 1, 0, stream>>>(flag, target, limit, status);
  return cudaGetLastError();
}

cudaError_t launch_peer_signal(uint32_t *flag, uint32_t value, cudaStream_t stream) {
  peer_signal_kernel<<<1, 1, 0, stream>>>(flag, value);
  return cudaGetLastError();
}

}  // namespace mcb

namespace {

static_assert(sizeof(mcb_ipc_handle) == sizeof(cudaIpcMemHandle_t),
              "mcb_ipc_handle must hold a cudaIpcMemHandle_t");

// Restores the caller's current device on scope exit.
struct DeviceScope {
  int prev = -1;
  bool switched = false;
  explicit DeviceScope(int dev) {
    if (cudaGetDevice(&prev) == cudaSuccess && prev != dev) switched = cudaSetDevice(dev) == cudaSuccess;
  }
  ~DeviceScope() {
    if (switched) cudaSetDevice(prev);
  }
};

}  // namespace

extern "C" {

MCB_API mcb_status mcb_peer_exchange_create_v1(int32_t device, uint64_t recv_bytes,
                                               mcb_peer_exchange **out,
                                               mcb_ipc_handle *handle) noexcept {
  if (!out || !handle || device < 0 || recv_bytes == 0) return MCB_STATUS_INVALID_ARGUMENT;
  *out = nullptr;
  if (recv_bytes > (uint64_t{1} << 40)) return MCB_STATUS_ARITHMETIC_OVERFLOW;
  int count = 0;
  if (cudaGetDeviceCount(&count) != cudaSuccess || count == 0) {
    (void)cudaGetLastError();
    return MCB_STATUS_CANDIDATE_UNAVAILABLE;
  }
  if (device >= count) return MCB_STATUS_INVALID_ARGUMENT;
  mcb_peer_exchange *x = new (std::nothrow) mcb_peer_exchange{};
  if (!x) return MCB_STATUS_ALLOCATION_FAILURE;
  DeviceScope scope(device);
  void *mem = nullptr;
  cudaIpcMemHandle_t h;
  if (cudaMalloc(&mem, mcb_peer_exchange::kHeaderBytes + recv_bytes) != cudaSuccess) {
    (void)cudaGetLastError();
    delete x;
    return MCB_STATUS_ALLOCATION_FAILURE;
  }
  if (cudaMemset(mem, 0, mcb_peer_exchange::kHeaderBytes) != cudaSuccess ||
      cudaDeviceSynchronize() != cudaSuccess || cudaIpcGetMemHandle(&h, mem) != cudaSuccess) {
    (void)cudaGetLastError();
    cudaFree(mem);
    delete x;
    return MCB_STATUS_CANDIDATE_FAILURE;
  }
  memcpy(handle->internal, &h, sizeof(h));
  x->device = device;
  x->recv_bytes = recv_bytes;
  x->local = mem;
  *out = x;
  return MCB_STATUS_OK;
}

MCB_API mcb_status mcb_peer_exchange_connect_v1(mcb_peer_exchange *x,
                                                const mcb_ipc_handle *peer) noexcept {
  if (!x || !peer) return MCB_STATUS_INVALID_ARGUMENT;
  if (x->remote) return MCB_STATUS_INVALID_ARGUMENT;  // already connected
  cudaIpcMemHandle_t h;
  memcpy(&h, peer->internal, sizeof(h));
  DeviceScope scope(x->device);
  void *r = nullptr;
  if (cudaIpcOpenMemHandle(&r, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
    (void)cudaGetLastError();
    return MCB_STATUS_CANDIDATE_FAILURE;
  }
  x->remote = r;
  return MCB_STATUS_OK;
}

MCB_API mcb_status mcb_peer_exchange_destroy_v1(mcb_peer_exchange *x) noexcept {
  if (!x) return MCB_STATUS_OK;
  mcb_status s = MCB_STATUS_OK;
  {
    DeviceScope scope(x->device);
    if (cudaDeviceSynchronize() != cudaSuccess) s = MCB_STATUS_CANDIDATE_FAILURE;
    if (x->remote && cudaIpcCloseMemHandle(x->remote) != cudaSuccess)
      s = MCB_STATUS_CANDIDATE_FAILURE;
    if (x->local && cudaFree(x->local) != cudaSuccess) s = MCB_STATUS_CANDIDATE_FAILURE;
    (void)cudaGetLastError();
  }
  delete x;
  return s;
}

}  // extern "C"

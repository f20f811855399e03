// NCCL collectives for sharded runs (mcb_comm_*_v1, mcb_allgather_v1,
// mcb_reduce_scatter_v1).
//
// Row, unit and batch shards need no collective on their data path: each
// rank computes its own rows / units / tokens (mcb_shard_plan_v1). A caller
// that wants the whole output on every rank gathers the shards afterwards
// with one NCCL all-gather per output, over NVLink / NVSwitch. The one real
// exchange is the head-sharded attention block: each rank's
// mcb_attn_block_heads_v1 partial holds its heads' share of the output
// projection, and one reduce-scatter sums the partials of a batch group and
// leaves each rank its rows. The reference is single-GPU, so none of this
// has a counterpart there.
//
// NCCL is resolved at run time: the copy already loaded in the process (for
// example by PyTorch) is reused, else libnccl.so.2 is opened privately, so a
// process never holds two NCCL builds. Without NCCL these entry points
// return MCB_STATUS_CANDIDATE_UNAVAILABLE; nothing else in the library
// depends on it.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <cstring>
#include <mutex>
#include <new>

#include "mcb.h"

struct mcb_comm {
  ncclComm_t nccl;
  int32_t world, rank, device;
};

namespace {

struct NcclApi {
  decltype(&ncclGetUniqueId) get_unique_id = nullptr;
  decltype(&ncclCommInitRank) comm_init_rank = nullptr;
  decltype(&ncclCommDestroy) comm_destroy = nullptr;
  decltype(&ncclAllGather) all_gather = nullptr;
  decltype(&ncclReduceScatter) reduce_scatter = nullptr;
  bool ok = false;
};

const NcclApi &nccl_api() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    void *h = dlopen("libnccl.so.2", RTLD_LAZY | RTLD_NOLOAD);
    if (!h) h = dlopen("libnccl.so.2", RTLD_LAZY | RTLD_LOCAL);
    if (!h) return;
    api.get_unique_id = reinterpret_cast<decltype(&ncclGetUniqueId)>(dlsym(h, "ncclGetUniqueId"));
    api.comm_init_rank =
        reinterpret_cast<decltype(&ncclCommInitRank)>(dlsym(h, "ncclCommInitRank"));
    api.comm_destroy = reinterpret_cast<decltype(&ncclCommDestroy)>(dlsym(h, "ncclCommDestroy"));
    api.all_gather = reinterpret_cast<decltype(&ncclAllGather)>(dlsym(h, "ncclAllGather"));
    api.reduce_scatter =
        reinterpret_cast<decltype(&ncclReduceScatter)>(dlsym(h, "ncclReduceScatter"));
    api.ok = api.get_unique_id && api.comm_init_rank && api.comm_destroy && api.all_gather &&
             api.reduce_scatter;
  });
  return api;
}

static_assert(sizeof(mcb_comm_id) == sizeof(ncclUniqueId), "mcb_comm_id must hold an ncclUniqueId");

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

MCB_API mcb_status mcb_comm_unique_id_v1(mcb_comm_id *out) noexcept {
  if (!out) return MCB_STATUS_INVALID_ARGUMENT;
  const NcclApi &api = nccl_api();
  if (!api.ok) return MCB_STATUS_CANDIDATE_UNAVAILABLE;
  ncclUniqueId id;
  if (api.get_unique_id(&id) != ncclSuccess) return MCB_STATUS_CANDIDATE_FAILURE;
  std::memcpy(out->internal, id.internal, sizeof(id.internal));
  return MCB_STATUS_OK;
}

MCB_API mcb_status mcb_comm_init_v1(const mcb_comm_id *id, int32_t world, int32_t rank,
                                    int32_t device, mcb_comm **out) noexcept {
  if (!id || !out || world < 1 || rank < 0 || rank >= world || device < 0)
    return MCB_STATUS_INVALID_ARGUMENT;
  *out = nullptr;
  const NcclApi &api = nccl_api();
  if (!api.ok) return MCB_STATUS_CANDIDATE_UNAVAILABLE;
  int count = 0;
  if (cudaGetDeviceCount(&count) != cudaSuccess || device >= count) {
    (void)cudaGetLastError();
    return MCB_STATUS_INVALID_ARGUMENT;
  }
  mcb_comm *c = new (std::nothrow) mcb_comm{};
  if (!c) return MCB_STATUS_ALLOCATION_FAILURE;
  ncclUniqueId nid;
  std::memcpy(nid.internal, id->internal, sizeof(nid.internal));
  DeviceScope scope(device);
  if (api.comm_init_rank(&c->nccl, world, nid, rank) != ncclSuccess) {
    delete c;
    return MCB_STATUS_CANDIDATE_FAILURE;
  }
  c->world = world;
  c->rank = rank;
  c->device = device;
  *out = c;
  return MCB_STATUS_OK;
}

MCB_API mcb_status mcb_allgather_v1(mcb_comm *comm, const void *send, void *recv,
                                    uint64_t bytes_per_rank, void *stream) noexcept {
  if (!comm) return MCB_STATUS_INVALID_ARGUMENT;
  if (bytes_per_rank == 0) return MCB_STATUS_OK;
  if (!send || !recv) return MCB_STATUS_INVALID_ARGUMENT;
  const uintptr_t s0 = reinterpret_cast<uintptr_t>(send), r0 = reinterpret_cast<uintptr_t>(recv);
  const uint64_t total = bytes_per_rank * static_cast<uint64_t>(comm->world);
  if (total / static_cast<uint64_t>(comm->world) != bytes_per_rank)
    return MCB_STATUS_ARITHMETIC_OVERFLOW;
  // In place only as NCCL defines it: send is this rank's slot of recv.
  const uintptr_t own = r0 + bytes_per_rank * static_cast<uint64_t>(comm->rank);
  if (s0 != own && s0 < r0 + total && r0 < s0 + bytes_per_rank) return MCB_STATUS_ALIAS_VIOLATION;
  const NcclApi &api = nccl_api();
  if (!api.ok) return MCB_STATUS_CANDIDATE_UNAVAILABLE;
  DeviceScope scope(comm->device);
  return api.all_gather(send, recv, bytes_per_rank, ncclUint8, comm->nccl,
                        static_cast<cudaStream_t>(stream)) == ncclSuccess
             ? MCB_STATUS_OK
             : MCB_STATUS_CANDIDATE_FAILURE;
}

MCB_API mcb_status mcb_reduce_scatter_v1(mcb_comm *comm, const void *send, void *recv,
                                         uint64_t count_per_rank, int32_t dtype,
                                         void *stream) noexcept {
  if (!comm) return MCB_STATUS_INVALID_ARGUMENT;
  ncclDataType_t nt;
  uint64_t elem;
  switch (dtype) {
    case MCB_DTYPE_F32: nt = ncclFloat32; elem = 4; break;
    case MCB_DTYPE_BF16: nt = ncclBfloat16; elem = 2; break;
    default: return MCB_STATUS_UNSUPPORTED_DTYPE;
  }
  if (count_per_rank == 0) return MCB_STATUS_OK;
  if (!send || !recv) return MCB_STATUS_INVALID_ARGUMENT;
  const uint64_t world = static_cast<uint64_t>(comm->world);
  const uint64_t recv_bytes = count_per_rank * elem;
  if (recv_bytes / elem != count_per_rank || (recv_bytes * world) / world != recv_bytes)
    return MCB_STATUS_ARITHMETIC_OVERFLOW;
  const uint64_t send_bytes = recv_bytes * world;
  const uintptr_t s0 = reinterpret_cast<uintptr_t>(send), r0 = reinterpret_cast<uintptr_t>(recv);
  // In place only as NCCL defines it: recv is this rank's slot of send.
  const uintptr_t own = s0 + recv_bytes * static_cast<uint64_t>(comm->rank);
  if (r0 != own && r0 < s0 + send_bytes && s0 < r0 + recv_bytes) return MCB_STATUS_ALIAS_VIOLATION;
  const NcclApi &api = nccl_api();
  if (!api.ok) return MCB_STATUS_CANDIDATE_UNAVAILABLE;
  DeviceScope scope(comm->device);
  return api.reduce_scatter(send, recv, count_per_rank, nt, ncclSum, comm->nccl,
                            static_cast<cudaStream_t>(stream)) == ncclSuccess
             ? MCB_STATUS_OK
             : MCB_STATUS_CANDIDATE_FAILURE;
}

MCB_API mcb_status mcb_comm_destroy_v1(mcb_comm *comm) noexcept {
  if (!comm) return MCB_STATUS_OK;
  const NcclApi &api = nccl_api();
  mcb_status s = MCB_STATUS_OK;
  if (api.ok) {
    DeviceScope scope(comm->device);
    if (api.comm_destroy(comm->nccl) != ncclSuccess) s = MCB_STATUS_CANDIDATE_FAILURE;
  }
  delete comm;
  return s;
}

}  // extern "C"

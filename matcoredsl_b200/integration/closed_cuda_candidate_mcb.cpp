// Reference-side adapter: MatcoreDSL's closed-host CUDA candidate entry points
// implemented over this library's C ABI (include/mcb.h).
//
// A maintainer compiles this file into the reference's runtime in place of
// compiler/lib/runtime/closed_cuda_candidate_v1.cpp (it includes that file's
// own header, closed_cuda_candidate_v1.h, and nothing else of the
// reference) and links libmcb.so. It keeps the contract that header states
// (closed_cuda_candidate_v1.h:8-20; closed_cuda_candidate_v1.cpp:24-55,86-120):
//  - no library or driver call runs on the caller's thread: each entry point
//    runs its work on a fresh, joined worker thread whose FP environment is
//    reset to the default, so the caller's FP environment, errno and
//    thread-local driver state are untouched;
//  - E changes only after a fully successful run: inputs are copied into
//    adapter-owned host buffers, the library writes into an adapter-owned
//    output buffer, and E is written from it only when the call returned
//    MCB_STATUS_OK;
//  - a failure after which device work may still be pending (a CUDA error
//    or an expired device-side wait) poisons the adapter: that call's staging
//    is retained (never freed under possible device use) and every later
//    call fails with Code::candidate_failure without calling the library.
// Device work itself is the library's: strict f32 (separate multiply and
// add, increasing k, +0 seed, C rounded to binary32), bit-identical to the
// reference's strict leaf.
#include "closed_cuda_candidate_v1.h"

#include <atomic>
#include <cerrno>
#include <cfenv>
#include <cstdint>
#include <cstring>
#include <limits>
#include <memory>
#include <new>
#include <thread>
#include <vector>

#include "mcb.h"

#if defined(__FAST_MATH__)
#error "the strict adapter must not be compiled with fast math"
#endif

namespace matcore::mdslc::runtime::closed_host_v1::detail {
namespace {

std::atomic<bool> poisoned{false};

struct ErrnoRestore {
  int value = errno;
  ~ErrnoRestore() { errno = value; }
};

// Runs `work` on a fresh worker thread with the default FP environment.
template <typename Work>
Code isolated(Work &&work) noexcept {
  ErrnoRestore preserve;
  if (poisoned.load(std::memory_order_acquire)) return Code::candidate_failure;
  Code result = Code::candidate_failure;
  try {
    std::thread worker([&]() noexcept {
      if (std::fesetenv(FE_DFL_ENV) != 0) {
        result = Code::unsupported_fp_environment;
        return;
      }
      try {
        result = work();
      } catch (const std::bad_alloc &) {
        result = Code::allocation_failure;
      } catch (...) {
        result = Code::candidate_failure;
      }
    });
    worker.join();
  } catch (const std::bad_alloc &) {
    result = Code::allocation_failure;
  } catch (...) {
    result = Code::candidate_failure;
  }
  return result;
}

// Staging retained after an uncertain failure (see the file comment).
struct Staging {
  std::vector<float> a, b, d, e;
  Staging *next = nullptr;
};
std::atomic<Staging *> quarantine_head{nullptr};
void quarantine(std::unique_ptr<Staging> &staging) noexcept {
  poisoned.store(true, std::memory_order_release);
  Staging *kept = staging.release();
  kept->next = quarantine_head.load(std::memory_order_relaxed);
  while (!quarantine_head.compare_exchange_weak(kept->next, kept, std::memory_order_release,
                                                std::memory_order_relaxed)) {
  }
}

bool bytes(std::uint64_t rows, std::uint64_t columns, std::size_t &result) noexcept {
  constexpr auto limit =
      static_cast<std::uint64_t>(std::numeric_limits<std::int64_t>::max()) / sizeof(float);
  if (rows > limit || columns > limit || (rows && columns > limit / rows)) return false;
  result = static_cast<std::size_t>(rows * columns * sizeof(float));
  return true;
}

bool range(const void *pointer, std::size_t size, std::uintptr_t &begin,
           std::uintptr_t &end) noexcept {
  begin = reinterpret_cast<std::uintptr_t>(pointer);
  if (size && (!pointer || begin % alignof(float))) return false;
  if (begin > std::numeric_limits<std::uintptr_t>::max() - size) return false;
  end = begin + size;
  return true;
}

mcb_tensor host_matrix(const float *data, std::uint64_t rows, std::uint64_t columns) noexcept {
  mcb_tensor t{};
  t.abi_version = MCB_ABI_VERSION_V1;
  t.struct_size = sizeof(mcb_tensor);
  t.data = const_cast<float *>(data);
  t.dtype = MCB_DTYPE_F32;
  t.rank = 2;
  t.dims[0] = static_cast<int64_t>(rows);
  t.dims[1] = static_cast<int64_t>(columns);
  t.strides[0] = static_cast<int64_t>(columns);
  t.strides[1] = 1;
  t.memory_space = MCB_MEMORY_HOST;
  return t;
}

// mcb_status -> Code; `uncertain` is set when device work may still be pending.
Code map_status(mcb_status s, bool &uncertain) noexcept {
  uncertain = false;
  switch (s) {
    case MCB_STATUS_OK: return Code::ok;
    case MCB_STATUS_SHAPE_MISMATCH: return Code::shape_mismatch;
    case MCB_STATUS_ARITHMETIC_OVERFLOW: return Code::extent_overflow;
    case MCB_STATUS_ALIAS_VIOLATION: return Code::invalid_view;
    case MCB_STATUS_ALLOCATION_FAILURE: return Code::allocation_failure;
    case MCB_STATUS_CANDIDATE_UNAVAILABLE: return Code::candidate_unavailable;
    case MCB_STATUS_UNSUPPORTED_DTYPE:
    case MCB_STATUS_UNSUPPORTED_RANK:
    case MCB_STATUS_UNSUPPORTED_LAYOUT:
    case MCB_STATUS_UNSUPPORTED_MEMORY_SPACE:
    case MCB_STATUS_UNAVAILABLE_VARIANT:
    case MCB_STATUS_INSUFFICIENT_WORKSPACE: return Code::candidate_incompatible;
    case MCB_STATUS_DEVICE_TIMEOUT:
    case MCB_STATUS_CANDIDATE_FAILURE:
      uncertain = true;
      return Code::candidate_failure;
    default: return Code::candidate_failure;
  }
}

// Shared tail of both entry points: runs `call` on the staged operands and
// publishes E only on success.
template <typename Call>
Code run_staged(std::unique_ptr<Staging> &staging, CandidateOutput out, std::size_t out_bytes,
                Call &&call) {
  bool uncertain = false;
  const Code code = map_status(call(), uncertain);
  if (uncertain) {
    quarantine(staging);
    return code;
  }
  if (code == Code::ok && out_bytes) std::memcpy(out.data, staging->e.data(), out_bytes);
  return code;
}

}  // namespace

Code cudaCandidateAvailable() noexcept {
  if (poisoned.load(std::memory_order_acquire)) return Code::candidate_unavailable;
  return isolated([]() -> Code {
    bool uncertain = false;
    const Code c = map_status(mcb_candidate_available(-1), uncertain);
    return c == Code::candidate_failure ? Code::candidate_unavailable : c;
  });
}

// The kernels are compiled into libmcb.so: available when its C ABI matches.
Code cudaFusedPairImageAvailable() noexcept {
  return mcb_abi_version() == MCB_ABI_VERSION_V1 ? Code::ok : Code::candidate_unavailable;
}

Code cudaGemmCandidate(CandidateInput a, CandidateInput b, CandidateOutput c) noexcept {
  return isolated([&]() -> Code {
    std::size_t sa, sb, sc;
    if (!bytes(a.rows, a.columns, sa) || !bytes(b.rows, b.columns, sb) ||
        !bytes(c.rows, c.columns, sc))
      return Code::extent_overflow;
    if (a.columns != b.rows || c.rows != a.rows || c.columns != b.columns)
      return Code::shape_mismatch;
    std::uintptr_t ab, ae, bb, be, cb, ce;
    if (!range(a.data, sa, ab, ae) || !range(b.data, sb, bb, be) ||
        !range(c.data, sc, cb, ce) ||
        (sc && ((sa && cb < ae && ab < ce) || (sb && cb < be && bb < ce))))
      return Code::invalid_view;
    if (!sc) return Code::ok;
    auto staging = std::make_unique<Staging>();
    if (sa) staging->a.assign(a.data, a.data + sa / sizeof(float));
    if (sb) staging->b.assign(b.data, b.data + sb / sizeof(float));
    staging->e.resize(sc / sizeof(float));
    return run_staged(staging, c, sc, [&] {
      const mcb_tensor ta = host_matrix(staging->a.data(), a.rows, a.columns);
      const mcb_tensor tb = host_matrix(staging->b.data(), b.rows, b.columns);
      const mcb_tensor tc = host_matrix(staging->e.data(), c.rows, c.columns);
      return mcb_strict_gemm_f32_v1(&tc, &ta, &tb, nullptr);
    });
  });
}

Code cudaFusedPairCandidate(CandidateInput a, CandidateInput b, CandidateInput d,
                            CandidateOutput e) noexcept {
  return isolated([&]() -> Code {
    if (a.columns != b.rows || b.columns != d.rows || e.rows != a.rows || e.columns != d.columns)
      return Code::shape_mismatch;
    std::size_t sizes[4];
    if (!bytes(a.rows, a.columns, sizes[0]) || !bytes(b.rows, b.columns, sizes[1]) ||
        !bytes(d.rows, d.columns, sizes[2]) || !bytes(e.rows, e.columns, sizes[3]))
      return Code::extent_overflow;
    const void *pointers[4] = {a.data, b.data, d.data, e.data};
    std::uintptr_t begin[4], end[4];
    for (int i = 0; i < 4; ++i)
      if (!range(pointers[i], sizes[i], begin[i], end[i])) return Code::invalid_view;
    for (int i = 0; i < 3; ++i)
      if (sizes[3] && sizes[i] && begin[3] < end[i] && begin[i] < end[3])
        return Code::invalid_view;
    if (!sizes[3]) return Code::ok;
    // Nonempty E with N = 0 is the Session's positive-zero bypass, never a
    // device call (closed_cuda_candidate_v1.h:17-18).
    if (b.columns == 0) return Code::candidate_incompatible;
    auto staging = std::make_unique<Staging>();
    if (sizes[0]) staging->a.assign(a.data, a.data + sizes[0] / sizeof(float));
    if (sizes[1]) staging->b.assign(b.data, b.data + sizes[1] / sizeof(float));
    if (sizes[2]) staging->d.assign(d.data, d.data + sizes[2] / sizeof(float));
    staging->e.resize(sizes[3] / sizeof(float));
    return run_staged(staging, e, sizes[3], [&] {
      const mcb_tensor ta = host_matrix(staging->a.data(), a.rows, a.columns);
      const mcb_tensor tb = host_matrix(staging->b.data(), b.rows, b.columns);
      const mcb_tensor td = host_matrix(staging->d.data(), d.rows, d.columns);
      const mcb_tensor te = host_matrix(staging->e.data(), e.rows, e.columns);
      return mcb_strict_fused_pair_f32_v1(&te, &ta, &tb, &td, nullptr);
    });
  });
}

}  // namespace matcore::mdslc::runtime::closed_host_v1::detail

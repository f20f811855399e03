// CPU test of the reference-side adapter (matcoredsl_b200/integration/
// closed_cuda_candidate_mcb.cpp) linked against the real libmcb.so, with the
// library's CUDA runtime calls replaced by fakes through
// mcb_test_set_runtime_hooks_v1. Modelled on the reference's fake-driver test
// (compiler/tests/generated_gpu/cuda_adapter_test.cpp): every fake aborts if
// it runs on the caller's thread and clobbers errno and the FP environment of
// the thread it runs on; device memory is host memory; launches compute the
// strict product on the CPU.
//
//   adapter_fault_test count      no failure; prints the number of fake calls
//   adapter_fault_test <n>        the n-th fake call fails
//   adapter_fault_test timeout    the launch reports an expired device wait
//   adapter_fault_test gemm       the isolated strict GEMM entry point
//   adapter_fault_test zero-N     nonempty E with N = 0 (no library call)
//   adapter_fault_test real       no fakes: availability on this machine
//
// Exit code 0 and a PASS line when every check holds.
#include <cerrno>
#include <cfenv>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <thread>
#include <vector>

#include "closed_cuda_candidate_v1.h"
#include "mcb.h"

namespace detail = matcore::mdslc::runtime::closed_host_v1::detail;
using matcore::mdslc::runtime::closed_host_v1::Code;

namespace {
std::thread::id caller;
unsigned calls = 0, fail_at = 0;
bool device_timeout = false;
void *status_word = nullptr;  // the library's 4-byte device status allocation
std::vector<void *> allocations;

// Runs first in every fake: the caller's thread must never get here.
int32_t enter(int32_t failure = 999) {
  if (std::this_thread::get_id() == caller) std::abort();
  errno = EDOM;
  std::fesetround(FE_UPWARD);
  std::feraiseexcept(FE_INVALID);
  ++calls;
  return calls == fail_at ? failure : 0;
}

int32_t get_device_count(int32_t *n) {
  if (int32_t e = enter()) return e;
  *n = 1;
  return 0;
}
int32_t get_device(int32_t *d) {
  if (int32_t e = enter()) return e;
  *d = 0;
  return 0;
}
int32_t set_device(int32_t d) {
  if (int32_t e = enter()) return e;
  return d == 0 ? 0 : 101;  // cudaErrorInvalidDevice
}
int32_t device_info(int32_t, int32_t *major, int32_t *minor, int32_t *sms, int32_t *smem) {
  if (int32_t e = enter()) return e;
  *major = 10;
  *minor = 0;
  *sms = 148;
  *smem = 227 * 1024;
  return 0;
}
int32_t malloc_device(void **p, uint64_t bytes) {
  if (int32_t e = enter(2)) return e;  // cudaErrorMemoryAllocation
  *p = std::malloc(bytes ? bytes : 1);
  if (!*p) return 2;
  std::memset(*p, 0xA5, bytes);  // never read as a result
  if (bytes == 4 && !status_word) status_word = *p;
  allocations.push_back(*p);
  return 0;
}
int32_t free_device(void *p) {
  if (int32_t e = enter()) return e;
  for (auto &a : allocations)
    if (a == p) {
      std::free(a);
      a = nullptr;
      return 0;
    }
  std::abort();  // never allocated here
}
int32_t memset_device(void *p, int32_t v, uint64_t bytes) {
  if (int32_t e = enter()) return e;
  std::memset(p, v, bytes);
  return 0;
}
int32_t memcpy_async(void *d, const void *s, uint64_t bytes, int32_t, void *) {
  if (int32_t e = enter()) return e;
  std::memcpy(d, s, bytes);
  return 0;
}
int32_t memcpy2d_async(void *d, uint64_t dp, const void *s, uint64_t sp, uint64_t w, uint64_t rows,
                       int32_t, void *) {
  if (int32_t e = enter()) return e;
  for (uint64_t r = 0; r < rows; ++r)
    std::memcpy(static_cast<char *>(d) + r * dp, static_cast<const char *>(s) + r * sp, w);
  return 0;
}
int32_t memcpy_sync(void *d, const void *s, uint64_t bytes, int32_t) {
  if (int32_t e = enter()) return e;
  std::memcpy(d, s, bytes);
  return 0;
}
int32_t stream_synchronize(void *) { return enter(); }

// Strict f32: separate multiply and add in increasing k from +0 (the test is
// compiled with -ffp-contract=off).
void strict(const float *a, const float *b, float *c, int64_t m, int64_t k, int64_t n,
            int64_t lda, int64_t ldb, int64_t ldc) {
  for (int64_t i = 0; i < m; ++i)
    for (int64_t j = 0; j < n; ++j) {
      float sum = 0.0f;
      for (int64_t r = 0; r < k; ++r) {
        const float prod = a[i * lda + r] * b[r * ldb + j];
        sum = sum + prod;
      }
      c[i * ldc + j] = sum;
    }
}
int32_t launch(const mcb_hook_launch *l) {
  if (int32_t e = enter()) return e;
  const auto *a = static_cast<const float *>(l->in[0]);
  const auto *b = static_cast<const float *>(l->in[1]);
  if (std::strcmp(l->op, "strict_gemm") == 0) {
    strict(a, b, static_cast<float *>(l->out), l->m, l->k, l->n, l->ld[0], l->ld[1], l->ld[3]);
  } else if (std::strcmp(l->op, "strict_fused_pair") == 0) {
    std::vector<float> c(static_cast<size_t>(l->m * l->n));
    strict(a, b, c.data(), l->m, l->k, l->n, l->ld[0], l->ld[1], l->n);
    strict(c.data(), static_cast<const float *>(l->in[2]), static_cast<float *>(l->out), l->m,
           l->n, l->p, l->n, l->ld[2], l->ld[3]);
  } else {
    std::abort();
  }
  if (device_timeout && status_word) *static_cast<uint32_t *>(status_word) = 1u;
  return 0;
}

bool caller_state_intact() {
  return errno == EBUSY && std::fegetround() == FE_DOWNWARD &&
         std::fetestexcept(FE_ALL_EXCEPT) == FE_DIVBYZERO;
}
}  // namespace

int main(int argc, char **argv) {
  caller = std::this_thread::get_id();
  const std::string mode = argc == 2 ? argv[1] : "count";
  std::fesetround(FE_DOWNWARD);
  std::feclearexcept(FE_ALL_EXCEPT);
  std::feraiseexcept(FE_DIVBYZERO);
  errno = EBUSY;

  if (mode == "real") {  // no fakes: this machine has no sm_100 GPU
    const Code c = detail::cudaCandidateAvailable();
    if (!caller_state_intact()) return 1;
    if (detail::cudaFusedPairImageAvailable() != Code::ok) return 2;
    std::printf("PASS real availability=%d\n", static_cast<int>(c));
    return 0;
  }

  mcb_runtime_hooks h{};
  h.abi_version = MCB_ABI_VERSION_V1;
  h.struct_size = sizeof(h);
  h.get_device_count = get_device_count;
  h.get_device = get_device;
  h.set_device = set_device;
  h.device_info = device_info;
  h.malloc_device = malloc_device;
  h.free_device = free_device;
  h.memset_device = memset_device;
  h.memcpy_async = memcpy_async;
  h.memcpy2d_async = memcpy2d_async;
  h.memcpy_sync = memcpy_sync;
  h.stream_synchronize = stream_synchronize;
  h.launch = launch;
  if (mcb_test_set_runtime_hooks_v1(&h) != MCB_STATUS_OK) return 10;

  if (mode == "timeout") device_timeout = true;
  else if (mode != "count" && mode != "gemm" && mode != "zero-N")
    fail_at = static_cast<unsigned>(std::strtoul(mode.c_str(), nullptr, 10));

  // E = (A B) D with A = 1 (2x3), B = 2 (3x4), D = 3 (4x4): every E is 72;
  // the GEMM C = A B is 6 everywhere.
  std::vector<float> a(6, 1.0f), b(12, 2.0f), d(16, 3.0f), out(8, 9876.0f);
  const bool zero_n = mode == "zero-N";
  Code result;
  float correct;
  if (mode == "gemm") {
    result = detail::cudaGemmCandidate({a.data(), 2, 3}, {b.data(), 3, 4}, {out.data(), 2, 4});
    correct = 6.0f;
  } else {
    result = detail::cudaFusedPairCandidate({a.data(), 2, 3}, {b.data(), 3, zero_n ? 0u : 4u},
                                            {d.data(), zero_n ? 0u : 4u, 4}, {out.data(), 2, 4});
    correct = 72.0f;
  }
  if (!caller_state_intact()) return 1;
  const bool fault = fail_at || device_timeout || zero_n;
  if ((result == Code::ok) == fault) return 2;
  for (float v : out)
    if (v != (fault ? 9876.0f : correct)) return 3;  // E untouched on failure
  if (zero_n && (result != Code::candidate_incompatible || calls != 0)) return 4;

  // After a failure: a candidate failure (possibly pending device work)
  // poisons the adapter, which then makes no library call at all; any other
  // failure leaves it usable, and the same call then succeeds.
  const unsigned before = calls;
  fail_at = 0;
  device_timeout = false;
  if (status_word) *static_cast<uint32_t *>(status_word) = 0u;
  const Code again = detail::cudaFusedPairCandidate({a.data(), 2, 3}, {b.data(), 3, 4},
                                                    {d.data(), 4, 4}, {out.data(), 2, 4});
  if (!caller_state_intact()) return 5;
  if (result == Code::candidate_failure) {
    if (again != Code::candidate_failure || calls != before) return 6;
    if (detail::cudaCandidateAvailable() == Code::ok || calls != before) return 7;
    for (float v : out)
      if (v != 9876.0f) return 8;
  } else {
    if (again != Code::ok) return 9;
    for (float v : out)
      if (v != 72.0f) return 11;
  }
  std::printf("PASS adapter mode=%s code=%d calls=%u\n", mode.c_str(), static_cast<int>(result),
              before);
  return 0;
}

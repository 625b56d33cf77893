// Library-wide C ABI pieces: version and the thread-local error message.
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>

#include "kve_common.cuh"
#include "tma.cuh"

namespace kve {

static thread_local char g_last_error[512] = "";

int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

static std::atomic<unsigned long long> g_launches{0};

void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

bool pdl_enabled() {
  static const bool on = [] {
    const char* v = getenv("KVE_PDL");
    return !(v && v[0] == '0');
  }();
  return on;
}

}  // namespace kve

extern "C" int kve_version(void) { return 1; }

extern "C" unsigned long long kve_launch_count(void) { return kve::g_launches.load(std::memory_order_relaxed); }

extern "C" const char* kve_last_error(void) { return kve::g_last_error; }

namespace kve {
namespace {

// One thread waits on a shared-memory mbarrier that nothing arrives at, through the
// same bounded wait every pipeline of this library uses, with its limit cut short.
__global__ void selftest_mbar_timeout_kernel(int* status, uint64_t limit_ns) {
  __shared__ __align__(8) uint64_t bar;
  mbar_init(smem_u32(&bar), 1);
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  mbar_wait(smem_u32(&bar), 0, status, limit_ns);
}

}  // namespace
}  // namespace kve

extern "C" int kve_selftest_mbar_timeout(int* dev_status, int64_t limit_ns, cudaStream_t stream) {
  using namespace kve;
  if (!dev_status || limit_ns < 0 || limit_ns > (int64_t)kWaitLimitNs)
    return set_error(KVE_ERR_ARG, "kve_selftest_mbar_timeout: dev_status required, 0 <= limit_ns <= %llu",
                     (unsigned long long)kWaitLimitNs);
  selftest_mbar_timeout_kernel<<<1, 1, 0, stream>>>(dev_status, (uint64_t)limit_ns);
  count_launch();
  return check_launch("kve_selftest_mbar_timeout");
}

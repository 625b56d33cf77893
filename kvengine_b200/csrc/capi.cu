// Library-wide C ABI pieces: version and the thread-local error message.
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>

#include "kve_common.cuh"

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

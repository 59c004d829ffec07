// api.cu -- error reporting and version of the C ABI.
#include <atomic>
#include <string>

#include "common.cuh"

namespace vmlx {

static thread_local std::string g_last_error;

int set_error(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

void clear_error() { g_last_error.clear(); }

static std::atomic<int> g_overlap{0};
bool launch_overlap() { return g_overlap.load(std::memory_order_relaxed) != 0; }

}  // namespace vmlx

extern "C" const char* vmlx_last_error(void) { return vmlx::g_last_error.c_str(); }

extern "C" int vmlx_version(void) { return 100; }

extern "C" int vmlx_set_launch_overlap(int enable) {
  int prev = vmlx::g_overlap.exchange(enable ? 1 : 0);
  return prev;
}

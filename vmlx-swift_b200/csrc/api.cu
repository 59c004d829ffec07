// api.cu -- error reporting and version of the C ABI.
#include <atomic>
#include <mutex>
#include <string>
#include <utility>
#include <vector>

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

// cudaFuncSetAttribute applies to the current device only, so a process that drives
// several GPUs must raise a kernel's dynamic shared-memory limit once per (kernel,
// device).  The table is small (one entry per kernel instance and device) and guarded
// by a mutex because host threads may drive different GPUs concurrently.
int ensure_max_dynamic_smem(const void* func, int bytes) {
  static std::mutex mu;
  static std::vector<std::pair<std::pair<const void*, int>, int>> done;  // ((func, device), bytes)
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return check_cuda(e, "cudaGetDevice");
  std::lock_guard<std::mutex> lock(mu);
  for (auto& d : done)
    if (d.first.first == func && d.first.second == dev && d.second >= bytes) return VMLX_OK;
  e = cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) return check_cuda(e, "cudaFuncSetAttribute(MaxDynamicSharedMemorySize)");
  for (auto& d : done)
    if (d.first.first == func && d.first.second == dev) { d.second = bytes; return VMLX_OK; }
  done.push_back({{func, dev}, bytes});
  return VMLX_OK;
}

// SM count of the current device (cached per device).
int sm_count() {
  static std::atomic<int> cache[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0) dev = 0;
  if (dev >= 64) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    return n > 0 ? n : 148;
  }
  int n = cache[dev].load(std::memory_order_relaxed);
  if (n > 0) return n;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
  cache[dev].store(n, std::memory_order_relaxed);
  return n;
}

static std::atomic<int> g_overlap{0};
bool launch_overlap() { return g_overlap.load(std::memory_order_relaxed) != 0; }

}  // namespace vmlx

extern "C" const char* vmlx_last_error(void) { return vmlx::g_last_error.c_str(); }

extern "C" int vmlx_version(void) { return 100; }

extern "C" int vmlx_set_launch_overlap(int enable) {
  int prev = vmlx::g_overlap.exchange(enable ? 1 : 0);
  return prev;
}

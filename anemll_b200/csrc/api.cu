// Error reporting shared by all entry points of the C ABI, and the count of kernel launches.
#include <atomic>

#include "common.cuh"

namespace anemll {

static thread_local char g_last_error[512] = "";
static std::atomic<long long> g_launches{0};

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
}

int launch_status(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("%s: CUDA error %d (%s)", what, (int)e, cudaGetErrorString(e));
    return (int)e;
  }
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return ANEMLL_OK;
}

}  // namespace anemll

extern "C" const char* anemll_last_error(void) { return anemll::g_last_error; }

extern "C" int anemll_version(void) { return 1; }

extern "C" long long anemll_launch_count(void) { return anemll::g_launches.load(std::memory_order_relaxed); }

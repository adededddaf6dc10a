// Error reporting shared by all entry points of the C ABI.
#include "common.cuh"

namespace anemll {

static thread_local char g_last_error[512] = "";

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
  return ANEMLL_OK;
}

}  // namespace anemll

extern "C" const char* anemll_last_error(void) { return anemll::g_last_error; }

extern "C" int anemll_version(void) { return 1; }

// Library-level entry points: version, error reporting, device queries,
// launch flags.
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>

#include "common.cuh"
#include "launch.cuh"

namespace jsx {

static thread_local char g_error[1024] = "";
static int g_launch_flags = -1;

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_error, sizeof(g_error), fmt, ap);
  va_end(ap);
}

int cuda_status(cudaError_t e, const char* what) {
  set_error("%s failed: %s (%d)", what, cudaGetErrorString(e), (int)e);
  return JSX_ECUDA;
}

int sm_count() {
  static int cache[128] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 128) return 1;
  if (cache[dev] == 0) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cache[dev] = n > 0 ? n : 1;
  }
  return cache[dev];
}

int launch_flags() {
  if (g_launch_flags < 0) {
    const char* env = getenv("JSX_PDL");
    g_launch_flags = (env && env[0] == '0') ? 0 : JSX_LAUNCH_PDL;
  }
  return g_launch_flags;
}

}  // namespace jsx

using namespace jsx;

extern "C" int jsx_abi_version(void) { return 1; }

extern "C" const char* jsx_last_error(void) { return g_error; }

extern "C" int jsx_device_sm_count(int* out) {
  JSX_REQUIRE(out != nullptr, "null out");
  int dev = 0;
  JSX_CUDA(cudaGetDevice(&dev));
  JSX_CUDA(cudaDeviceGetAttribute(out, cudaDevAttrMultiProcessorCount, dev));
  return JSX_OK;
}

extern "C" int jsx_set_launch_flags(int flags) {
  JSX_REQUIRE((flags & ~JSX_LAUNCH_PDL) == 0, "unknown launch flags 0x%x", flags);
  g_launch_flags = flags;
  return JSX_OK;
}

extern "C" int jsx_get_launch_flags(void) { return launch_flags(); }

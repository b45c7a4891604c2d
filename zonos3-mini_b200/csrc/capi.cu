// Library-wide C ABI: error reporting and version.
#include <stdarg.h>
#include <stdio.h>

#include "common.cuh"

namespace {
thread_local char g_last_error[1024] = "";
}

namespace zb {

int fail(int code, const char* fmt, ...) {
  va_list args;
  va_start(args, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, args);
  va_end(args);
  return code;
}

int check_launch(const char* what) {
  cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) return fail(kCudaError, "%s: launch failed: %s", what, cudaGetErrorString(err));
  return kOk;
}

int sm_count() {
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (cached[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cached[dev] = n;
  }
  return cached[dev];
}

}  // namespace zb

ZB_API const char* zb_last_error(void) { return g_last_error; }

ZB_API void zb_clear_error(void) { g_last_error[0] = '\0'; }

ZB_API int zb_version(void) { return 1; }

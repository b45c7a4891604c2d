// Library-wide C ABI: error reporting and version.
#include <stdarg.h>
#include <stdio.h>

#include "common.cuh"

namespace {
thread_local char g_last_error[1024] = "";
}

// Library status word (one per device): bits set by kernels whose bounded waits expired.
__device__ unsigned g_zb_device_status;

namespace zb {

std::atomic<uint64_t> g_launch_count{0};

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

unsigned* device_status_ptr() {
  static unsigned* cached[64] = {nullptr};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  if (cached[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_zb_device_status) != cudaSuccess) return nullptr;
    cached[dev] = static_cast<unsigned*>(p);
  }
  return cached[dev];
}

}  // namespace zb

// Reads (and with clear != 0 resets) the current device's status word. Synchronous; for diagnostics and tests.
ZB_API int zb_device_status(unsigned* flags, int clear) {
  ZB_REQUIRE(flags != nullptr, "zb_device_status: flags is null");
  unsigned* p = zb::device_status_ptr();
  if (p == nullptr) return zb::fail(zb::kCudaError, "zb_device_status: status word unavailable");
  ZB_CUDA(cudaMemcpy(flags, p, sizeof(unsigned), cudaMemcpyDeviceToHost));
  if (clear) ZB_CUDA(cudaMemset(p, 0, sizeof(unsigned)));
  return zb::kOk;
}

ZB_API const char* zb_last_error(void) { return g_last_error; }

ZB_API void zb_clear_error(void) { g_last_error[0] = '\0'; }

ZB_API int zb_version(void) { return 2; }

ZB_API uint64_t zb_launch_count(void) { return zb::g_launch_count.load(std::memory_order_relaxed); }

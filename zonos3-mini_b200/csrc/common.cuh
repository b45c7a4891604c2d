// Shared helpers of the zonos3-mini B200 kernels: status codes, the per-thread error string behind
// zb_last_error(), argument checks and small device utilities.
//
// Error convention: every extern "C" entry point returns an int status (0 = success) and never lets a C++
// exception cross the ABI. A failed check records a message that zb_last_error() returns on the calling
// host thread, the way the reference's RuntimeCheck/panic records one before raising PanicError
// (servers/sgl/src/zonos3_sgl/kernel/csrc/include/zonos3/utils.h:54-88).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

// Exported C-ABI symbol (the library builds with -fvisibility=hidden).
#define ZB_API extern "C" __attribute__((visibility("default")))

namespace zb {

enum Status : int {
  kOk = 0,
  kInvalidArgument = 1,  // shape, dtype, pointer or alignment rejected before any launch
  kCudaError = 2,        // a CUDA runtime call or launch failed
  kUnsupported = 3,      // a size outside what the kernels are built for
  kDeviceTimeout = 4,    // a bounded device-side wait gave up (the kernel returned early)
};

// Records a printf-style message for zb_last_error() and returns `code`.
int fail(int code, const char* fmt, ...);

// Checks cudaGetLastError() after a launch; records `what` with the CUDA error string on failure.
int check_launch(const char* what);

// Number of SMs of the current device (cached per device).
int sm_count();

}  // namespace zb

#define ZB_REQUIRE(cond, ...)                                   \
  do {                                                          \
    if (!(cond)) return zb::fail(zb::kInvalidArgument, __VA_ARGS__); \
  } while (0)

#define ZB_REQUIRE_ALIGNED(ptr, bytes, name)                                              \
  ZB_REQUIRE((reinterpret_cast<uintptr_t>(ptr) % (bytes)) == 0, "%s must be %d-byte aligned", \
             name, (int)(bytes))

#define ZB_CUDA(call)                                                                      \
  do {                                                                                     \
    cudaError_t err_ = (call);                                                             \
    if (err_ != cudaSuccess)                                                               \
      return zb::fail(zb::kCudaError, "%s failed: %s", #call, cudaGetErrorString(err_));   \
  } while (0)

namespace zb {

__device__ __forceinline__ float bf16_round(float x) {
  return __bfloat162float(__float2bfloat16_rn(x));
}

__device__ __forceinline__ float4 ld_stream_f4(const float* p) {
  return __ldcs(reinterpret_cast<const float4*>(p));
}

__device__ __forceinline__ void st_stream_f4(float* p, float4 v) {
  __stcs(reinterpret_cast<float4*>(p), v);
}

// Four consecutive bf16 values (8 bytes) widened to float.
__device__ __forceinline__ void ld_bf16x4(const __nv_bfloat16* p, float out[4]) {
  uint2 raw = *reinterpret_cast<const uint2*>(p);
  __nv_bfloat162 a = *reinterpret_cast<__nv_bfloat162*>(&raw.x);
  __nv_bfloat162 b = *reinterpret_cast<__nv_bfloat162*>(&raw.y);
  float2 fa = __bfloat1622float2(a), fb = __bfloat1622float2(b);
  out[0] = fa.x; out[1] = fa.y; out[2] = fb.x; out[3] = fb.y;
}

// Eight consecutive bf16 values (16 bytes) widened to float.
__device__ __forceinline__ void ld_bf16x8(const __nv_bfloat16* p, float out[8]) {
  uint4 raw = *reinterpret_cast<const uint4*>(p);
  const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __nv_bfloat162 h = *reinterpret_cast<const __nv_bfloat162*>(&w[i]);
    float2 f = __bfloat1622float2(h);
    out[2 * i] = f.x;
    out[2 * i + 1] = f.y;
  }
}

__device__ __forceinline__ uint4 pack_bf16x8(const float v[8]) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
    w[i] = *reinterpret_cast<uint32_t*>(&h);
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, off));
  return v;
}

}  // namespace zb

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

#include <atomic>
#include <utility>
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

// Device address of the library's status word on the current device (bit flags that kernels set with atomicOr
// when a bounded wait expires; zb_device_status() reads and clears it). nullptr if it cannot be resolved.
unsigned* device_status_ptr();

enum DeviceStatusBits : unsigned {
  kStatusAttnresLoadTimeout = 1u << 0,
  kStatusGemmTimeout = 1u << 1,
  kStatusPrefillTimeout = 1u << 2,
  kStatusAttnresExchangeTimeout = 1u << 3,
  kStatusAttnDecodeTimeout = 1u << 4,
  kStatusEmbedIndex = 1u << 5,  // an embedding id outside its table (read as a zero row)
};

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

// ------------------------------------------------------------------------------ mbarrier / bulk-copy helpers

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

// Makes mbarrier initialisation visible to the async proxy (TMA) and the rest of the cluster.
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

// Adds `bytes` of expected transaction to the current phase without arriving.
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.expect_tx.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

// Cluster barrier split in two: a relaxed arrival (orders nothing; pairs with fence_mbar_init for barrier
// initialisation) and the wait for every thread of the cluster to have arrived.
__device__ __forceinline__ void cluster_arrive_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.aligned;" ::: "memory"); }

// The shared::cluster address of this CTA's shared-memory word `local` in cluster CTA `rank`.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t local, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local), "r"(rank));
  return r;
}

// 4-byte store into another cluster CTA's shared memory, completing 4 bytes of transaction on that CTA's mbarrier.
__device__ __forceinline__ void st_async_b32(uint32_t remote_addr, uint32_t value, uint32_t remote_bar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.b32 [%0], %1, [%2];" ::"r"(remote_addr),
               "r"(value), "r"(remote_bar)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
      : "=r"(done)
      : "r"(bar), "r"(parity)
      : "memory");
  return done != 0;
}

// try_wait that may suspend the thread for up to `hint_ns` until the phase completes (the thread resumes as soon as
// it does), so that waiting warps do not take issue slots from working ones.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint32_t bar, uint32_t parity, uint32_t hint_ns) {
  uint32_t done;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}"
      : "=r"(done)
      : "r"(bar), "r"(parity), "r"(hint_ns)
      : "memory");
  return done != 0;
}

// Waits for phase `parity` of an mbarrier for at most ~`limit_ns`; on expiry ORs `code` into *status and
// returns false (the caller carries on without hanging the GPU).
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity, unsigned* status, unsigned code,
                                                  uint64_t limit_ns = 1000000000ull) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t start = globaltimer_ns();
  for (;;) {
    if (mbar_try_wait_sleep(bar, parity, 20000u)) return true;
    if (globaltimer_ns() - start > limit_ns) {
      if (status) atomicOr(status, code);
      return false;
    }
  }
}

// 1-D bulk copy global -> this CTA's shared memory, completing `bytes` of transaction on mbarrier `bar`.
// src and dst 16-byte aligned, bytes a multiple of 16. No multicast.
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(bar)
               : "memory");
}

// Programmatic dependent launch. Every kernel of the library is launched with zb::launch(), which lets it start
// while the kernel before it in the stream is still running; its first statement is pdl_enter(): wait until that
// kernel has completed and its writes are visible (griddepcontrol.wait; a no-op for a plain launch), then let the
// next kernel start (griddepcontrol.launch_dependents). Nothing a kernel reads or writes in global memory is touched
// before the wait, so the stream order of the memory effects is unchanged; what overlaps the previous kernel's tail
// is the next kernel's launch and CTA setup.
__device__ __forceinline__ void pdl_enter() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
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

// Kernel launches the library has issued from this process (all devices, eager and captured alike).
extern std::atomic<uint64_t> g_launch_count;

// Launches `kernel` on `stream` with programmatic stream serialisation allowed (see pdl_enter) and, when
// cluster_x > 1, clusters of cluster_x CTAs along x; counts the launch in g_launch_count.
template <typename... KArgs, typename... Args>
inline cudaError_t launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                          unsigned cluster_x, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  unsigned n = 0;
  attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[n].val.programmaticStreamSerializationAllowed = 1;
  ++n;
  if (cluster_x > 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = cluster_x;
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  const cudaError_t err = cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
  if (err == cudaSuccess) g_launch_count.fetch_add(1, std::memory_order_relaxed);
  return err;
}

}  // namespace zb

// Allocation-free MoE down projection + combine.
//
// zb_moe_gemm_down writes one weighted expert-output row per (token, slot) pair into a caller-provided [T*k, D]
// buffer, and zb_moe_combine sums each token's k rows. That buffer is scratch: the caller needs neither its size
// nor its contents, only `out`. Some callers cannot provide it, because they cannot call cudaMalloc at all: a
// serving runtime that reserves its whole device-memory budget at start-up and forbids allocation afterwards
// (cudaMalloc can stall the device and fail under fragmentation mid-serving), or a foreign-language binding (C,
// Go, Java) that only hands over the tensors it owns and has no device allocator of its own. For them this entry
// point takes the same inputs and output and keeps the intermediate rows in a fixed array compiled into the
// library instead.
//
// The array holds kNoAllocScratchElems bf16 values (8 MiB), so T * k * D must not exceed 4,194,304 (for example
// 256 decode streams x top-8 x hidden 2048); larger calls are rejected before any work is queued. Every GPU that
// loads the library reserves the array until the process exits. All calls share it and it keeps the previous
// call's contents, so each call clears the rows it uses first (a pair whose expert id is invalid then adds zero),
// and two calls that overlap on the GPU (different streams running at the same time) race on it. The down projection
// drops any pair id at or beyond T * k, so a permutation built for other sizes cannot write past the cleared rows
// (or past the array). The first call on a device resolves the array's device address (cudaGetSymbolAddress) with
// that device current; make that first call before any stream capture. The resolved address is kept per device
// ordinal for the life of the process (one context per device, the CUDA runtime's primary context). No cudaMalloc,
// cudaFree or allocating library routine is called.
#include <atomic>

#include "common.cuh"

namespace zb {
int moe_gemm_down_bounded(const uint16_t* h, int64_t capacity, const uint16_t* down, int E, int D, int I,
                          const int32_t* offsets, const int32_t* counts, const int32_t* sorted_pairs,
                          const float* weights, uint16_t* y, int64_t pair_limit, cudaStream_t stream);
}  // namespace zb

ZB_API int zb_moe_combine(const uint16_t* y, int T, int k, int D, uint16_t* out, int64_t out_stride,
                          cudaStream_t stream);

namespace {

constexpr int64_t kNoAllocScratchElems = int64_t(4) << 20;  // bf16 elements (8 MiB)

// The scratch rows. In host code this name is only a stand-in for the symbol; its device address comes from
// cudaGetSymbolAddress below.
static __device__ __align__(256) uint16_t g_moe_noalloc_scratch[kNoAllocScratchElems];

constexpr int kMaxDevices = 64;

// Device address of the scratch array on the current device, resolved once per device (first calls from several
// host threads may each resolve it; they store the same address).
int scratch_address(uint16_t** out) {
  static std::atomic<uint16_t*> cached[kMaxDevices];
  int dev = 0;
  ZB_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices)
    return zb::fail(zb::kUnsupported, "moe_down_combine_noalloc: device ordinal %d (max %d)", dev, kMaxDevices - 1);
  uint16_t* addr = cached[dev].load(std::memory_order_acquire);
  if (addr == nullptr) {
    void* p = nullptr;
    cudaError_t err = cudaGetSymbolAddress(&p, g_moe_noalloc_scratch);
    if (err != cudaSuccess || p == nullptr)
      return zb::fail(zb::kCudaError, "moe_down_combine_noalloc: cudaGetSymbolAddress failed: %s",
                      cudaGetErrorString(err));
    addr = static_cast<uint16_t*>(p);
    cached[dev].store(addr, std::memory_order_release);
  }
  *out = addr;
  return zb::kOk;
}

}  // namespace

ZB_API int zb_moe_down_combine_noalloc(const uint16_t* h, int64_t capacity, const uint16_t* down, int E, int D, int I,
                                       const int32_t* offsets, const int32_t* counts, const int32_t* sorted_pairs,
                                       const float* weights, int T, int k, uint16_t* out, int64_t out_stride,
                                       cudaStream_t stream) {
  ZB_REQUIRE(T >= 0 && k > 0 && D > 0, "moe_down_combine_noalloc: bad sizes T=%d k=%d D=%d", T, k, D);
  const int64_t elems = (int64_t)T * k * D;
  if (elems > kNoAllocScratchElems)
    return zb::fail(zb::kUnsupported,
                    "moe_down_combine_noalloc: T*k*D = %lld exceeds the static scratch of %lld bf16 elements "
                    "(use zb_moe_gemm_down + zb_moe_combine with a caller buffer)",
                    (long long)elems, (long long)kNoAllocScratchElems);
  if (T == 0) return zb::kOk;
  uint16_t* scratch = nullptr;
  if (int rc = scratch_address(&scratch)) return rc;
  ZB_CUDA(cudaMemsetAsync(scratch, 0, (size_t)elems * sizeof(uint16_t), stream));
  if (int rc = zb::moe_gemm_down_bounded(h, capacity, down, E, D, I, offsets, counts, sorted_pairs, weights, scratch,
                                         (int64_t)T * k, stream))
    return rc;
  return zb_moe_combine(scratch, T, k, D, out, out_stride, stream);
}

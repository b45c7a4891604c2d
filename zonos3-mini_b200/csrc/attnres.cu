// Full AttnRes route: one softmax mix over every bank source so far, optionally fused with the RMSNorm that
// follows it and with the append of the current source to the bank.
//
// Reference: full_attnres_route (model/src/zonos3/reference/lm.py:384-389; servers/sgl/src/zonos3_sgl/models/
// zonos3.py:99-113) and the fused Triton route _block_attnres_fwd_kernel (servers/sgl/src/zonos3_sgl/models/
// training_attnres_kernels.py:1268-1348), whose rounding points this kernel keeps: key = bf16(v * inv_rms),
// product = bf16(key * q), logit = fp32 sum, fp32 softmax, weight = bf16, term = bf16(v * weight), fp32 sum of
// terms, bf16 output. The Triton kernel runs one warp per token and reads the bank twice; here each token's sources
// are staged on chip once and every sweep reads shared memory.
#include <cooperative_groups.h>


#include "common.cuh"

namespace cg = cooperative_groups;

namespace {

constexpr int kMaxSources = 256;
constexpr size_t kRouteSmemBudget = 200 * 1024;

struct RouteParams {
  const __nv_bfloat16* bank;  // [>= S, T, D]
  int64_t bank_stride;        // elements between two sources of the bank
  int S;                      // bank sources routed over
  const __nv_bfloat16* source;  // optional current source [T, D] (routed as source S)
  __nv_bfloat16* append;        // optional: where to write `source` (the next bank row)
  const __nv_bfloat16* query;   // [D]
  float eps;
  const __nv_bfloat16* norm_weight;  // optional RMSNorm weight applied to the mix
  float norm_eps;
  __nv_bfloat16* out;      // [T, D]: normalised mix if norm_weight, else the mix
  __nv_bfloat16* mix_out;  // optional [T, D]: the un-normalised mix (when norm_weight is given)
  float* rms_cache;        // optional [T, rms_stride]: inverse RMS of source s for token t at t * rms_stride + s
  int64_t rms_stride;
  int cached;              // bank rows [0, cached) have valid cache entries; later rows compute and store theirs
  int T, D;
  unsigned* status;
};

__device__ __forceinline__ uint32_t hmul2_bits(uint32_t a, uint32_t b) {
  __nv_bfloat162 r = __hmul2(*reinterpret_cast<const __nv_bfloat162*>(&a), *reinterpret_cast<const __nv_bfloat162*>(&b));
  return *reinterpret_cast<uint32_t*>(&r);
}
__device__ __forceinline__ uint32_t f2_to_bf2(float x, float y) {
  __nv_bfloat162 r = __floats2bfloat162_rn(x, y);
  return *reinterpret_cast<uint32_t*>(&r);
}

// Packed fp32 pairs (one 64-bit register pair; sm_100 executes add / mul / fma on both halves at once).
__device__ __forceinline__ uint64_t bf2_to_x2(uint32_t w) {  // bf16x2 word -> (lo, hi) fp32 pair
  return ((uint64_t)(w & 0xffff0000u) << 32) | (uint64_t)(w << 16);
}
__device__ __forceinline__ uint64_t add_x2(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t mul_x2(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t fma_x2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
__device__ __forceinline__ uint64_t splat_x2(float x) {
  const uint64_t u = __float_as_uint(x);
  return (u << 32) | u;
}
__device__ __forceinline__ float sum_x2(uint64_t v) {
  return __uint_as_float((uint32_t)v) + __uint_as_float((uint32_t)(v >> 32));
}
__device__ __forceinline__ uint32_t x2_to_bf2(uint64_t v) {  // round both halves to bf16 (lo in the low half)
  return f2_to_bf2(__uint_as_float((uint32_t)v), __uint_as_float((uint32_t)(v >> 32)));
}

// One route, one pass over HBM. A token is a cluster of CL CTAs; CTA r owns columns [r*C, (r+1)*C) of every source
// and stages that slice of all ns sources in shared memory (one cp.async.bulk per source, each with its own
// mbarrier, all issued at once; the sources without a cached inverse RMS first, behind one copy of the query slice
// and the token's cached inverse RMS row). The 8 warps then take work units
// round-robin, each as soon as its source has landed:
//   sum-of-squares units (sources without a cached inverse RMS): partial sum of squares of the slice;
//   logit units (every source): inverse RMS (cached, or from the exchanged sums of squares), then the partial logit
//   sum of bf16(bf16(v * inv_rms) * q) — one cvt rounds two keys, one bf16x2 multiply gives two rounded products.
// Every warp then forms the logits, the fp32 softmax and the bf16 weights itself, and mixes 4 (or 2) columns per
// thread: sum over sources of bf16(v * w) in fp32, from shared memory; the optional RMSNorm of the mix and the
// append of the current source follow.
// Partial sums cross the cluster by push: st.async stores into every peer's shared memory that complete bytes on
// the peer's exchange mbarrier, summed in rank order so that every CTA of a token computes identical values. No
// cluster-wide barrier follows the start (whose relaxed arrive only publishes the mbarrier initialisation), so no
// CTA waits on a memory fence or on its peers' progress beyond the data it needs.
constexpr int kRouteThreads = 256;
constexpr int kRouteWarps = kRouteThreads / 32;

// Shared-memory layout of one CTA: ns source slices of C columns, ns + 4 mbarriers, the exchange buffers.
struct RouteLayout {
  size_t bars, qs, inv_rms, xss, xlg, xnrm, wp, red, total;
  __host__ __device__ RouteLayout(int ns, int C, int CL) {
    bars = (size_t)ns * C * 2;               // [ns] source copies + [4] exchanges + [1] query / cache row
    qs = (bars + (size_t)(ns + 6) * 8 + 15) / 16 * 16;  // [C] bf16 query slice
    inv_rms = qs + (size_t)C * 2;            // [ns rounded up to 4] fp32 cached inverse RMS
    xss = inv_rms + (size_t)(ns + 3) / 4 * 16;  // [CL][ns] fp32 partial sums of squares
    xlg = xss + (size_t)CL * ns * 4;         // [CL][ns] fp32 partial logits
    xnrm = xlg + (size_t)CL * ns * 4;        // [8] fp32 partial sums of squares of the mix
    wp = xnrm + 8 * 4;                       // [kRouteWarps][ns] bf16x2 weights (each warp its own row)
    red = wp + (size_t)kRouteWarps * ns * 4; // [kRouteWarps]
    total = red + kRouteWarps * 4;
  }
};

// Writes `v` into slot `idx` of this CTA's exchange buffer `buf` and of every peer's (the CTA's own rank row),
// completing 4 bytes on each peer's mbarrier `bar` and arriving on the local one. Called by a whole warp.
__device__ __forceinline__ void publish(float v, float* buf, uint64_t* bar, int CL, int rank, int lane) {
  if (lane < CL) {
    if (lane == rank) {
      *buf = v;
      zb::mbar_arrive(zb::smem_addr(bar));
    } else {
      zb::st_async_b32(zb::mapa_shared(zb::smem_addr(buf), lane), __float_as_uint(v),
                       zb::mapa_shared(zb::smem_addr(bar), lane));
    }
  }
}

template <int C>
__global__ void __launch_bounds__(kRouteThreads) attnres_route_kernel(RouteParams p) {
  constexpr int kWarps = kRouteWarps;
  constexpr int kLaneVecs = C / 256;   // 16-byte vectors of a lane in the per-source sweeps
  // columns of a thread in the mix: 4 (C = 1024) or 2; with C = 256 only the first 128 threads mix
  constexpr int kColsT = C / kRouteThreads >= 2 ? C / kRouteThreads : 2;
  cg::cluster_group cluster = cg::this_cluster();
  const int CL = (int)cluster.num_blocks();
  const int rank = (int)cluster.block_rank();
  const int64_t t = blockIdx.x / CL;
  const int c0 = rank * C;
  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  const int ns = p.S + (p.source ? 1 : 0);
  const int D = p.D;
  const bool cache = p.rms_cache != nullptr;
  const int first = cache ? p.cached : 0;  // sources [0, first) take their inverse RMS from the cache
  const int nnew = ns - first;

  extern __shared__ __align__(128) unsigned char smem_raw[];
  const RouteLayout lay(ns, C, CL);
  __nv_bfloat16* tiles = reinterpret_cast<__nv_bfloat16*>(smem_raw);  // [ns][C]
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem_raw + lay.bars);
  uint64_t* xbar = bars + ns;  // [0] sums of squares, [1] logits, [2] mix norm (peers), [3] mix norm (local warps)
  uint64_t* meta = xbar + 4;   // query slice and cached inverse RMS row landed
  const __nv_bfloat16* qs = reinterpret_cast<const __nv_bfloat16*>(smem_raw + lay.qs);
  float* xss = reinterpret_cast<float*>(smem_raw + lay.xss);
  float* xlg = reinterpret_cast<float*>(smem_raw + lay.xlg);
  float* xnrm = reinterpret_cast<float*>(smem_raw + lay.xnrm);
  float* inv_rms = reinterpret_cast<float*>(smem_raw + lay.inv_rms);
  uint32_t* wp = reinterpret_cast<uint32_t*>(smem_raw + lay.wp) + (size_t)warp * ns;
  float* red = reinterpret_cast<float*>(smem_raw + lay.red);

  if (tid == 0) {
    for (int s = 0; s < ns; ++s) zb::mbar_init(zb::smem_addr(&bars[s]), 1);
    if (nnew) zb::mbar_init(zb::smem_addr(&xbar[0]), nnew);
    zb::mbar_init(zb::smem_addr(&xbar[1]), ns);
    zb::mbar_init(zb::smem_addr(&xbar[2]), 1);
    zb::mbar_init(zb::smem_addr(&xbar[3]), kWarps);
    zb::mbar_init(zb::smem_addr(meta), 1);
    if (CL > 1) {  // the bytes the peers push
      if (nnew) zb::mbar_expect_tx(zb::smem_addr(&xbar[0]), (CL - 1) * nnew * 4);
      zb::mbar_expect_tx(zb::smem_addr(&xbar[1]), (CL - 1) * ns * 4);
      zb::mbar_arrive_expect_tx(zb::smem_addr(&xbar[2]), (CL - 1) * 4);
    }
    zb::fence_mbar_init();
    // ahead of the sources: the query slice and the token's cached inverse RMS prefix (a token-major cache row)
    const uint32_t inv_bytes = first ? (uint32_t)((first * 4 + 15) / 16 * 16) : 0u;
    zb::mbar_arrive_expect_tx(zb::smem_addr(meta), (uint32_t)C * 2 + inv_bytes);
    zb::bulk_g2s(zb::smem_addr(qs), p.query + c0, C * 2, zb::smem_addr(meta));
    if (inv_bytes)
      zb::bulk_g2s(zb::smem_addr(inv_rms), p.rms_cache + t * p.rms_stride, inv_bytes, zb::smem_addr(meta));
  }
  if (warp == 0) {  // lanes of warp 0 issue the copies: the sources without a cached inverse RMS first
    __syncwarp();
    constexpr uint32_t kSlice = C * 2;
    for (int i = lane; i < ns; i += 32) {
      const int s = i < nnew ? first + i : i - nnew;
      const uint32_t bar = zb::smem_addr(&bars[s]);
      const __nv_bfloat16* src = (s < p.S ? p.bank + (int64_t)s * p.bank_stride : p.source) + t * D + c0;
      zb::mbar_arrive_expect_tx(bar, kSlice);
      zb::bulk_g2s(zb::smem_addr(tiles + (size_t)s * C), src, kSlice, bar);
    }
  }
  __syncthreads();
  if (CL > 1) zb::cluster_arrive_relaxed();
  if (CL > 1) zb::cluster_wait();  // every peer's exchange mbarriers are initialised from here on
  zb::mbar_wait_bounded(zb::smem_addr(meta), 0, p.status, zb::kStatusAttnresLoadTimeout);
  uint4 q4[kLaneVecs];
#pragma unroll
  for (int u = 0; u < kLaneVecs; ++u) q4[u] = *reinterpret_cast<const uint4*>(qs + u * 256 + lane * 8);

  const float inv_d = 1.0f / (float)D;
  for (int u = warp; u < nnew + ns; u += kWarps) {
    if (u < nnew) {  // sum-of-squares unit
      const int s = first + u;
      zb::mbar_wait_bounded(zb::smem_addr(&bars[s]), 0, p.status, zb::kStatusAttnresLoadTimeout);
      const __nv_bfloat16* row = tiles + (size_t)s * C;
      uint64_t ss2 = 0;
#pragma unroll
      for (int v = 0; v < kLaneVecs; ++v) {
        const uint4 x = *reinterpret_cast<const uint4*>(row + v * 256 + lane * 8);
        const uint32_t w[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const uint64_t f = bf2_to_x2(w[k]);
          ss2 = fma_x2(f, f, ss2);
        }
      }
      publish(zb::warp_sum(sum_x2(ss2)), xss + (size_t)rank * ns + s, &xbar[0], CL, rank, lane);
      continue;
    }
    const int s = u - nnew;  // logit unit of source s (cached sources first, so their units run first)
    float inv;
    if (s < first) {
      inv = inv_rms[s];
    } else {
      zb::mbar_wait_bounded(zb::smem_addr(&xbar[0]), 0, p.status, zb::kStatusAttnresExchangeTimeout);
      float total = 0.f;
      for (int r = 0; r < CL; ++r) total += xss[(size_t)r * ns + s];
      inv = rsqrtf(total * inv_d + p.eps);
      if (cache && rank == 0 && lane == 0) p.rms_cache[t * p.rms_stride + s] = inv;
    }
    zb::mbar_wait_bounded(zb::smem_addr(&bars[s]), 0, p.status, zb::kStatusAttnresLoadTimeout);
    const __nv_bfloat16* row = tiles + (size_t)s * C;
    const uint64_t rr2 = splat_x2(inv);
    uint64_t lg2[2] = {0, 0};  // two accumulators: independent add chains
    uint4 x[kLaneVecs];
#pragma unroll
    for (int v = 0; v < kLaneVecs; ++v) x[v] = *reinterpret_cast<const uint4*>(row + v * 256 + lane * 8);
#pragma unroll
    for (int v = 0; v < kLaneVecs; ++v) {
      const uint32_t w[4] = {x[v].x, x[v].y, x[v].z, x[v].w};
      const uint32_t qq[4] = {q4[v].x, q4[v].y, q4[v].z, q4[v].w};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const uint32_t key = x2_to_bf2(mul_x2(bf2_to_x2(w[k]), rr2));  // bf16(v * inv_rms), two at once
        lg2[k & 1] = add_x2(lg2[k & 1], bf2_to_x2(hmul2_bits(key, qq[k])));  // + bf16(key * q)
      }
    }
    publish(zb::warp_sum(sum_x2(add_x2(lg2[0], lg2[1]))), xlg + (size_t)rank * ns + s, &xbar[1], CL, rank, lane);
  }

  // every warp: logits (rank-ordered sums), fp32 softmax, bf16 weights into its own row
  zb::mbar_wait_bounded(zb::smem_addr(&xbar[1]), 0, p.status, zb::kStatusAttnresExchangeTimeout);
  auto logit = [&](int s) {
    float total = 0.f;
    for (int r = 0; r < CL; ++r) total += xlg[(size_t)r * ns + s];
    return total;
  };
  constexpr int kPerLane = kMaxSources / 32;
  float lv[kPerLane];
  float m = -INFINITY;
#pragma unroll
  for (int i = 0; i < kPerLane; ++i) {
    const int s = lane + 32 * i;
    lv[i] = s < ns ? logit(s) : -INFINITY;
    m = fmaxf(m, lv[i]);
  }
  m = zb::warp_max(m);
  float den = 0.f;
#pragma unroll
  for (int i = 0; i < kPerLane; ++i) {
    lv[i] = lane + 32 * i < ns ? expf(lv[i] - m) : 0.f;
    den += lv[i];
  }
  den = zb::warp_sum(den);
#pragma unroll
  for (int i = 0; i < kPerLane; ++i) {
    const int s = lane + 32 * i;
    if (s < ns) wp[s] = (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(lv[i] / den)) * 0x10001u;
  }
  __syncwarp();

  // mix: thread per kColsT columns, all sources from shared memory
  float mix[kColsT];
  const int cc = tid * kColsT;
  const bool mixer = cc < C;
  {
    uint64_t acc[kColsT / 2], acc_odd[kColsT / 2];  // even and odd sources: two independent add chains
#pragma unroll
    for (int j = 0; j < kColsT / 2; ++j) acc[j] = acc_odd[j] = 0;
    if (mixer) {
      auto term = [&](int s, uint64_t (&a)[kColsT / 2]) {
        const uint32_t w2 = wp[s];
        const __nv_bfloat16* row = tiles + (size_t)s * C + cc;
        if constexpr (kColsT == 4) {
          const uint2 v = *reinterpret_cast<const uint2*>(row);
          a[0] = add_x2(a[0], bf2_to_x2(hmul2_bits(v.x, w2)));  // + bf16(v * w), two at once
          a[1] = add_x2(a[1], bf2_to_x2(hmul2_bits(v.y, w2)));
        } else {
          a[0] = add_x2(a[0], bf2_to_x2(hmul2_bits(*reinterpret_cast<const uint32_t*>(row), w2)));
        }
      };
      int s = 0;
#pragma unroll 2
      for (; s + 1 < ns; s += 2) {
        term(s, acc);
        term(s + 1, acc_odd);
      }
      if (s < ns) term(s, acc);
    }
#pragma unroll
    for (int j = 0; j < kColsT / 2; ++j) acc[j] = add_x2(acc[j], acc_odd[j]);
#pragma unroll
    for (int j = 0; j < kColsT / 2; ++j) {
      mix[2 * j] = __uint_as_float((uint32_t)acc[j]);
      mix[2 * j + 1] = __uint_as_float((uint32_t)(acc[j] >> 32));
    }
  }
#pragma unroll
  for (int j = 0; j < kColsT; ++j) mix[j] = zb::bf16_round(mix[j]);
  const int64_t off = t * D + c0 + cc;
  auto store = [&](__nv_bfloat16* dst, const float* vals) {
    if constexpr (kColsT == 4) {
      *reinterpret_cast<uint2*>(dst) = make_uint2(f2_to_bf2(vals[0], vals[1]), f2_to_bf2(vals[2], vals[3]));
    } else {
      *reinterpret_cast<uint32_t*>(dst) = f2_to_bf2(vals[0], vals[1]);
    }
  };
  if (p.norm_weight) {
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < kColsT; ++j) ss = fmaf(mix[j], mix[j], ss);  // zero for threads that do not mix
    ss = zb::warp_sum(ss);
    if (lane == 0) {
      red[warp] = ss;
      zb::mbar_arrive(zb::smem_addr(&xbar[3]));
    }
    zb::mbar_wait_bounded(zb::smem_addr(&xbar[3]), 0, p.status, zb::kStatusAttnresExchangeTimeout);
    float local = 0.f;
    for (int w = 0; w < kWarps; ++w) local += red[w];
    float total = local;
    if (CL > 1) {
      if (warp == 0 && lane < CL && lane != rank)
        zb::st_async_b32(zb::mapa_shared(zb::smem_addr(&xnrm[rank]), lane), __float_as_uint(local),
                         zb::mapa_shared(zb::smem_addr(&xbar[2]), lane));
      zb::mbar_wait_bounded(zb::smem_addr(&xbar[2]), 0, p.status, zb::kStatusAttnresExchangeTimeout);
      total = 0.f;
      for (int r = 0; r < CL; ++r) total += r == rank ? local : xnrm[r];
    }
    const float rn = rsqrtf(total * inv_d + p.norm_eps);
    if (mixer) {
      float y[kColsT];
#pragma unroll
      for (int j = 0; j < kColsT; ++j) y[j] = mix[j] * rn * __bfloat162float(p.norm_weight[c0 + cc + j]);
      if (p.mix_out) store(p.mix_out + off, mix);
      store(p.out + off, y);
    }
  } else if (mixer) {
    store(p.out + off, mix);
  }
  if (p.append) {
    for (int i = tid; i < C / 8; i += kRouteThreads)
      *reinterpret_cast<uint4*>(p.append + t * D + c0 + 8 * i) =
          *reinterpret_cast<const uint4*>(tiles + (size_t)(ns - 1) * C + 8 * i);
  }
}

template <int C>
int launch(const RouteParams& p, cudaStream_t stream) {
  const int ns = p.S + (p.source ? 1 : 0);
  const size_t smem = RouteLayout(ns, C, p.D / C).total;
  auto kernel = attnres_route_kernel<C>;
  if (smem > 48 * 1024) ZB_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  const int CL = p.D / C;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(p.T * CL));
  cfg.blockDim = dim3(kRouteThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = CL;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  ZB_CUDA(cudaLaunchKernelEx(&cfg, kernel, p));
  return zb::check_launch("attnres_route");
}

}  // namespace

ZB_API int zb_attnres_route(const uint16_t* bank, int64_t bank_stride, int S, const uint16_t* source,
                            uint16_t* append, const uint16_t* query, float eps, const uint16_t* norm_weight,
                            float norm_eps, uint16_t* out, uint16_t* mix_out, float* rms_cache, int64_t rms_stride,
                            int cached, int T, int D, cudaStream_t stream) {
  const int ns = S + (source ? 1 : 0);
  ZB_REQUIRE(S >= 0 && T >= 0 && D > 0, "attnres_route: bad sizes S=%d T=%d D=%d", S, T, D);
  ZB_REQUIRE(ns >= 1, "attnres_route: no source to route over");
  if (ns > kMaxSources) return zb::fail(zb::kUnsupported, "attnres_route: %d sources (max %d)", ns, kMaxSources);
  if (D % 256 != 0 || D > 8192)
    return zb::fail(zb::kUnsupported, "attnres_route: D=%d (a multiple of 256, at most 8192)", D);
  // C = columns per CTA: the widest of 1024 / 512 / 256 that divides D into at most 8 CTAs and whose ns slices
  // fit the shared-memory budget (1024 at D=2048 and 49 sources: two CTAs per SM)
  int C = 0;
  for (int c : {1024, 512, 256}) {
    if (D % c == 0 && D / c <= 8 && RouteLayout(ns, c, D / c).total <= kRouteSmemBudget) {
      C = c;
      break;
    }
  }
  if (C == 0) return zb::fail(zb::kUnsupported, "attnres_route: %d sources of D=%d exceed shared memory", ns, D);
  if (T == 0) return zb::kOk;
  ZB_REQUIRE(query && out, "attnres_route: null query/out");
  ZB_REQUIRE(out != source && out != append && (mix_out == nullptr || (mix_out != out && mix_out != source)),
             "attnres_route: out / mix_out must not alias the sources");
  ZB_REQUIRE(S == 0 || bank, "attnres_route: null bank with S=%d", S);
  ZB_REQUIRE(!append || source, "attnres_route: append needs a source");
  ZB_REQUIRE(!mix_out || norm_weight, "attnres_route: mix_out is only written with norm_weight");
  ZB_REQUIRE(S == 0 || bank_stride >= (int64_t)T * D, "attnres_route: bank_stride smaller than T*D");
  ZB_REQUIRE(bank_stride % 8 == 0, "attnres_route: bank_stride must be a multiple of 8 elements");
  ZB_REQUIRE(!rms_cache || (rms_stride >= (ns + 3) / 4 * 4 && rms_stride % 4 == 0 && cached >= 0 && cached <= S),
             "attnres_route: rms cache rows need a stride >= the sources rounded up to 4 (a multiple of 4) and "
             "0 <= cached <= S");
  for (const void* ptr : {(const void*)bank, (const void*)source, (const void*)append, (const void*)query,
                          (const void*)norm_weight, (const void*)out, (const void*)mix_out,
                          (const void*)rms_cache}) {
    ZB_REQUIRE_ALIGNED(ptr, 16, "attnres_route tensors");
  }
  RouteParams p{reinterpret_cast<const __nv_bfloat16*>(bank), bank_stride, S,
                reinterpret_cast<const __nv_bfloat16*>(source), reinterpret_cast<__nv_bfloat16*>(append),
                reinterpret_cast<const __nv_bfloat16*>(query), eps,
                reinterpret_cast<const __nv_bfloat16*>(norm_weight), norm_eps,
                reinterpret_cast<__nv_bfloat16*>(out), reinterpret_cast<__nv_bfloat16*>(mix_out), rms_cache,
                rms_stride, cached, T, D, zb::device_status_ptr()};
  if (C == 1024) return launch<1024>(p, stream);
  if (C == 512) return launch<512>(p, stream);
  return launch<256>(p, stream);
}

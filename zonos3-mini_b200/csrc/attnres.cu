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
  zb::pdl_enter();
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
  ZB_CUDA(zb::launch(kernel, dim3((unsigned)(p.T * CL)), dim3(kRouteThreads), smem, stream, (unsigned)CL, p));
  return zb::check_launch("attnres_route");
}

// ------------------------------------------------------------------------------ route over a logit table
// A source's logit for a route depends only on the source row and the route's query: sum_d bf16(key_d * q_d) with
// key = bf16(v * inv_rms(v)). When a forward registers the queries of its routes up front, route r computes route
// r+1's logits of every bank row while its own mix streams those rows through registers (the key from the row's
// cached inverse RMS, one bf16x2 multiply per two products with the next query), and of its current source, and
// stores them in a table table[r+1][t][s] (fp32, `table_stride` floats per token, T * table_stride per route). Route
// r+1 then needs only its own current source's logit before the softmax: no source is staged on chip, nothing is
// read twice. One CTA per token, D / 8 threads, 8 columns of every source per thread, U loads of 16 bytes in flight
// per thread (the first U issued before the logit work). Rounding points as in attnres_route_kernel; the mix sums
// the terms in source order.
struct TabledParams {
  const __nv_bfloat16* bank;  // [>= S, T, D]: rows whose logits for this route are in the table
  int64_t bank_stride;
  int S;
  const __nv_bfloat16* source;  // [T, D] current source (routed as source S)
  __nv_bfloat16* append;        // optional: where to copy `source` (the next bank row)
  int appended;                 // the current source is bank row S after this route (appended or in place)
  const __nv_bfloat16* queries;  // [num_routes, D]
  int num_routes, route;
  float eps;
  const __nv_bfloat16* norm_weight;
  float norm_eps;
  __nv_bfloat16* out;
  __nv_bfloat16* mix_out;
  float* table;  // [num_routes][T][table_stride]
  int64_t table_stride;
  float* inv_rms;  // [T][inv_stride]: key inverse RMS of bank row s at column s
  int64_t inv_stride;
  int T, D;
};

__device__ __forceinline__ uint4 ld_nc_u4(const __nv_bfloat16* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

// Shared memory of one tabled-route CTA: per-warp partial sums, the bank rows' inverse RMS, softmax weight rows.
struct TabledLayout {
  size_t stash, red_ss, red_lg, red_nrm, inv, red_next, wp, total;
  __host__ __device__ TabledLayout(int nwarps, int ns) {
    stash = 0;                                     // [2][nwarps * 32] uint4: current source, norm weight slices
    red_ss = stash + (size_t)nwarps * 32 * 32;     // [nwarps] sums of squares of the current source
    red_lg = red_ss + (size_t)nwarps * 4;          // [nwarps] partial logits of the current source for this route
    red_nrm = red_lg + (size_t)nwarps * 4;         // [nwarps] sums of squares of the mix
    inv = red_nrm + (size_t)nwarps * 4;            // [ns] inverse RMS of the bank rows
    red_next = inv + (size_t)ns * 4;               // [nwarps][ns] partial logits for the next route
    wp = (red_next + (size_t)nwarps * ns * 4 + 7) / 8 * 8;  // [nwarps][ns] (bf16x2 weight, inverse RMS) per source
    total = wp + (size_t)nwarps * ns * 8;
  }
};

// Warp sums of 16 values at once: lanes l and l + 16 end with the sum over the warp of v[l % 16] (31 shuffles
// instead of 16 x 5).
__device__ __forceinline__ float warp_transpose_sum16(float (&v)[16], int lane) {
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] += __shfl_xor_sync(0xffffffffu, v[i], 16);
#pragma unroll
  for (int half = 8; half >= 1; half >>= 1) {
    const bool upper = lane & half;
#pragma unroll
    for (int i = 0; i < half; ++i) {
      const float send = upper ? v[i] : v[i + half];
      const float keep = upper ? v[i + half] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, half);
    }
  }
  return v[0];
}

// lo += float(low bf16 of w), hi += float(high bf16 of w): sm_100's mixed-precision add takes the bf16 halves as
// they are (the conversion is exact), so no unpacking precedes the fp32 adds.
__device__ __forceinline__ void add_bf2(uint32_t w, float& lo, float& hi) {
  asm("{\n .reg .b16 l, h;\n mov.b32 {l, h}, %2;\n add.rn.f32.bf16 %0, l, %0;\n add.rn.f32.bf16 %1, h, %1;\n}"
      : "+f"(lo), "+f"(hi)
      : "r"(w));
}

// Sum over 8 columns of bf16(key * q) (two fp32 add chains: the low and the high halves).
__device__ __forceinline__ float dot8(const uint32_t (&key)[4], const uint4& q) {
  float lo = 0.f, hi = 0.f;
  add_bf2(hmul2_bits(key[0], q.x), lo, hi);
  add_bf2(hmul2_bits(key[1], q.y), lo, hi);
  add_bf2(hmul2_bits(key[2], q.z), lo, hi);
  add_bf2(hmul2_bits(key[3], q.w), lo, hi);
  return lo + hi;
}

// The 8 keys bf16(v * inv_rms) of a 16-byte source vector.
__device__ __forceinline__ void keys8(const uint4& x, uint64_t inv2, uint32_t (&key)[4]) {
  key[0] = x2_to_bf2(mul_x2(bf2_to_x2(x.x), inv2));
  key[1] = x2_to_bf2(mul_x2(bf2_to_x2(x.y), inv2));
  key[2] = x2_to_bf2(mul_x2(bf2_to_x2(x.z), inv2));
  key[3] = x2_to_bf2(mul_x2(bf2_to_x2(x.w), inv2));
}

template <int U, int kMaxThreads, int kMinBlocks>
__global__ void __launch_bounds__(kMaxThreads, kMinBlocks) attnres_tabled_kernel(TabledParams p) {
  zb::pdl_enter();
  static_assert(U == 16, "a round of U sources is one 16-wide transposed warp sum");
  extern __shared__ __align__(128) unsigned char smem_raw[];
  static_assert(kMaxThreads >= 128, "the inverse-RMS registers cover 256 sources with >= 128 threads");
  const int nwarps = blockDim.x / 32;
  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  const int64_t t = blockIdx.x;
  const int D = p.D, S = p.S, ns = S + 1;
  const int c = tid * 8;
  const bool ahead = p.route + 1 < p.num_routes;  // this route computes the next route's logits
  const TabledLayout lay(nwarps, ns);
  float* red_ss = reinterpret_cast<float*>(smem_raw + lay.red_ss);
  float* red_lg = reinterpret_cast<float*>(smem_raw + lay.red_lg);
  float* red_nrm = reinterpret_cast<float*>(smem_raw + lay.red_nrm);
  float* inv_s = reinterpret_cast<float*>(smem_raw + lay.inv);
  float* red_next = reinterpret_cast<float*>(smem_raw + lay.red_next);
  uint2* wp = reinterpret_cast<uint2*>(smem_raw + lay.wp) + (size_t)warp * ns;
  uint4* stash = reinterpret_cast<uint4*>(smem_raw + lay.stash);

  // every load that depends on nothing, issued first, in the order they are needed: the current source, this and
  // the next route's query slices, the route's table row and the bank rows' inverse RMS (the critical path until the
  // softmax), the norm weight slice (cp.async into shared memory: no register waits for it), and only then the first
  // U bank sources, whose 16 MB over all CTAs would otherwise queue ahead of the current source's row
  uint4 cur = ld_nc_u4(p.source + t * D + c);
  const __nv_bfloat16* q_c = p.queries + (int64_t)p.route * D + c;
  const uint4 q_route = ld_nc_u4(q_c);
  uint4 q_next = make_uint4(0u, 0u, 0u, 0u);
  if (ahead) q_next = ld_nc_u4(q_c + D);
  constexpr int kPerLane = kMaxSources / 32;
  const float* trow = p.table + ((int64_t)p.route * p.T + t) * p.table_stride;
  // lane-strided slots that hold a source (the same for every lane): the softmax works on these only
  const int slots = (S + 1 + 31) / 32;
  float lv[kPerLane];
#pragma unroll
  for (int i = 0; i < kPerLane; ++i) {
    const int s = lane + 32 * i;
    lv[i] = -INFINITY;
    if (i < slots && s < S) lv[i] = trow[s];
  }
  // the bank rows' inverse RMS (for the look-ahead keys): loaded now, stored to shared memory once the logit work
  // has hidden the load
  constexpr int kInvRegs = kMaxSources / 128;  // blockDim >= 128
  float inv_reg[kInvRegs];
#pragma unroll
  for (int j = 0; j < kInvRegs; ++j) {
    const int s = tid + j * blockDim.x;
    inv_reg[j] = ahead && s < S ? p.inv_rms[t * p.inv_stride + s] : 0.f;
  }
  if (p.norm_weight) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 16;\n cp.async.commit_group;" ::"r"(
                     zb::smem_addr(&stash[blockDim.x + tid])),
                 "l"(p.norm_weight + c)
                 : "memory");
  }
  asm volatile("" ::: "memory");  // keep the loads above ahead of the bank prefetch
  const __nv_bfloat16* bank_t = p.bank + t * D + c;
  uint4 buf[U];
#pragma unroll
  for (int i = 0; i < U; ++i)
    if (i < S) buf[i] = ld_nc_u4(bank_t + (int64_t)i * p.bank_stride);

  // inverse RMS of the current source (kept for the later routes when it becomes bank row S)
  const uint32_t w[4] = {cur.x, cur.y, cur.z, cur.w};
  {
    uint64_t ss2 = 0;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const uint64_t f = bf2_to_x2(w[k]);
      ss2 = fma_x2(f, f, ss2);
    }
    const float ss = zb::warp_sum(sum_x2(ss2));
    if (lane == 0) red_ss[warp] = ss;
  }
  __syncthreads();
  float ss_total = 0.f;
  for (int i = 0; i < nwarps; ++i) ss_total += red_ss[i];
  const float inv_cur = rsqrtf(ss_total * (1.0f / (float)D) + p.eps);
  if (p.appended && tid == 0) p.inv_rms[t * p.inv_stride + S] = inv_cur;
  uint32_t key[4];
  keys8(cur, splat_x2(inv_cur), key);

  // the current source's logit for this route
  {
    const float part = zb::warp_sum(dot8(key, q_route));
    if (lane == 0) red_lg[warp] = part;
  }
#pragma unroll
  for (int j = 0; j < kInvRegs; ++j) {
    const int s = tid + j * blockDim.x;
    if (ahead && s < S) inv_s[s] = inv_reg[j];
  }
  __syncthreads();
  float lg_cur = 0.f;
  for (int i = 0; i < nwarps; ++i) lg_cur += red_lg[i];

  // every warp: fp32 softmax over the table row and the current logit, bf16 weights into its own row
  float m = -INFINITY;
#pragma unroll
  for (int i = 0; i < kPerLane; ++i) {
    if (i < slots) {
      if (lane + 32 * i == S) lv[i] = lg_cur;
      m = fmaxf(m, lv[i]);
    }
  }
  m = zb::warp_max(m);
  float den = 0.f;
#pragma unroll
  for (int i = 0; i < kPerLane; ++i) {
    if (i < slots) {
      lv[i] = lane + 32 * i < ns ? expf(lv[i] - m) : 0.f;
      den += lv[i];
    }
  }
  den = zb::warp_sum(den);
#pragma unroll
  for (int i = 0; i < kPerLane; ++i) {
    const int s = lane + 32 * i;
    if (i < slots && s < ns)
      wp[s] = make_uint2((uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(lv[i] / den)) * 0x10001u,
                         __float_as_uint(s < S ? inv_s[s] : 0.f));
  }
  // the current source's next-route logit (its keys are at hand); the source and the norm weight wait in shared
  // memory while the mix holds the registers
  if (ahead && p.appended) {
    const float part = zb::warp_sum(dot8(key, q_next));
    if (lane == 0) red_next[warp * ns + S] = part;
  }
  stash[tid] = cur;
  __syncwarp();

  // mix: sum over sources of bf16(v * w) in fp32, in source order; each consumed load is replaced by the one U
  // sources ahead. Look-ahead: the partial next-route logit of every source, warp-summed 16 sources at a time.
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  auto term = [&](const uint4& v, uint32_t w2) {  // + bf16(v * w), column by column
    add_bf2(hmul2_bits(v.x, w2), acc[0], acc[1]);
    add_bf2(hmul2_bits(v.y, w2), acc[2], acc[3]);
    add_bf2(hmul2_bits(v.z, w2), acc[4], acc[5]);
    add_bf2(hmul2_bits(v.w, w2), acc[6], acc[7]);
  };
  auto step = [&](int s, const uint4& x, float& part) {
    const uint2 wi = wp[s];
    term(x, wi.x);
    if (ahead) {
      uint32_t kx[4];
      keys8(x, splat_x2(__uint_as_float(wi.y)), kx);
      part = dot8(kx, q_next);
    }
  };
  const __nv_bfloat16* next_ld = bank_t + (int64_t)U * p.bank_stride;  // the row load U sources ahead
  int s0 = 0;
  for (; s0 + U <= S; s0 += U) {  // whole rounds of U sources
    float part[U];
#pragma unroll
    for (int i = 0; i < U; ++i) {
      part[i] = 0.f;
      step(s0 + i, buf[i], part[i]);
      if (s0 + i + U < S) buf[i] = ld_nc_u4(next_ld);
      next_ld += p.bank_stride;
    }
    if (ahead) {
      const float total = warp_transpose_sum16(part, lane);
      if (lane < U) red_next[warp * ns + s0 + lane] = total;
    }
  }
  if (s0 < S) {  // the last S % U sources, already loaded
    float part[U];
#pragma unroll
    for (int i = 0; i < U; ++i) {
      part[i] = 0.f;
      if (s0 + i < S) step(s0 + i, buf[i], part[i]);
    }
    if (ahead) {
      const float total = warp_transpose_sum16(part, lane);
      if (lane < U && s0 + lane < S) red_next[warp * ns + s0 + lane] = total;
    }
  }
  cur = stash[tid];
  term(cur, wp[S].x);
  float mix[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) mix[j] = zb::bf16_round(acc[j]);
  const int64_t off = t * D + c;
  if (p.norm_weight) {
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) ss = fmaf(mix[j], mix[j], ss);
    ss = zb::warp_sum(ss);
    if (lane == 0) red_nrm[warp] = ss;
    __syncthreads();
    float total = 0.f;
    for (int i = 0; i < nwarps; ++i) total += red_nrm[i];
    const float rn = rsqrtf(total * (1.0f / (float)D) + p.norm_eps);
    asm volatile("cp.async.wait_all;" ::: "memory");  // this thread's norm weight slice (its own copy)
    const uint4 nw = stash[blockDim.x + tid];
    const uint32_t nww[4] = {nw.x, nw.y, nw.z, nw.w};
    float y[8];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      y[2 * j] = mix[2 * j] * rn * __uint_as_float(nww[j] << 16);
      y[2 * j + 1] = mix[2 * j + 1] * rn * __uint_as_float(nww[j] & 0xffff0000u);
    }
    if (p.mix_out) *reinterpret_cast<uint4*>(p.mix_out + off) = zb::pack_bf16x8(mix);
    *reinterpret_cast<uint4*>(p.out + off) = zb::pack_bf16x8(y);
  } else {
    *reinterpret_cast<uint4*>(p.out + off) = zb::pack_bf16x8(mix);
  }
  if (p.append) *reinterpret_cast<uint4*>(p.append + off) = cur;

  // the next route's logits: each source's warp sums added in warp order
  if (ahead) {
    __syncthreads();
    const int nnext = S + (p.appended ? 1 : 0);
    float* next_row = p.table + ((int64_t)(p.route + 1) * p.T + t) * p.table_stride;
    for (int s = tid; s < nnext; s += blockDim.x) {
      float lg = 0.f;
      for (int i = 0; i < nwarps; ++i) lg += red_next[i * ns + s];
      next_row[s] = lg;
    }
  }
}

template <int U, int kMaxThreads, int kMinBlocks>
int launch_tabled(const TabledParams& p, cudaStream_t stream) {
  const size_t smem = TabledLayout(p.D / 256, p.S + 1).total;
  auto kernel = attnres_tabled_kernel<U, kMaxThreads, kMinBlocks>;
  if (smem > 48 * 1024) ZB_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  ZB_CUDA(zb::launch(kernel, dim3((unsigned)p.T), dim3(p.D / 8), smem, stream, 1, p));
  return zb::check_launch("attnres_route_tabled");
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

ZB_API int zb_attnres_route_tabled(const uint16_t* bank, int64_t bank_stride, int S, const uint16_t* source,
                                   uint16_t* append, int source_in_bank, const uint16_t* queries, int num_routes,
                                   int route, float eps, const uint16_t* norm_weight, float norm_eps, uint16_t* out,
                                   uint16_t* mix_out, float* table, int64_t table_stride, float* inv_rms,
                                   int64_t inv_stride, int T, int D, cudaStream_t stream) {
  ZB_REQUIRE(S >= 0 && T >= 0 && D > 0, "attnres_route_tabled: bad sizes S=%d T=%d D=%d", S, T, D);
  ZB_REQUIRE(num_routes > 0 && route >= 0 && route < num_routes,
             "attnres_route_tabled: route %d outside [0, %d)", route, num_routes);
  if (D % 256 != 0 || D > 4096)
    return zb::fail(zb::kUnsupported, "attnres_route_tabled: D=%d (a multiple of 256, at most 4096)", D);
  // the look-ahead keeps each thread's share of the rows' inverse RMS in kMaxSources / 128 registers
  if (S + 1 > std::min(kMaxSources, (kMaxSources / 128) * (D / 8)))
    return zb::fail(zb::kUnsupported, "attnres_route_tabled: %d sources at D=%d (max %d)", S + 1, D,
                    std::min(kMaxSources, (kMaxSources / 128) * (D / 8)));
  if (D % 256 != 0 || D > 4096)
    return zb::fail(zb::kUnsupported, "attnres_route_tabled: D=%d (a multiple of 256, at most 4096)", D);
  if (T == 0) return zb::kOk;
  const int appended = (append != nullptr || source_in_bank) ? 1 : 0;
  ZB_REQUIRE(source && queries && out && table && inv_rms,
             "attnres_route_tabled: null source/queries/out/table/inv_rms");
  ZB_REQUIRE(!(append && source_in_bank), "attnres_route_tabled: a source already in the bank is not appended");
  ZB_REQUIRE(S == 0 || bank, "attnres_route_tabled: null bank with S=%d", S);
  ZB_REQUIRE(S == 0 || bank_stride >= (int64_t)T * D, "attnres_route_tabled: bank_stride smaller than T*D");
  ZB_REQUIRE(bank_stride % 8 == 0, "attnres_route_tabled: bank_stride must be a multiple of 8 elements");
  ZB_REQUIRE(table_stride >= S + appended && inv_stride >= S + appended,
             "attnres_route_tabled: table / inverse-RMS rows (%lld / %lld floats) below the %d sources",
             (long long)table_stride, (long long)inv_stride, S + appended);
  ZB_REQUIRE(out != source && out != append && (mix_out == nullptr || (mix_out != out && mix_out != source)),
             "attnres_route_tabled: out / mix_out must not alias the sources");
  ZB_REQUIRE(!mix_out || norm_weight, "attnres_route_tabled: mix_out is only written with norm_weight");
  for (const void* ptr : {(const void*)bank, (const void*)source, (const void*)append, (const void*)queries,
                          (const void*)norm_weight, (const void*)out, (const void*)mix_out}) {
    ZB_REQUIRE_ALIGNED(ptr, 16, "attnres_route_tabled tensors");
  }
  TabledParams p{reinterpret_cast<const __nv_bfloat16*>(bank), bank_stride, S,
                 reinterpret_cast<const __nv_bfloat16*>(source), reinterpret_cast<__nv_bfloat16*>(append), appended,
                 reinterpret_cast<const __nv_bfloat16*>(queries), num_routes, route, eps,
                 reinterpret_cast<const __nv_bfloat16*>(norm_weight), norm_eps,
                 reinterpret_cast<__nv_bfloat16*>(out), reinterpret_cast<__nv_bfloat16*>(mix_out), table,
                 table_stride, inv_rms, inv_stride, T, D};
  if (D <= 2048) return launch_tabled<16, 256, 2>(p, stream);
  return launch_tabled<16, 512, 1>(p, stream);
}

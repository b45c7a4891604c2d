// MoE routing: fused router (RMSNorm -> router GEMM -> top-k -> gate weights), the stable token permutation
// by expert, and the gather of token rows into the permuted, tile-padded layout the grouped GEMM reads.
//
// Reference: Router.forward / _select_balanced_topk (servers/sgl/src/zonos3_sgl/models/zonos3.py:746-828),
// Zonos3LM._feed_forward's router (model/src/zonos3/reference/lm.py:610-617), FusedMoE's renormalisation
// (servers/sgl/src/zonos3_sgl/layers/moe/fused_moe/layer.py:159-161) and the histogram / padding / sorted ids of
// moe_align_block_size (servers/sgl/src/zonos3_sgl/layers/moe/fused_moe/fused_moe_impl.py:28-86).
//
// Selection order: scores = float(bf16 logit) - bias; the k best by (score descending, expert index ascending).
// torch.topk leaves the order of equal scores unspecified; this total order is the documented contract.
// Permutation: the flattened (token, slot) pairs p = token * k + slot, stably sorted by expert (ascending p within
// an expert); each expert's segment is padded to a multiple of `block` rows (padding rows hold -1).
#include <algorithm>

#include "common.cuh"

namespace {

constexpr int kRouterWarps = 2;              // 16 tokens per warp
constexpr int kRouterTokens = 16 * kRouterWarps;
constexpr int kChunk = 64;                   // K columns per smem chunk
constexpr int kPad = 8;                      // row padding (elements) against bank conflicts
constexpr int kMaxExperts = 128;

enum WeightMode : int { kSelectedSoftmax = 0, kFullSoftmax = 1 };

// Orderable key of a score: larger score -> larger key; equal scores -> lower index wins.
__device__ __forceinline__ unsigned long long score_key(float s, int idx) {
  unsigned u = __float_as_uint(s);
  u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  return ((unsigned long long)u << 32) | (unsigned)(0xFFFFFFFFu - (unsigned)idx);
}

__device__ __forceinline__ unsigned long long warp_max_u64(unsigned long long v) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    unsigned long long o = __shfl_xor_sync(0xffffffffu, v, off);
    v = o > v ? o : v;
  }
  return v;
}

// One warp selects the top-k of one token. `logit(e)` gives the float value of expert e's (bf16-rounded) logit.
template <typename LogitFn>
__device__ __forceinline__ void select_token(LogitFn logit, const float* bias, int E, int k, int mode, int renorm,
                                             int32_t* ids_out, float* w_out) {
  const int lane = threadIdx.x % 32;
  float lg[kMaxExperts / 32];
  unsigned long long key[kMaxExperts / 32];
#pragma unroll
  for (int j = 0; j < kMaxExperts / 32; ++j) {
    const int e = lane + 32 * j;
    if (e < E) {
      lg[j] = logit(e);
      key[j] = score_key(lg[j] - (bias ? bias[e] : 0.f), e);
    } else {
      lg[j] = -INFINITY;
      key[j] = 0ull;
    }
  }
  float sel_logit = 0.f;  // lane r < k keeps the logit of rank r
  int sel_id = 0;
  for (int r = 0; r < k; ++r) {
    unsigned long long best = 0ull;
#pragma unroll
    for (int j = 0; j < kMaxExperts / 32; ++j) best = key[j] > best ? key[j] : best;
    best = warp_max_u64(best);
    const int e = (int)(0xFFFFFFFFu - (unsigned)(best & 0xFFFFFFFFull));
    float l = 0.f;
#pragma unroll
    for (int j = 0; j < kMaxExperts / 32; ++j) {
      if (lane + 32 * j == e) {
        l = lg[j];
        key[j] = 0ull;  // removed
      }
    }
    l = __shfl_sync(0xffffffffu, l, e % 32);
    if (lane == r) {
      sel_logit = l;
      sel_id = e;
    }
  }
  float w;
  if (mode == kSelectedSoftmax) {
    float m = lane < k ? sel_logit : -INFINITY;
    m = zb::warp_max(m);
    const float ex = lane < k ? expf(sel_logit - m) : 0.f;
    w = ex / zb::warp_sum(ex);
  } else {
    float m = -INFINITY;
#pragma unroll
    for (int j = 0; j < kMaxExperts / 32; ++j) m = fmaxf(m, lg[j]);
    m = zb::warp_max(m);
    float den = 0.f;
#pragma unroll
    for (int j = 0; j < kMaxExperts / 32; ++j)
      if (lane + 32 * j < E) den += expf(lg[j] - m);
    den = zb::warp_sum(den);
    w = lane < k ? expf(sel_logit - m) / den : 0.f;
  }
  if (renorm) {
    const float total = zb::warp_sum(lane < k ? w : 0.f);
    w = w / (total + 1e-8f);
  }
  if (lane < k) {
    ids_out[lane] = sel_id;
    w_out[lane] = w;
  }
}

struct RouterParams {
  const __nv_bfloat16* x;
  int64_t x_stride;
  const __nv_bfloat16* norm_w;
  float eps;
  const __nv_bfloat16* w_router;  // [E, D]
  const float* bias;
  int T, D, E, k, mode, renorm;
  __nv_bfloat16* logits_out;  // optional [T, E]
  int32_t* ids;
  float* weights;
};

__device__ __forceinline__ void mma_bf16_16816(float c[4], const uint32_t a[4], const uint32_t b[2]) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

// NT = number of 8-expert column tiles (E <= 8 * NT).
template <int NT>
__global__ void __launch_bounds__(32 * kRouterWarps) moe_router_kernel(RouterParams p) {
  __shared__ __align__(16) __nv_bfloat16 a_s[kRouterTokens][kChunk + kPad];
  __shared__ __align__(16) __nv_bfloat16 b_s[NT * 8][kChunk + kPad];
  __shared__ float rms_s[kRouterTokens];
  __shared__ float logit_s[kRouterTokens][NT * 8 + 1];
  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  const int tok0 = blockIdx.x * kRouterTokens;

  // inverse RMS of every token of the tile (fp32), the rmsnorm_eda factor
  for (int r = warp; r < kRouterTokens; r += kRouterWarps) {
    const int t = tok0 + r;
    float ss = 0.f;
    if (t < p.T) {
      const __nv_bfloat16* row = p.x + (int64_t)t * p.x_stride;
      for (int c = lane * 8; c < p.D; c += 256) {
        float v[8];
        zb::ld_bf16x8(row + c, v);
#pragma unroll
        for (int j = 0; j < 8; ++j) ss = fmaf(v[j], v[j], ss);
      }
    }
    ss = zb::warp_sum(ss);
    if (lane == 0) rms_s[r] = rsqrtf(ss / (float)p.D + p.eps);
  }
  __syncthreads();

  float acc[NT][4];
#pragma unroll
  for (int n = 0; n < NT; ++n) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.f;
  const int g = lane >> 2, tq = lane & 3;
  for (int k0 = 0; k0 < p.D; k0 += kChunk) {
    // A chunk: router input = bf16(x * inv_rms * norm_weight)
    for (int idx = tid; idx < kRouterTokens * (kChunk / 8); idx += 32 * kRouterWarps) {
      const int r = idx / (kChunk / 8), c = (idx % (kChunk / 8)) * 8;
      const int t = tok0 + r;
      float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      if (t < p.T) {
        float w[8];
        zb::ld_bf16x8(p.x + (int64_t)t * p.x_stride + k0 + c, v);
        zb::ld_bf16x8(p.norm_w + k0 + c, w);
        const float s = rms_s[r];
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = v[j] * s * w[j];
      }
      *reinterpret_cast<uint4*>(&a_s[r][c]) = zb::pack_bf16x8(v);
    }
    for (int idx = tid; idx < NT * 8 * (kChunk / 8); idx += 32 * kRouterWarps) {
      const int e = idx / (kChunk / 8), c = (idx % (kChunk / 8)) * 8;
      uint4 w = make_uint4(0u, 0u, 0u, 0u);
      if (e < p.E) w = *reinterpret_cast<const uint4*>(p.w_router + (int64_t)e * p.D + k0 + c);
      *reinterpret_cast<uint4*>(&b_s[e][c]) = w;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < kChunk; kk += 16) {
      uint32_t a[4];
      const int r0 = warp * 16 + g;
      a[0] = *reinterpret_cast<const uint32_t*>(&a_s[r0][kk + 2 * tq]);
      a[1] = *reinterpret_cast<const uint32_t*>(&a_s[r0 + 8][kk + 2 * tq]);
      a[2] = *reinterpret_cast<const uint32_t*>(&a_s[r0][kk + 2 * tq + 8]);
      a[3] = *reinterpret_cast<const uint32_t*>(&a_s[r0 + 8][kk + 2 * tq + 8]);
#pragma unroll
      for (int n = 0; n < NT; ++n) {
        uint32_t b[2];
        b[0] = *reinterpret_cast<const uint32_t*>(&b_s[n * 8 + g][kk + 2 * tq]);
        b[1] = *reinterpret_cast<const uint32_t*>(&b_s[n * 8 + g][kk + 2 * tq + 8]);
        mma_bf16_16816(acc[n], a, b);
      }
    }
    __syncthreads();
  }
  // logits rounded to bf16 (the router_linear output dtype)
#pragma unroll
  for (int n = 0; n < NT; ++n) {
    const int r0 = warp * 16 + g, c0 = n * 8 + 2 * tq;
    logit_s[r0][c0] = zb::bf16_round(acc[n][0]);
    logit_s[r0][c0 + 1] = zb::bf16_round(acc[n][1]);
    logit_s[r0 + 8][c0] = zb::bf16_round(acc[n][2]);
    logit_s[r0 + 8][c0 + 1] = zb::bf16_round(acc[n][3]);
  }
  __syncthreads();
  for (int r = warp; r < kRouterTokens; r += kRouterWarps) {
    const int t = tok0 + r;
    if (t >= p.T) break;
    if (p.logits_out) {
      for (int e = lane; e < p.E; e += 32)
        p.logits_out[(int64_t)t * p.E + e] = __float2bfloat16_rn(logit_s[r][e]);
    }
    select_token([&](int e) { return logit_s[r][e]; }, p.bias, p.E, p.k, p.mode, p.renorm,
                 p.ids + (int64_t)t * p.k, p.weights + (int64_t)t * p.k);
  }
}

struct SelectParams {
  const void* logits;
  int bf16;
  const float* bias;
  int T, E, k, mode, renorm;
  int32_t* ids;
  float* weights;
};

__global__ void __launch_bounds__(256) moe_select_kernel(SelectParams p) {
  const int t = blockIdx.x * 8 + threadIdx.x / 32;
  if (t >= p.T) return;
  const int64_t base = (int64_t)t * p.E;
  if (p.bf16) {
    const __nv_bfloat16* l = static_cast<const __nv_bfloat16*>(p.logits) + base;
    select_token([&](int e) { return __bfloat162float(l[e]); }, p.bias, p.E, p.k, p.mode, p.renorm,
                 p.ids + (int64_t)t * p.k, p.weights + (int64_t)t * p.k);
  } else {
    const float* l = static_cast<const float*>(p.logits) + base;
    select_token([&](int e) { return l[e]; }, p.bias, p.E, p.k, p.mode, p.renorm, p.ids + (int64_t)t * p.k,
                 p.weights + (int64_t)t * p.k);
  }
}

// ----------------------------------------------------------------------------------------------- permutation

constexpr int kPermWarps = 32;

struct PermuteParams {
  const int32_t* ids;  // [P] flattened (token, slot) experts
  int P, E, block;
  int64_t capacity;    // rows of sorted_pairs
  int32_t* counts;     // [E]
  int32_t* offsets;    // [E + 1] padded segment starts; offsets[E] = padded rows in use
  int32_t* sorted_pairs;  // [capacity], -1 = padding
  int32_t* position;      // [P]
};

// One CTA of 32 warps. Warp w owns the contiguous pair range [w*C, (w+1)*C); pass 1 counts per (warp, expert),
// the scan turns the counts into per-(warp, expert) write cursors, pass 2 re-reads the range in order and places
// every pair at cursor + its rank among the equal experts of its 32-pair group (match.any), which keeps the
// sort stable without atomics on the output order.
__global__ void __launch_bounds__(32 * kPermWarps) moe_permute_kernel(PermuteParams p) {
  extern __shared__ int32_t hist[];  // [kPermWarps][E] counts, then cursors
  __shared__ int32_t seg[kMaxExperts + 1];
  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  for (int i = tid; i < kPermWarps * p.E; i += blockDim.x) hist[i] = 0;
  __syncthreads();
  const int chunk = (p.P + kPermWarps - 1) / kPermWarps;
  const int lo = warp * chunk, hi = min(p.P, lo + chunk);
  for (int i = lo + lane; i < hi; i += 32) {
    const int e = p.ids[i];
    if (e >= 0 && e < p.E) atomicAdd(&hist[warp * p.E + e], 1);
  }
  __syncthreads();
  if (tid < p.E) {
    int total = 0;
    for (int w = 0; w < kPermWarps; ++w) total += hist[w * p.E + tid];
    p.counts[tid] = total;
    seg[tid] = (total + p.block - 1) / p.block * p.block;
  }
  __syncthreads();
  if (tid == 0) {
    int run = 0;
    for (int e = 0; e < p.E; ++e) {
      const int n = seg[e];
      seg[e] = run;
      run += n;
    }
    seg[p.E] = run;
  }
  __syncthreads();
  if (tid <= p.E) p.offsets[tid] = seg[tid];
  if (tid < p.E) {
    int cursor = seg[tid];
    for (int w = 0; w < kPermWarps; ++w) {
      const int n = hist[w * p.E + tid];
      hist[w * p.E + tid] = cursor;
      cursor += n;
    }
  }
  __syncthreads();
  for (int base = lo; base < hi; base += 32) {
    const int i = base + lane;
    const bool live = i < hi;
    const int e = live ? p.ids[i] : -1;
    const bool ok = live && e >= 0 && e < p.E;
    const unsigned peers = __match_any_sync(0xffffffffu, ok ? e : -1);
    const int rank = __popc(peers & ((1u << lane) - 1u));
    int pos = -1;
    if (ok) {
      pos = hist[warp * p.E + e] + rank;
      p.sorted_pairs[pos] = i;
      p.position[i] = pos;
    } else if (live) {
      p.position[i] = -1;
    }
    __syncwarp();
    if (ok && rank == 0) hist[warp * p.E + e] += __popc(peers);
    __syncwarp();
  }
  __syncthreads();
  // padding rows of every segment (from the last warp's final cursor), and everything past the last segment
  for (int e = warp; e < p.E; e += kPermWarps) {
    const int start = hist[(kPermWarps - 1) * p.E + e];
    for (int r = start + lane; r < seg[e + 1]; r += 32) p.sorted_pairs[r] = -1;
  }
  for (int64_t r = seg[p.E] + tid; r < p.capacity; r += blockDim.x) p.sorted_pairs[r] = -1;
}

struct GatherParams {
  const __nv_bfloat16* x;
  int64_t x_stride;
  const int32_t* sorted_pairs;
  int k;
  int64_t rows;
  int D;
  __nv_bfloat16* out;  // [rows, D]
};

// Row r of the permuted activations = x[sorted_pairs[r] / k] (zeros for padding rows); 16-byte vectors.
__global__ void __launch_bounds__(256) moe_gather_kernel(GatherParams p) {
  const int vec_per_row = p.D / 8;
  const int64_t total = p.rows * vec_per_row;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / vec_per_row;
    const int c = (int)(i % vec_per_row) * 8;
    const int pair = p.sorted_pairs[r];
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (pair >= 0) v = *reinterpret_cast<const uint4*>(p.x + (int64_t)(pair / p.k) * p.x_stride + c);
    *reinterpret_cast<uint4*>(p.out + r * p.D + c) = v;
  }
}

struct CombineParams {
  const __nv_bfloat16* y;  // [T * k, D] per-(token, slot) expert outputs, already weighted
  int T, k, D;
  __nv_bfloat16* out;      // [T, D]
  int64_t out_stride;
};

// out[t] = bf16( sum over slots of float(y[t * k + slot]) ), slots in order (the server's moe_sum_reduce).
__global__ void __launch_bounds__(256) moe_combine_kernel(CombineParams p) {
  const int vec_per_row = p.D / 8;
  const int64_t total = (int64_t)p.T * vec_per_row;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = i / vec_per_row;
    const int c = (int)(i % vec_per_row) * 8;
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int s = 0; s < p.k; ++s) {
      float v[8];
      zb::ld_bf16x8(p.y + (t * p.k + s) * p.D + c, v);
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] += v[j];
    }
    *reinterpret_cast<uint4*>(p.out + t * p.out_stride + c) = zb::pack_bf16x8(acc);
  }
}

}  // namespace

ZB_API int zb_moe_combine(const uint16_t* y, int T, int k, int D, uint16_t* out, int64_t out_stride,
                          cudaStream_t stream) {
  ZB_REQUIRE(T >= 0 && k > 0 && D > 0 && D % 8 == 0, "moe_combine: bad sizes T=%d k=%d D=%d", T, k, D);
  if (T == 0) return zb::kOk;
  ZB_REQUIRE(y && out, "moe_combine: null pointer");
  ZB_REQUIRE(out_stride >= D && out_stride % 8 == 0, "moe_combine: out_stride");
  ZB_REQUIRE_ALIGNED(y, 16, "y");
  ZB_REQUIRE_ALIGNED(out, 16, "out");
  CombineParams p{reinterpret_cast<const __nv_bfloat16*>(y), T, k, D, reinterpret_cast<__nv_bfloat16*>(out),
                  out_stride};
  const int64_t vecs = (int64_t)T * (D / 8);
  const int64_t grid = std::min<int64_t>((vecs + 255) / 256, (int64_t)zb::sm_count() * 8);
  moe_combine_kernel<<<(unsigned)grid, 256, 0, stream>>>(p);
  return zb::check_launch("moe_combine");
}

ZB_API int zb_moe_router(const uint16_t* x, int64_t x_stride, const uint16_t* norm_weight, float eps,
                         const uint16_t* w_router, const float* bias, int T, int D, int E, int k, int weight_mode,
                         int renormalize, uint16_t* logits_out, int32_t* ids, float* weights, cudaStream_t stream) {
  ZB_REQUIRE(T >= 0 && D > 0 && E > 0 && k > 0, "moe_router: bad sizes T=%d D=%d E=%d k=%d", T, D, E, k);
  if (E > kMaxExperts || k > E || k > 32)
    return zb::fail(zb::kUnsupported, "moe_router: E=%d k=%d (E <= %d, k <= min(E, 32))", E, k, kMaxExperts);
  if (D % kChunk != 0) return zb::fail(zb::kUnsupported, "moe_router: D=%d must be a multiple of %d", D, kChunk);
  ZB_REQUIRE(weight_mode == kSelectedSoftmax || weight_mode == kFullSoftmax, "moe_router: weight_mode %d", weight_mode);
  if (T == 0) return zb::kOk;
  ZB_REQUIRE(x && norm_weight && w_router && ids && weights, "moe_router: null pointer");
  ZB_REQUIRE(x_stride >= D && x_stride % 8 == 0, "moe_router: x_stride");
  ZB_REQUIRE_ALIGNED(x, 16, "x");
  ZB_REQUIRE_ALIGNED(w_router, 16, "w_router");
  ZB_REQUIRE_ALIGNED(norm_weight, 16, "norm_weight");
  RouterParams p{reinterpret_cast<const __nv_bfloat16*>(x), x_stride,
                 reinterpret_cast<const __nv_bfloat16*>(norm_weight), eps,
                 reinterpret_cast<const __nv_bfloat16*>(w_router), bias, T, D, E, k, weight_mode, renormalize,
                 reinterpret_cast<__nv_bfloat16*>(logits_out), ids, weights};
  const unsigned grid = (unsigned)((T + kRouterTokens - 1) / kRouterTokens);
  const int nt = (E + 7) / 8;
  if (nt <= 1) moe_router_kernel<1><<<grid, 32 * kRouterWarps, 0, stream>>>(p);
  else if (nt <= 2) moe_router_kernel<2><<<grid, 32 * kRouterWarps, 0, stream>>>(p);
  else if (nt <= 4) moe_router_kernel<4><<<grid, 32 * kRouterWarps, 0, stream>>>(p);
  else if (nt <= 8) moe_router_kernel<8><<<grid, 32 * kRouterWarps, 0, stream>>>(p);
  else moe_router_kernel<16><<<grid, 32 * kRouterWarps, 0, stream>>>(p);
  return zb::check_launch("moe_router");
}

ZB_API int zb_moe_select(const void* logits, int logits_bf16, const float* bias, int T, int E, int k,
                         int weight_mode, int renormalize, int32_t* ids, float* weights, cudaStream_t stream) {
  ZB_REQUIRE(T >= 0 && E > 0 && k > 0, "moe_select: bad sizes T=%d E=%d k=%d", T, E, k);
  if (E > kMaxExperts || k > E || k > 32)
    return zb::fail(zb::kUnsupported, "moe_select: E=%d k=%d (E <= %d, k <= min(E, 32))", E, k, kMaxExperts);
  ZB_REQUIRE(weight_mode == kSelectedSoftmax || weight_mode == kFullSoftmax, "moe_select: weight_mode %d", weight_mode);
  if (T == 0) return zb::kOk;
  ZB_REQUIRE(logits && ids && weights, "moe_select: null pointer");
  SelectParams p{logits, logits_bf16, bias, T, E, k, weight_mode, renormalize, ids, weights};
  moe_select_kernel<<<(unsigned)((T + 7) / 8), 256, 0, stream>>>(p);
  return zb::check_launch("moe_select");
}

ZB_API int zb_moe_permute(const int32_t* ids, int T, int k, int E, int block, int64_t capacity, int32_t* counts,
                          int32_t* offsets, int32_t* sorted_pairs, int32_t* position, cudaStream_t stream) {
  ZB_REQUIRE(T >= 0 && k > 0 && E > 0 && block > 0, "moe_permute: bad sizes T=%d k=%d E=%d block=%d", T, k, E, block);
  if (E > kMaxExperts) return zb::fail(zb::kUnsupported, "moe_permute: E=%d (max %d)", E, kMaxExperts);
  const int64_t P = (int64_t)T * k;
  const int64_t need = ((P + (int64_t)E * (block - 1)) + block - 1) / block * block;
  ZB_REQUIRE(capacity >= need, "moe_permute: capacity %lld < %lld padded rows", (long long)capacity, (long long)need);
  ZB_REQUIRE(P < (1ll << 30), "moe_permute: %lld pairs", (long long)P);
  ZB_REQUIRE(counts && offsets && sorted_pairs && position && (P == 0 || ids), "moe_permute: null pointer");
  PermuteParams p{ids, (int)P, E, block, capacity, counts, offsets, sorted_pairs, position};
  const size_t smem = (size_t)kPermWarps * E * sizeof(int32_t);
  moe_permute_kernel<<<1, 32 * kPermWarps, smem, stream>>>(p);
  return zb::check_launch("moe_permute");
}

ZB_API int zb_moe_gather(const uint16_t* x, int64_t x_stride, const int32_t* sorted_pairs, int k, int64_t rows,
                         int D, uint16_t* out, cudaStream_t stream) {
  ZB_REQUIRE(k > 0 && rows >= 0 && D > 0 && D % 8 == 0, "moe_gather: bad sizes k=%d rows=%lld D=%d", k,
             (long long)rows, D);
  if (rows == 0) return zb::kOk;
  ZB_REQUIRE(x && sorted_pairs && out, "moe_gather: null pointer");
  ZB_REQUIRE(x_stride >= D && x_stride % 8 == 0, "moe_gather: x_stride");
  ZB_REQUIRE_ALIGNED(x, 16, "x");
  ZB_REQUIRE_ALIGNED(out, 16, "out");
  GatherParams p{reinterpret_cast<const __nv_bfloat16*>(x), x_stride, sorted_pairs, k, rows, D,
                 reinterpret_cast<__nv_bfloat16*>(out)};
  const int64_t vecs = rows * (D / 8);
  const int64_t grid = std::min<int64_t>((vecs + 255) / 256, (int64_t)zb::sm_count() * 8);
  moe_gather_kernel<<<(unsigned)grid, 256, 0, stream>>>(p);
  return zb::check_launch("moe_gather");
}

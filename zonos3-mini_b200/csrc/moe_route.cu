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
#include <cooperative_groups.h>

#include <algorithm>

#include "common.cuh"

namespace cg = cooperative_groups;

namespace {

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

// The top-k of NT tokens by one warp at once (their shuffle reductions interleave): token i's expert e logit is
// logits[i * row_stride + e]; tokens i >= nt are skipped. Same selection and weights as select_token.
template <int NT>
__device__ __forceinline__ void select_tokens(const float* logits, int row_stride, int nt, const float* bias, int E,
                                              int k, int mode, int renorm, int32_t* ids_out, float* w_out) {
  const int lane = threadIdx.x % 32;
  float lg[NT][kMaxExperts / 32];
  unsigned long long key[NT][kMaxExperts / 32];
#pragma unroll
  for (int i = 0; i < NT; ++i) {
#pragma unroll
    for (int j = 0; j < kMaxExperts / 32; ++j) {
      const int e = lane + 32 * j;
      if (i < nt && e < E) {
        lg[i][j] = logits[i * row_stride + e];
        key[i][j] = score_key(lg[i][j] - (bias ? bias[e] : 0.f), e);
      } else {
        lg[i][j] = -INFINITY;
        key[i][j] = 0ull;
      }
    }
  }
  float sel_logit[NT];
  int sel_id[NT];
#pragma unroll
  for (int i = 0; i < NT; ++i) {
    sel_logit[i] = 0.f;
    sel_id[i] = 0;
  }
  for (int r = 0; r < k; ++r) {
    unsigned long long best[NT];
#pragma unroll
    for (int i = 0; i < NT; ++i) {
      best[i] = 0ull;
#pragma unroll
      for (int j = 0; j < kMaxExperts / 32; ++j) best[i] = key[i][j] > best[i] ? key[i][j] : best[i];
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
#pragma unroll
      for (int i = 0; i < NT; ++i) {
        const unsigned long long o = __shfl_xor_sync(0xffffffffu, best[i], off);
        best[i] = o > best[i] ? o : best[i];
      }
    }
#pragma unroll
    for (int i = 0; i < NT; ++i) {
      const int e = (int)(0xFFFFFFFFu - (unsigned)(best[i] & 0xFFFFFFFFull));
      float l = 0.f;
#pragma unroll
      for (int j = 0; j < kMaxExperts / 32; ++j) {
        if (lane + 32 * j == e) {
          l = lg[i][j];
          key[i][j] = 0ull;  // removed
        }
      }
      l = __shfl_sync(0xffffffffu, l, e % 32);
      if (lane == r) {
        sel_logit[i] = l;
        sel_id[i] = e;
      }
    }
  }
#pragma unroll
  for (int i = 0; i < NT; ++i) {
    float w;
    if (mode == kSelectedSoftmax) {
      float m = lane < k ? sel_logit[i] : -INFINITY;
      m = zb::warp_max(m);
      const float ex = lane < k ? expf(sel_logit[i] - m) : 0.f;
      w = ex / zb::warp_sum(ex);
    } else {
      float m = -INFINITY;
#pragma unroll
      for (int j = 0; j < kMaxExperts / 32; ++j) m = fmaxf(m, lg[i][j]);
      m = zb::warp_max(m);
      float den = 0.f;
#pragma unroll
      for (int j = 0; j < kMaxExperts / 32; ++j)
        if (lane + 32 * j < E) den += expf(lg[i][j] - m);
      den = zb::warp_sum(den);
      w = lane < k ? expf(sel_logit[i] - m) / den : 0.f;
    }
    if (renorm) {
      const float total = zb::warp_sum(lane < k ? w : 0.f);
      w = w / (total + 1e-8f);
    }
    if (i < nt && lane < k) {
      ids_out[i * k + lane] = sel_id[i];
      w_out[i * k + lane] = w;
    }
  }
}

// The top-k of NT tokens with E <= 64 by one warp (lane l holds experts l and l + 32): every key counts the keys
// above it (all 64 compared, no serial rounds; keys are unique, so the ranks are a permutation), the winners of
// ranks < k are placed through `slots` ([NT][k] shared scratch of this warp), then weights as select_token.
template <int NT>
__device__ __forceinline__ void select_tokens_rank(const float* logits, int row_stride, int nt, const float* bias,
                                                   int E, int k, int mode, int renorm, int32_t* ids_out,
                                                   float* w_out, float2* slots) {
  const int lane = threadIdx.x % 32;
  unsigned long long ka[NT], kb[NT];
  float la[NT], lb[NT];
  int ra[NT], rb[NT];
#pragma unroll
  for (int i = 0; i < NT; ++i) {
    const int e0 = lane, e1 = lane + 32;
    la[i] = (i < nt && e0 < E) ? logits[i * row_stride + e0] : -INFINITY;
    lb[i] = (i < nt && e1 < E) ? logits[i * row_stride + e1] : -INFINITY;
    ka[i] = e0 < E ? score_key(la[i] - (bias ? bias[e0] : 0.f), e0) : 0ull;
    kb[i] = e1 < E ? score_key(lb[i] - (bias ? bias[e1] : 0.f), e1) : 0ull;
    ra[i] = rb[i] = 0;
  }
#pragma unroll 4
  for (int src = 0; src < 32; ++src) {
#pragma unroll
    for (int i = 0; i < NT; ++i) {
      const unsigned long long x = __shfl_sync(0xffffffffu, ka[i], src);
      const unsigned long long y = __shfl_sync(0xffffffffu, kb[i], src);
      ra[i] += (x > ka[i]) + (y > ka[i]);
      rb[i] += (x > kb[i]) + (y > kb[i]);
    }
  }
#pragma unroll
  for (int i = 0; i < NT; ++i) {
    if (ra[i] < k) slots[i * k + ra[i]] = make_float2(la[i], __int_as_float(lane));
    if (rb[i] < k) slots[i * k + rb[i]] = make_float2(lb[i], __int_as_float(lane + 32));
  }
  __syncwarp();
#pragma unroll
  for (int i = 0; i < NT; ++i) {
    const float2 sl = lane < k ? slots[i * k + lane] : make_float2(0.f, 0.f);
    const float sel_logit = sl.x;
    const int sel_id = __float_as_int(sl.y);
    float w;
    if (mode == kSelectedSoftmax) {
      float m = lane < k ? sel_logit : -INFINITY;
      m = zb::warp_max(m);
      const float ex = lane < k ? expf(sel_logit - m) : 0.f;
      w = ex / zb::warp_sum(ex);
    } else {
      const float m = zb::warp_max(fmaxf(la[i], lb[i]));
      float den = (lane < E ? expf(la[i] - m) : 0.f) + (lane + 32 < E ? expf(lb[i] - m) : 0.f);
      den = zb::warp_sum(den);
      w = lane < k ? expf(sel_logit - m) / den : 0.f;
    }
    if (renorm) {
      const float total = zb::warp_sum(lane < k ? w : 0.f);
      w = w / (total + 1e-8f);
    }
    if (i < nt && lane < k) {
      ids_out[i * k + lane] = sel_id;
      w_out[i * k + lane] = w;
    }
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

__device__ __forceinline__ void cp_async16(void* dst, const void* src, bool valid) {
  const uint32_t d = zb::smem_addr(dst);
  const int bytes = valid ? 16 : 0;  // zero-fill when invalid
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(d), "l"(src), "r"(bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// bf16x2 word scaled elementwise by (s * w0, s * w1) and rounded back to bf16x2: the router input
// bf16(x * inv_rms * rmsnorm_eda.weight) formed in registers from the raw x tile.
__device__ __forceinline__ uint32_t scale_bf16x2(uint32_t raw, float s, uint32_t wraw) {
  const float2 v = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw));
  const float2 w = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&wraw));
  __nv_bfloat162 o = __floats2bfloat162_rn(v.x * s * w.x, v.y * s * w.y);
  return *reinterpret_cast<uint32_t*>(&o);
}

constexpr int kRouterThreads = 256;  // 8 warps
constexpr int kRouterStages = 4;     // router-weight chunks in flight
constexpr int kRouterChunk = 128;    // columns of a router-weight chunk
constexpr int kRouterWRow = kRouterChunk + kPad;
constexpr size_t kRouterSmemBudget = 220 * 1024;

size_t router_smem(int TOK, int NE, int D) {
  return (size_t)TOK * (D + kPad) * 2 + (size_t)D * 2 + (size_t)kRouterStages * NE * kRouterWRow * 2 +
         (size_t)TOK * 4 + (size_t)TOK * (NE + 1) * 4;
}

// One CTA routes TOK tokens (32, or 16 for wide rows). Its [TOK x D] block of x is loaded into shared memory once
// (cp.async, next to the norm weight) while the first router-weight chunks start streaming; 8 threads per row
// (16 for TOK = 16) form the inverse RMS from shared memory and every element becomes the router input
// bf16(x * inv_rms * rmsnorm_eda.weight) once, in place. The router weight then streams through a 4-stage ring of
// [NE x 128] chunks; warp w computes the logits of token tile (w % MT) x its expert group with mma.sync m16n8k16
// (bf16 in, fp32 accumulate). Logits are rounded to bf16 (the router_linear output dtype) and each warp selects
// the top-k of TOK / 8 tokens at once.
template <int NH, int TOK>
__global__ void __launch_bounds__(kRouterThreads) moe_router_kernel(RouterParams p) {
  zb::pdl_enter();
  constexpr int NE = 32 * NH;           // experts covered by the CTA
  constexpr int MT = TOK / 16;          // token tiles
  constexpr int NG = 8 / MT;            // expert groups
  constexpr int NPW = NE / 8 / NG > 0 ? NE / 8 / NG : 1;  // n-tiles (8 experts) of a warp
  constexpr int TPW = TOK / 8;          // tokens selected by a warp
  const int D = p.D, LX = D + kPad;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __nv_bfloat16* x_s = reinterpret_cast<__nv_bfloat16*>(smem_raw);                // [TOK][LX]
  __nv_bfloat16* nw_s = x_s + (size_t)TOK * LX;                                    // [D]
  __nv_bfloat16* w_s = nw_s + D;                                                   // [stages][NE][kRouterWRow]
  float* rms_s = reinterpret_cast<float*>(w_s + (size_t)kRouterStages * NE * kRouterWRow);  // [TOK]
  float* logit_s = rms_s + TOK;                                                    // [TOK][NE + 1]
  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  const int tok0 = blockIdx.x * TOK;
  const int vecs = D / 8;
  const int n_chunks = D / kRouterChunk;

  // CTAs walk the router-weight chunks from different starting points, so they do not all request the same L2
  // lines at once (each token's logits still sum its chunks in one fixed order)
  const int rot = (int)(blockIdx.x % (unsigned)(n_chunks > 0 ? n_chunks : 1));
  auto load_w = [&](int chunk, int stage) {
    const int k0 = ((chunk + rot) % n_chunks) * kRouterChunk;
    __nv_bfloat16* b = w_s + (size_t)stage * NE * kRouterWRow;
    for (int idx = tid; idx < NE * (kRouterChunk / 8); idx += kRouterThreads) {
      const int e = idx / (kRouterChunk / 8), c = (idx % (kRouterChunk / 8)) * 8;
      cp_async16(b + e * kRouterWRow + c, p.w_router + (int64_t)(e < p.E ? e : 0) * D + k0 + c, e < p.E);
    }
  };
  // x block and norm weight (group 0), then the first router-weight chunks
  for (int idx = tid; idx < TOK * vecs; idx += kRouterThreads) {
    const int r = idx / vecs, c = (idx % vecs) * 8;
    const int t = tok0 + r;
    cp_async16(x_s + (size_t)r * LX + c, p.x + (int64_t)(t < p.T ? t : 0) * p.x_stride + c, t < p.T);
  }
  for (int idx = tid; idx < vecs; idx += kRouterThreads) cp_async16(nw_s + idx * 8, p.norm_w + idx * 8, true);
  cp_async_commit();
#pragma unroll
  for (int st = 0; st < kRouterStages - 1; ++st) {
    if (st < n_chunks) load_w(st, st);
    cp_async_commit();
  }
  cp_async_wait<kRouterStages - 1>();  // the x block has landed
  __syncthreads();
  {  // inverse RMS of every row: 256 / TOK threads per row
    constexpr int TPR = kRouterThreads / TOK;
    const int r = tid / TPR, part = tid % TPR;
    const uint4* row = reinterpret_cast<const uint4*>(x_s + (size_t)r * LX);
    float ss = 0.f;
    for (int j = part; j < vecs; j += TPR) {
      float f[8];
      const uint4 v = row[j];
      zb::ld_bf16x8(reinterpret_cast<const __nv_bfloat16*>(&v), f);
#pragma unroll
      for (int i = 0; i < 8; ++i) ss = fmaf(f[i], f[i], ss);
    }
#pragma unroll
    for (int off = 1; off < TPR; off <<= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
    if (part == 0) rms_s[r] = rsqrtf(ss / (float)D + p.eps);
  }
  __syncthreads();
  for (int idx = tid; idx < TOK * vecs; idx += kRouterThreads) {  // the router input, in place
    const int r = idx / vecs, c = (idx % vecs) * 8;
    uint4* cell = reinterpret_cast<uint4*>(x_s + (size_t)r * LX + c);
    const uint4 raw = *cell, wr = *reinterpret_cast<const uint4*>(nw_s + c);
    const float s = rms_s[r];
    *cell = make_uint4(scale_bf16x2(raw.x, s, wr.x), scale_bf16x2(raw.y, s, wr.y), scale_bf16x2(raw.z, s, wr.z),
                       scale_bf16x2(raw.w, s, wr.w));
  }

  const int mt = warp % MT, nbase = (warp / MT) * NPW;  // token tile, first n-tile of this warp
  const int g = lane >> 2, tq = lane & 3;
  float acc[NPW][4];
#pragma unroll
  for (int n = 0; n < NPW; ++n) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.f;
  const __nv_bfloat16* a = x_s + (size_t)(mt * 16) * LX;
  for (int chunk = 0; chunk < n_chunks; ++chunk) {
    const int stage = chunk % kRouterStages;
    cp_async_wait<kRouterStages - 2>();  // this chunk has landed
    __syncthreads();                      // (first pass: the router input is complete) the previous stage is free
    const int next = chunk + kRouterStages - 1;
    if (next < n_chunks) load_w(next, next % kRouterStages);
    cp_async_commit();
    if (nbase * 8 >= p.E) continue;  // this warp's experts are all padding
    const __nv_bfloat16* b = w_s + (size_t)stage * NE * kRouterWRow;
    const int k0 = ((chunk + rot) % n_chunks) * kRouterChunk;
#pragma unroll
    for (int kk = 0; kk < kRouterChunk; kk += 16) {
      uint32_t af[4];
      af[0] = *reinterpret_cast<const uint32_t*>(a + g * LX + k0 + kk + 2 * tq);
      af[1] = *reinterpret_cast<const uint32_t*>(a + (g + 8) * LX + k0 + kk + 2 * tq);
      af[2] = *reinterpret_cast<const uint32_t*>(a + g * LX + k0 + kk + 2 * tq + 8);
      af[3] = *reinterpret_cast<const uint32_t*>(a + (g + 8) * LX + k0 + kk + 2 * tq + 8);
#pragma unroll
      for (int n = 0; n < NPW; ++n) {
        const int e = (nbase + n) * 8 + g;
        uint32_t bf[2];
        bf[0] = *reinterpret_cast<const uint32_t*>(b + e * kRouterWRow + kk + 2 * tq);
        bf[1] = *reinterpret_cast<const uint32_t*>(b + e * kRouterWRow + kk + 2 * tq + 8);
        mma_bf16_16816(acc[n], af, bf);
      }
    }
  }
  cp_async_wait<0>();
  // logits rounded to bf16 (the router_linear output dtype)
  if (nbase * 8 < NE) {
#pragma unroll
    for (int n = 0; n < NPW; ++n) {
      const int c0 = (nbase + n) * 8 + 2 * tq;
      const int r0 = mt * 16 + g;
      logit_s[r0 * (NE + 1) + c0] = zb::bf16_round(acc[n][0]);
      logit_s[r0 * (NE + 1) + c0 + 1] = zb::bf16_round(acc[n][1]);
      logit_s[(r0 + 8) * (NE + 1) + c0] = zb::bf16_round(acc[n][2]);
      logit_s[(r0 + 8) * (NE + 1) + c0 + 1] = zb::bf16_round(acc[n][3]);
    }
  }
  __syncthreads();
  const int r0 = warp * TPW;
  const int nt = min(TPW, p.T - (tok0 + r0));
  if (nt <= 0) return;
  if (p.logits_out) {
    for (int i = 0; i < nt; ++i)
      for (int e = lane; e < p.E; e += 32)
        p.logits_out[(int64_t)(tok0 + r0 + i) * p.E + e] = __float2bfloat16_rn(logit_s[(r0 + i) * (NE + 1) + e]);
  }
  if (p.E <= 64) {  // slot scratch: the router-weight ring is free now
    float2* slots = reinterpret_cast<float2*>(w_s) + warp * TPW * 32;
    select_tokens_rank<TPW>(logit_s + r0 * (NE + 1), NE + 1, nt, p.bias, p.E, p.k, p.mode, p.renorm,
                            p.ids + (int64_t)(tok0 + r0) * p.k, p.weights + (int64_t)(tok0 + r0) * p.k, slots);
  } else {
    select_tokens<TPW>(logit_s + r0 * (NE + 1), NE + 1, nt, p.bias, p.E, p.k, p.mode, p.renorm,
                       p.ids + (int64_t)(tok0 + r0) * p.k, p.weights + (int64_t)(tok0 + r0) * p.k);
  }
}

template <int NH, int TOK>
int launch_router(const RouterParams& p, cudaStream_t stream) {
  const size_t smem = router_smem(TOK, 32 * NH, p.D);
  auto kernel = moe_router_kernel<NH, TOK>;
  ZB_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  const unsigned grid = (unsigned)((p.T + TOK - 1) / TOK);
  ZB_CUDA(zb::launch(kernel, dim3(grid), dim3(kRouterThreads), smem, stream, 1, p));
  return zb::check_launch("moe_router");
}

template <int NH>
int launch_router_nh(const RouterParams& p, cudaStream_t stream) {
  if (router_smem(32, 32 * NH, p.D) <= kRouterSmemBudget) return launch_router<NH, 32>(p, stream);
  if (router_smem(16, 32 * NH, p.D) <= kRouterSmemBudget) return launch_router<NH, 16>(p, stream);
  return zb::fail(zb::kUnsupported, "moe_router: D=%d with %d experts exceeds shared memory", p.D, 32 * NH);
}

// Router for few tokens: the D columns split across a cluster of kSplit CTAs, so the router weight (E x D) is read
// by kSplit CTAs in slices instead of whole by every CTA. CTA r of a cluster takes TOK = 32 tokens and columns
// [r*D/kSplit, (r+1)*D/kSplit): it stages its x and router-weight slices, forms the partial sums of squares of its
// rows, exchanges them through distributed shared memory (every CTA sums the ranks in order, so all agree on the
// inverse RMS), builds the router input bf16(x * inv_rms * rmsnorm_eda.weight) of its slice and the partial logits
// (mma.sync m16n8k16, fp32); after a cluster barrier CTA r sums the partial logits of tokens [4r, 4r + 4) over the
// ranks in order, rounds them to bf16 and selects their top-k exactly as the one-CTA router does.
constexpr int kSplit = 8;
constexpr int kSplitTok = 32;

size_t router_split_smem(int NE, int DS) {
  const int LXS = DS + kPad;
  return (size_t)kSplitTok * LXS * 2 + (size_t)NE * LXS * 2 + (size_t)DS * 2 + (size_t)kSplit * kSplitTok * 4 +
         (size_t)kSplitTok * 4 + (size_t)kSplitTok * (NE + 1) * 4 + (size_t)(kSplitTok / kSplit) * (NE + 1) * 4;
}

template <int NH>
__global__ void __launch_bounds__(kRouterThreads) moe_router_split_kernel(RouterParams p) {
  zb::pdl_enter();
  constexpr int NE = 32 * NH;
  constexpr int TOK = kSplitTok;
  constexpr int MT = TOK / 16, NG = 8 / MT, NPW = NE / 8 / NG > 0 ? NE / 8 / NG : 1;
  constexpr int TPC = TOK / kSplit;  // tokens a CTA selects
  cg::cluster_group cluster = cg::this_cluster();
  const int r = (int)cluster.block_rank();
  const int tok0 = (int)(blockIdx.x / kSplit) * TOK;
  const int D = p.D, DS = D / kSplit, LXS = DS + kPad, c0 = r * DS;
  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __nv_bfloat16* x_s = reinterpret_cast<__nv_bfloat16*>(smem_raw);  // [TOK][LXS]
  __nv_bfloat16* w_s = x_s + (size_t)TOK * LXS;                       // [NE][LXS]
  __nv_bfloat16* nw_s = w_s + (size_t)NE * LXS;                       // [DS]
  float* ssq = reinterpret_cast<float*>(nw_s + DS);                   // [kSplit][TOK] partial sums of squares
  float* rms_s = ssq + kSplit * TOK;                                  // [TOK]
  float* part = rms_s + TOK;                                          // [TOK][NE + 1] partial logits
  float* lg = part + TOK * (NE + 1);                                  // [TPC][NE + 1] logits of the selected tokens

  const int vs = DS / 8;
  for (int idx = tid; idx < TOK * vs; idx += kRouterThreads) {
    const int row = idx / vs, c = (idx % vs) * 8;
    const int t = tok0 + row;
    cp_async16(x_s + (size_t)row * LXS + c, p.x + (int64_t)(t < p.T ? t : 0) * p.x_stride + c0 + c, t < p.T);
  }
  for (int idx = tid; idx < NE * vs; idx += kRouterThreads) {
    const int e = idx / vs, c = (idx % vs) * 8;
    cp_async16(w_s + (size_t)e * LXS + c, p.w_router + (int64_t)(e < p.E ? e : 0) * D + c0 + c, e < p.E);
  }
  for (int idx = tid; idx < vs; idx += kRouterThreads) cp_async16(nw_s + idx * 8, p.norm_w + c0 + idx * 8, true);
  cp_async_commit();
  cp_async_wait<0>();
  __syncthreads();
  {  // partial sums of squares of this slice, 8 threads per row, pushed into every CTA's row r
    constexpr int TPR = kRouterThreads / TOK;
    const int row = tid / TPR, pt = tid % TPR;
    const uint4* xr = reinterpret_cast<const uint4*>(x_s + (size_t)row * LXS);
    float ss = 0.f;
    for (int j = pt; j < vs; j += TPR) {
      float f[8];
      const uint4 v = xr[j];
      zb::ld_bf16x8(reinterpret_cast<const __nv_bfloat16*>(&v), f);
#pragma unroll
      for (int i = 0; i < 8; ++i) ss = fmaf(f[i], f[i], ss);
    }
#pragma unroll
    for (int off = 1; off < TPR; off <<= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
    if (pt == 0)
      for (int q = 0; q < kSplit; ++q) *cluster.map_shared_rank(ssq + r * TOK + row, q) = ss;
  }
  cluster.sync();
  if (tid < TOK) {
    float total = 0.f;
    for (int q = 0; q < kSplit; ++q) total += ssq[q * TOK + tid];
    rms_s[tid] = rsqrtf(total / (float)D + p.eps);
  }
  __syncthreads();
  for (int idx = tid; idx < TOK * vs; idx += kRouterThreads) {  // the router input of this slice, in place
    const int row = idx / vs, c = (idx % vs) * 8;
    uint4* cell = reinterpret_cast<uint4*>(x_s + (size_t)row * LXS + c);
    const uint4 raw = *cell, wr = *reinterpret_cast<const uint4*>(nw_s + c);
    const float sc = rms_s[row];
    *cell = make_uint4(scale_bf16x2(raw.x, sc, wr.x), scale_bf16x2(raw.y, sc, wr.y), scale_bf16x2(raw.z, sc, wr.z),
                       scale_bf16x2(raw.w, sc, wr.w));
  }
  __syncthreads();
  {  // partial logits of the slice
    const int mt = warp % MT, nbase = (warp / MT) * NPW;
    const int g = lane >> 2, tq = lane & 3;
    float acc[NPW][4];
#pragma unroll
    for (int n = 0; n < NPW; ++n) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.f;
    const __nv_bfloat16* a = x_s + (size_t)(mt * 16) * LXS;
    if (nbase * 8 < p.E) {
      for (int kk = 0; kk < DS; kk += 16) {
        uint32_t af[4];
        af[0] = *reinterpret_cast<const uint32_t*>(a + g * LXS + kk + 2 * tq);
        af[1] = *reinterpret_cast<const uint32_t*>(a + (g + 8) * LXS + kk + 2 * tq);
        af[2] = *reinterpret_cast<const uint32_t*>(a + g * LXS + kk + 2 * tq + 8);
        af[3] = *reinterpret_cast<const uint32_t*>(a + (g + 8) * LXS + kk + 2 * tq + 8);
#pragma unroll
        for (int n = 0; n < NPW; ++n) {
          const int e = (nbase + n) * 8 + g;
          uint32_t bf[2];
          bf[0] = *reinterpret_cast<const uint32_t*>(w_s + (size_t)e * LXS + kk + 2 * tq);
          bf[1] = *reinterpret_cast<const uint32_t*>(w_s + (size_t)e * LXS + kk + 2 * tq + 8);
          mma_bf16_16816(acc[n], af, bf);
        }
      }
    }
#pragma unroll
    for (int n = 0; n < NPW; ++n) {
      const int cc = (nbase + n) * 8 + 2 * tq, r0 = mt * 16 + g;
      if (cc < NE) {
        part[r0 * (NE + 1) + cc] = acc[n][0];
        part[r0 * (NE + 1) + cc + 1] = acc[n][1];
        part[(r0 + 8) * (NE + 1) + cc] = acc[n][2];
        part[(r0 + 8) * (NE + 1) + cc + 1] = acc[n][3];
      }
    }
  }
  cluster.sync();  // every CTA's partial logits are complete
  if (warp < TPC) {
    const int lt = r * TPC + warp;  // token of the block this warp selects
    const int t = tok0 + lt;
    float* row = lg + warp * (NE + 1);
    for (int e = lane; e < p.E; e += 32) {
      float total = 0.f;
      for (int q = 0; q < kSplit; ++q) total += *cluster.map_shared_rank(part + lt * (NE + 1) + e, q);
      row[e] = zb::bf16_round(total);
    }
    __syncwarp();
    if (t < p.T) {
      if (p.logits_out)
        for (int e = lane; e < p.E; e += 32) p.logits_out[(int64_t)t * p.E + e] = __float2bfloat16_rn(row[e]);
      select_token([&](int e) { return row[e]; }, p.bias, p.E, p.k, p.mode, p.renorm, p.ids + (int64_t)t * p.k,
                   p.weights + (int64_t)t * p.k);
    }
  }
  cluster.sync();  // no CTA leaves while its peers still read its partial logits
}

template <int NH>
int launch_router_split(const RouterParams& p, cudaStream_t stream) {
  const size_t smem = router_split_smem(32 * NH, p.D / kSplit);
  auto kernel = moe_router_split_kernel<NH>;
  ZB_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  ZB_CUDA(zb::launch(kernel, dim3((unsigned)(((p.T + kSplitTok - 1) / kSplitTok) * kSplit)), dim3(kRouterThreads),
                     smem, stream, (unsigned)kSplit, p));
  return zb::check_launch("moe_router(split)");
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
  zb::pdl_enter();
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

constexpr int kPermPairs = 256;  // pairs of one CTA (8 warps x 32)
constexpr int kPermThreads = 256;

struct PermuteParams {
  const int32_t* ids;  // [P] flattened (token, slot) experts
  int P, E, block;
  int64_t capacity;       // rows of sorted_pairs
  int32_t* hist;          // scratch [num_ctas][E]: per-CTA expert counts
  int32_t* counts;        // [E]
  int32_t* offsets;       // [E + 1] padded segment starts; offsets[E] = padded rows in use
  int32_t* sorted_pairs;  // [capacity], -1 = padding
  int32_t* position;      // [P]
  // optional gather folded into the scatter: x_perm[position[i]] = x[i / k] (x_perm null: no gather)
  const __nv_bfloat16* x;
  int64_t x_stride;
  int k, D;
  __nv_bfloat16* x_perm;
  int groups;  // blocks per 256-pair slice: each ranks the slice and copies 256 / groups of its rows
};

// Pass 1: the expert histogram of each 256-pair slice (order-free shared-memory atomics).
__global__ void __launch_bounds__(kPermThreads) moe_count_kernel(PermuteParams p) {
  zb::pdl_enter();
  __shared__ int32_t h[kMaxExperts];
  for (int e = threadIdx.x; e < p.E; e += kPermThreads) h[e] = 0;
  __syncthreads();
  const int i = blockIdx.x * kPermPairs + threadIdx.x;
  if (i < p.P) {
    const int e = p.ids[i];
    if (e >= 0 && e < p.E) atomicAdd(&h[e], 1);
  }
  __syncthreads();
  for (int e = threadIdx.x; e < p.E; e += kPermThreads) p.hist[(int64_t)blockIdx.x * p.E + e] = h[e];
}

// Pass 2: every CTA derives the padded segment starts and its own write cursor per expert from all slice
// histograms (slices before it, in order), then places its 256 pairs: warp w handles pairs [32w, 32w+32) of the
// slice, ranks among equal experts inside the warp come from match.any, and the per-(warp, expert) counts are
// scanned across the warps. Pairs of one expert therefore keep ascending p (stable), with no atomics on order.
__global__ void __launch_bounds__(kPermThreads) moe_scatter_kernel(PermuteParams p) {
  zb::pdl_enter();
  __shared__ int32_t base[kMaxExperts];      // write cursor of this slice per expert
  __shared__ int32_t seg[kMaxExperts + 1];   // padded segment starts
  __shared__ int32_t total[kMaxExperts];
  __shared__ int32_t wcount[kPermThreads / 32][kMaxExperts];
  __shared__ int32_t pos_s[kPermPairs];
  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  const int G = p.groups;  // the slice's blocks: block 0 writes the permutation, every block copies its rows
  const int nslices = gridDim.x / G, me = blockIdx.x / G, sub = blockIdx.x % G;
  const bool writer = sub == 0;
  {  // totals and this slice's prefix per expert: thread (group g, expert e) sums a strided share of the slices
    int* part_all = &wcount[0][0];  // reused as [groups][E] partial sums before the rank pass
    int* part_before = part_all + kMaxExperts * 4;
    const int groups = min(kPermThreads / p.E, 4);
    const int e = tid % p.E, gi = tid / p.E;
    if (gi < groups) {
      int before = 0, all = 0;
#pragma unroll 8
      for (int c = gi; c < nslices; c += groups) {
        const int n = p.hist[(int64_t)c * p.E + e];
        before += c < me ? n : 0;
        all += n;
      }
      part_all[gi * kMaxExperts + e] = all;
      part_before[gi * kMaxExperts + e] = before;
    }
    __syncthreads();
    if (tid < p.E) {
      int all = 0, before = 0;
      for (int g = 0; g < groups; ++g) {
        all += part_all[g * kMaxExperts + tid];
        before += part_before[g * kMaxExperts + tid];
      }
      total[tid] = all;
      base[tid] = before;
    }
    __syncthreads();
  }
  for (int i = tid; i < (kPermThreads / 32) * kMaxExperts; i += kPermThreads) (&wcount[0][0])[i] = 0;
  __syncthreads();
  if (warp == 0) {  // exclusive scan of the padded totals (E <= 128: 4 per lane)
    int local[kMaxExperts / 32];
    int run = 0;
#pragma unroll
    for (int j = 0; j < kMaxExperts / 32; ++j) {
      const int e = lane * (kMaxExperts / 32) + j;
      local[j] = e < p.E ? (total[e] + p.block - 1) / p.block * p.block : 0;
      run += local[j];
    }
    int incl = run;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int o = __shfl_up_sync(0xffffffffu, incl, off);
      if (lane >= off) incl += o;
    }
    int start = incl - run;
#pragma unroll
    for (int j = 0; j < kMaxExperts / 32; ++j) {
      const int e = lane * (kMaxExperts / 32) + j;
      if (e < p.E) seg[e] = start;
      start += local[j];
    }
    if (lane == 31) seg[p.E] = incl;
  }
  __syncthreads();
  // ranks inside this slice
  const int i = me * kPermPairs + tid;
  const bool live = i < p.P;
  const int e = live ? p.ids[i] : -1;
  const bool ok = live && e >= 0 && e < p.E;
  const unsigned peers = __match_any_sync(0xffffffffu, ok ? e : -1);
  const int rank = __popc(peers & ((1u << lane) - 1u));
  if (ok && rank == 0) wcount[warp][e] = __popc(peers);
  __syncthreads();
  int pos = -1;
  if (ok) {
    pos = seg[e] + base[e] + rank;
    for (int w = 0; w < warp; ++w) pos += wcount[w][e];
  }
  if (writer) {
    if (ok) p.sorted_pairs[pos] = i;
    if (live) p.position[i] = pos;
    // padding rows of every segment (expert e handled by slice e % nslices), then rows past the last segment
    for (int x = me; x < p.E; x += nslices) {
      for (int r = seg[x] + total[x] + tid; r < seg[x + 1]; r += kPermThreads) p.sorted_pairs[r] = -1;
    }
    for (int64_t r = seg[p.E] + (int64_t)me * kPermThreads + tid; r < p.capacity;
         r += (int64_t)nslices * kPermThreads)
      p.sorted_pairs[r] = -1;
    if (me == 0) {
      for (int x = tid; x < p.E; x += kPermThreads) p.counts[x] = total[x];
      for (int x = tid; x <= p.E; x += kPermThreads) p.offsets[x] = seg[x];
    }
  }
  if (p.x_perm == nullptr) return;
  // the gather: this block's share of the slice's rows, a warp per row (8 independent 16-byte loads per lane in
  // flight); padding rows of x_perm are not written (the grouped GEMMs drop their results)
  pos_s[tid] = pos;
  __syncthreads();
  const int per = kPermPairs / G;
  const int vec_per_row = p.D / 8;
  for (int j = warp; j < per; j += kPermThreads / 32) {
    const int il = sub * per + j;
    const int dst_row = pos_s[il];
    if (dst_row < 0) continue;
    const int pair = me * kPermPairs + il;
    const uint4* src = reinterpret_cast<const uint4*>(p.x + (int64_t)(pair / p.k) * p.x_stride);
    uint4* dst = reinterpret_cast<uint4*>(p.x_perm + (int64_t)dst_row * p.D);
    for (int c0 = lane; c0 < vec_per_row; c0 += 32 * 8) {
      uint4 v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int c = c0 + 32 * u;
        v[u] = make_uint4(0u, 0u, 0u, 0u);
        if (c < vec_per_row) v[u] = __ldg(src + c);
      }
#pragma unroll
      for (int u = 0; u < 8; ++u)
        if (c0 + 32 * u < vec_per_row) dst[c0 + 32 * u] = v[u];
    }
  }
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

// Row r of the permuted activations = x[sorted_pairs[r] / k]; padding rows (sorted_pairs < 0) are not written: the
// grouped GEMMs compute every row independently and drop the padding rows' results, so their content never reaches
// an output (at decode most of the padded capacity is padding). A warp copies whole rows: the row's pair index is
// read once, then every lane keeps 8 independent 16-byte loads in flight.
__global__ void __launch_bounds__(256) moe_gather_kernel(GatherParams p) {
  zb::pdl_enter();
  const int lane = threadIdx.x % 32;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x / 32);
  const int vec_per_row = p.D / 8;
  for (int64_t r = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32; r < p.rows; r += warps) {
    const int pair = p.sorted_pairs[r];
    if (pair < 0) continue;
    const uint4* src = reinterpret_cast<const uint4*>(p.x + (int64_t)(pair / p.k) * p.x_stride);
    uint4* dst = reinterpret_cast<uint4*>(p.out + r * p.D);
    for (int c0 = lane; c0 < vec_per_row; c0 += 32 * 8) {
      uint4 v[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int c = c0 + 32 * j;
        v[j] = make_uint4(0u, 0u, 0u, 0u);
        if (c < vec_per_row) v[j] = __ldg(src + c);
      }
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (c0 + 32 * j < vec_per_row) dst[c0 + 32 * j] = v[j];
    }
  }
}

struct CombineParams {
  const __nv_bfloat16* y;  // [T * k, D] per-(token, slot) expert outputs, already weighted
  int T, k, D;
  __nv_bfloat16* out;      // [T, D]
  int64_t out_stride;
};

// out[t] = bf16( sum over slots of float(y[t * k + slot]) ), slots in order (the server's moe_sum_reduce). A warp
// sums whole token rows: every lane keeps the 16-byte vectors of 2 columns x up to 8 slots in flight.
__global__ void __launch_bounds__(256) moe_combine_kernel(CombineParams p) {
  zb::pdl_enter();
  const int lane = threadIdx.x % 32;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x / 32);
  const int vec_per_row = p.D / 8;
  const int chunks = (vec_per_row + 63) / 64;  // 512-column pieces of a row: the warps' units
  for (int64_t u = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32; u < (int64_t)p.T * chunks;
       u += warps) {
    const int64_t t = u / chunks;
    const uint4* rows = reinterpret_cast<const uint4*>(p.y + t * p.k * p.D);
    uint4* dst = reinterpret_cast<uint4*>(p.out + t * p.out_stride);
    {
      const int c0 = (int)(u % chunks) * 64 + lane;
      if (c0 >= vec_per_row) continue;
      const bool has1 = c0 + 32 < vec_per_row;
      float acc0[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f}, acc1[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      for (int s0 = 0; s0 < p.k; s0 += 8) {
        uint4 r0[8], r1[8];
#pragma unroll
        for (int s = 0; s < 8; ++s) {
          if (s0 + s < p.k) {
            r0[s] = __ldcs(rows + (int64_t)(s0 + s) * vec_per_row + c0);
            if (has1) r1[s] = __ldcs(rows + (int64_t)(s0 + s) * vec_per_row + c0 + 32);
          }
        }
#pragma unroll
        for (int s = 0; s < 8; ++s) {
          if (s0 + s < p.k) {
            float v[8];
            zb::ld_bf16x8(reinterpret_cast<const __nv_bfloat16*>(&r0[s]), v);
#pragma unroll
            for (int j = 0; j < 8; ++j) acc0[j] += v[j];
            if (has1) {
              zb::ld_bf16x8(reinterpret_cast<const __nv_bfloat16*>(&r1[s]), v);
#pragma unroll
              for (int j = 0; j < 8; ++j) acc1[j] += v[j];
            }
          }
        }
      }
      dst[c0] = zb::pack_bf16x8(acc0);
      if (has1) dst[c0 + 32] = zb::pack_bf16x8(acc1);
    }
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
  const int64_t units = (int64_t)T * ((D / 8 + 63) / 64);  // a warp per 512-column piece of a token's row
  const int64_t grid = std::min<int64_t>((units + 7) / 8, (int64_t)zb::sm_count() * 8);
  ZB_CUDA(zb::launch(moe_combine_kernel, dim3((unsigned)grid), dim3(256), 0, stream, 1, p));
  return zb::check_launch("moe_combine");
}

ZB_API int zb_moe_router(const uint16_t* x, int64_t x_stride, const uint16_t* norm_weight, float eps,
                         const uint16_t* w_router, const float* bias, int T, int D, int E, int k, int weight_mode,
                         int renormalize, uint16_t* logits_out, int32_t* ids, float* weights, cudaStream_t stream) {
  ZB_REQUIRE(T >= 0 && D > 0 && E > 0 && k > 0, "moe_router: bad sizes T=%d D=%d E=%d k=%d", T, D, E, k);
  if (E > kMaxExperts || k > E || k > 32)
    return zb::fail(zb::kUnsupported, "moe_router: E=%d k=%d (E <= %d, k <= min(E, 32))", E, k, kMaxExperts);
  if (D % kRouterChunk != 0)
    return zb::fail(zb::kUnsupported, "moe_router: D=%d must be a multiple of %d", D, kRouterChunk);
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
  const int nh = (E + 31) / 32;
  // few tokens: the one-CTA-per-32-tokens router would run on a handful of SMs, each streaming the whole router
  // weight; split the columns across clusters instead
  if ((int64_t)(T + kSplitTok - 1) / kSplitTok * kSplit <= 2 * (int64_t)zb::sm_count() && D % (kSplit * 16) == 0 &&
      router_split_smem(32 * (nh <= 1 ? 1 : nh <= 2 ? 2 : 4), D / kSplit) <= kRouterSmemBudget) {
    if (nh <= 1) return launch_router_split<1>(p, stream);
    if (nh <= 2) return launch_router_split<2>(p, stream);
    return launch_router_split<4>(p, stream);
  }
  if (nh <= 1) return launch_router_nh<1>(p, stream);
  if (nh <= 2) return launch_router_nh<2>(p, stream);
  return launch_router_nh<4>(p, stream);
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
  ZB_CUDA(zb::launch(moe_select_kernel, dim3((unsigned)((T + 7) / 8)), dim3(256), 0, stream, 1, p));
  return zb::check_launch("moe_select");
}

ZB_API int zb_moe_permute(const int32_t* ids, int T, int k, int E, int block, int64_t capacity, int32_t* hist,
                          int32_t* counts, int32_t* offsets, int32_t* sorted_pairs, int32_t* position,
                          cudaStream_t stream) {
  ZB_REQUIRE(T >= 0 && k > 0 && E > 0 && block > 0, "moe_permute: bad sizes T=%d k=%d E=%d block=%d", T, k, E, block);
  if (E > kMaxExperts) return zb::fail(zb::kUnsupported, "moe_permute: E=%d (max %d)", E, kMaxExperts);
  const int64_t P = (int64_t)T * k;
  const int64_t need = ((P + (int64_t)E * (block - 1)) + block - 1) / block * block;
  ZB_REQUIRE(capacity >= need, "moe_permute: capacity %lld < %lld padded rows", (long long)capacity, (long long)need);
  ZB_REQUIRE(P < (1ll << 30), "moe_permute: %lld pairs", (long long)P);
  ZB_REQUIRE(hist && counts && offsets && sorted_pairs && position && (P == 0 || ids), "moe_permute: null pointer");
  PermuteParams p{ids, (int)P, E, block, capacity, hist, counts, offsets, sorted_pairs, position};
  p.groups = 1;
  const unsigned slices = (unsigned)std::max<int64_t>(1, (P + kPermPairs - 1) / kPermPairs);
  ZB_CUDA(zb::launch(moe_count_kernel, dim3(slices), dim3(kPermThreads), 0, stream, 1, p));
  if (int rc = zb::check_launch("moe_permute(count)")) return rc;
  ZB_CUDA(zb::launch(moe_scatter_kernel, dim3(slices), dim3(kPermThreads), 0, stream, 1, p));
  return zb::check_launch("moe_permute(scatter)");
}

ZB_API int zb_moe_permute_gather(const int32_t* ids, int T, int k, int E, int block, int64_t capacity, int32_t* hist,
                                 int32_t* counts, int32_t* offsets, int32_t* sorted_pairs, int32_t* position,
                                 const uint16_t* x, int64_t x_stride, int D, uint16_t* x_perm, cudaStream_t stream) {
  ZB_REQUIRE(T >= 0 && k > 0 && E > 0 && block > 0, "moe_permute_gather: bad sizes T=%d k=%d E=%d block=%d", T, k, E,
             block);
  if (E > kMaxExperts) return zb::fail(zb::kUnsupported, "moe_permute_gather: E=%d (max %d)", E, kMaxExperts);
  const int64_t P = (int64_t)T * k;
  const int64_t need = ((P + (int64_t)E * (block - 1)) + block - 1) / block * block;
  ZB_REQUIRE(capacity >= need, "moe_permute_gather: capacity %lld < %lld padded rows", (long long)capacity,
             (long long)need);
  ZB_REQUIRE(P < (1ll << 30), "moe_permute_gather: %lld pairs", (long long)P);
  ZB_REQUIRE(hist && counts && offsets && sorted_pairs && position && x_perm && (P == 0 || (ids && x)),
             "moe_permute_gather: null pointer");
  ZB_REQUIRE(D > 0 && D % 8 == 0 && x_stride >= D && x_stride % 8 == 0, "moe_permute_gather: D=%d, x_stride %lld", D,
             (long long)x_stride);
  ZB_REQUIRE_ALIGNED(x, 16, "x");
  ZB_REQUIRE_ALIGNED(x_perm, 16, "x_perm");
  PermuteParams p{ids, (int)P, E, block, capacity, hist, counts, offsets, sorted_pairs, position,
                  reinterpret_cast<const __nv_bfloat16*>(x), x_stride, k, D, reinterpret_cast<__nv_bfloat16*>(x_perm),
                  1};
  const int64_t slices = std::max<int64_t>(1, (P + kPermPairs - 1) / kPermPairs);
  // blocks per slice: about two per SM over the whole grid, a power of two dividing the slice's 256 pairs
  while (p.groups < 32 && slices * p.groups * 2 <= 2 * zb::sm_count()) p.groups *= 2;
  ZB_CUDA(zb::launch(moe_count_kernel, dim3((unsigned)slices), dim3(kPermThreads), 0, stream, 1, p));
  if (int rc = zb::check_launch("moe_permute_gather(count)")) return rc;
  ZB_CUDA(zb::launch(moe_scatter_kernel, dim3((unsigned)(slices * p.groups)), dim3(kPermThreads), 0, stream, 1, p));
  return zb::check_launch("moe_permute_gather(scatter + gather)");
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
  const int64_t grid = std::min<int64_t>((rows + 7) / 8, (int64_t)zb::sm_count() * 8);  // a warp per row
  ZB_CUDA(zb::launch(moe_gather_kernel, dim3((unsigned)grid), dim3(256), 0, stream, 1, p));
  return zb::check_launch("moe_gather");
}

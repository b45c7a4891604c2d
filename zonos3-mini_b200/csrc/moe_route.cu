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

constexpr int kRouterTokens = 16;           // tokens of one router CTA (one m16 tile)
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

constexpr int kRouterThreads = 128;  // 4 warps, each a quarter of the experts
constexpr int kRouterStages = 4;
constexpr int kRow = kChunk + kPad;  // smem row length (elements)

// One CTA routes 16 tokens. A 4-stage cp.async pipeline streams K chunks of x [16 x 64], the router weight
// [NE x 64] and the norm weight [64]; warp w computes the logits of experts [w*8*NH, (w+1)*8*NH) for the 16 tokens
// with mma.sync m16n8k16 (bf16 in, fp32 accumulate), the A fragments scaled by inv_rms * norm weight in registers.
// The inverse RMS of the tokens comes first (4 tokens per warp, 8 independent 16-byte loads per lane in flight),
// and every warp then selects the top-k of 4 tokens.
template <int NH>  // n-tiles (8 experts each) per warp: E <= 32 * NH
__global__ void __launch_bounds__(kRouterThreads) moe_router_kernel(RouterParams p) {
  constexpr int NE = 32 * NH;  // experts covered by the CTA
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __nv_bfloat16* a_s = reinterpret_cast<__nv_bfloat16*>(smem_raw);               // [stages][16][kRow]
  __nv_bfloat16* b_s = a_s + kRouterStages * kRouterTokens * kRow;                // [stages][NE][kRow]
  __nv_bfloat16* w_s = b_s + kRouterStages * NE * kRow;                            // [stages][kChunk]
  float* rms_s = reinterpret_cast<float*>(w_s + kRouterStages * kChunk);          // [16]
  float* logit_s = rms_s + kRouterTokens;                                         // [16][NE + 1]
  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  const int tok0 = blockIdx.x * kRouterTokens;
  const int n_chunks = p.D / kChunk;

  auto load_chunk = [&](int chunk, int stage) {
    const int k0 = chunk * kChunk;
    __nv_bfloat16* a = a_s + stage * kRouterTokens * kRow;
    __nv_bfloat16* b = b_s + stage * NE * kRow;
    for (int idx = tid; idx < kRouterTokens * (kChunk / 8); idx += kRouterThreads) {
      const int r = idx / (kChunk / 8), c = (idx % (kChunk / 8)) * 8;
      const int t = tok0 + r;
      cp_async16(a + r * kRow + c, p.x + (int64_t)(t < p.T ? t : 0) * p.x_stride + k0 + c, t < p.T);
    }
    for (int idx = tid; idx < NE * (kChunk / 8); idx += kRouterThreads) {
      const int e = idx / (kChunk / 8), c = (idx % (kChunk / 8)) * 8;
      cp_async16(b + e * kRow + c, p.w_router + (int64_t)(e < p.E ? e : 0) * p.D + k0 + c, e < p.E);
    }
    if (tid < kChunk / 8) cp_async16(w_s + stage * kChunk + tid * 8, p.norm_w + k0 + tid * 8, true);
  };

  // prologue: start the first stages while the inverse RMS is computed
#pragma unroll
  for (int s = 0; s < kRouterStages - 1; ++s) {
    if (s < n_chunks) load_chunk(s, s);
    cp_async_commit();
  }
  for (int r = warp; r < kRouterTokens; r += kRouterThreads / 32) {
    const int t = tok0 + r;
    float ss = 0.f;
    if (t < p.T) {
      const __nv_bfloat16* row = p.x + (int64_t)t * p.x_stride;
      for (int c0 = lane * 8; c0 < p.D; c0 += 256 * 8) {
        float v[8][8];
#pragma unroll
        for (int u = 0; u < 8; ++u)
          if (c0 + u * 256 < p.D) zb::ld_bf16x8(row + c0 + u * 256, v[u]);
#pragma unroll
        for (int u = 0; u < 8; ++u)
          if (c0 + u * 256 < p.D)
#pragma unroll
            for (int j = 0; j < 8; ++j) ss = fmaf(v[u][j], v[u][j], ss);
      }
    }
    ss = zb::warp_sum(ss);
    if (lane == 0) rms_s[r] = rsqrtf(ss / (float)p.D + p.eps);
  }
  __syncthreads();

  const int nbase = warp * NH;  // first n-tile of this warp
  const int g = lane >> 2, tq = lane & 3;
  const float s_lo = rms_s[g], s_hi = rms_s[g + 8];
  float acc[NH][4];
#pragma unroll
  for (int n = 0; n < NH; ++n) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.f;

  for (int chunk = 0; chunk < n_chunks; ++chunk) {
    const int stage = chunk % kRouterStages;
    cp_async_wait<kRouterStages - 2>();
    __syncthreads();
    // refill the stage consumed in the previous iteration
    const int next = chunk + kRouterStages - 1;
    if (next < n_chunks) load_chunk(next, next % kRouterStages);
    cp_async_commit();
    if (nbase * 8 >= p.E) continue;  // this warp's experts are all padding
    const __nv_bfloat16* a = a_s + stage * kRouterTokens * kRow;
    const __nv_bfloat16* b = b_s + stage * NE * kRow;
    const __nv_bfloat16* wv = w_s + stage * kChunk;
#pragma unroll
    for (int kk = 0; kk < kChunk; kk += 16) {
      const uint32_t w0 = *reinterpret_cast<const uint32_t*>(wv + kk + 2 * tq);
      const uint32_t w1 = *reinterpret_cast<const uint32_t*>(wv + kk + 2 * tq + 8);
      uint32_t af[4];
      af[0] = scale_bf16x2(*reinterpret_cast<const uint32_t*>(a + g * kRow + kk + 2 * tq), s_lo, w0);
      af[1] = scale_bf16x2(*reinterpret_cast<const uint32_t*>(a + (g + 8) * kRow + kk + 2 * tq), s_hi, w0);
      af[2] = scale_bf16x2(*reinterpret_cast<const uint32_t*>(a + g * kRow + kk + 2 * tq + 8), s_lo, w1);
      af[3] = scale_bf16x2(*reinterpret_cast<const uint32_t*>(a + (g + 8) * kRow + kk + 2 * tq + 8), s_hi, w1);
#pragma unroll
      for (int n = 0; n < NH; ++n) {
        const int e = (nbase + n) * 8 + g;
        uint32_t bf[2];
        bf[0] = *reinterpret_cast<const uint32_t*>(b + e * kRow + kk + 2 * tq);
        bf[1] = *reinterpret_cast<const uint32_t*>(b + e * kRow + kk + 2 * tq + 8);
        mma_bf16_16816(acc[n], af, bf);
      }
    }
  }
  cp_async_wait<0>();
  // logits rounded to bf16 (the router_linear output dtype)
#pragma unroll
  for (int n = 0; n < NH; ++n) {
    const int c0 = (nbase + n) * 8 + 2 * tq;
    logit_s[g * (NE + 1) + c0] = zb::bf16_round(acc[n][0]);
    logit_s[g * (NE + 1) + c0 + 1] = zb::bf16_round(acc[n][1]);
    logit_s[(g + 8) * (NE + 1) + c0] = zb::bf16_round(acc[n][2]);
    logit_s[(g + 8) * (NE + 1) + c0 + 1] = zb::bf16_round(acc[n][3]);
  }
  __syncthreads();
  for (int r = warp; r < kRouterTokens; r += kRouterThreads / 32) {
    const int t = tok0 + r;
    if (t >= p.T) break;
    const float* lrow = logit_s + r * (NE + 1);
    if (p.logits_out) {
      for (int e = lane; e < p.E; e += 32) p.logits_out[(int64_t)t * p.E + e] = __float2bfloat16_rn(lrow[e]);
    }
    select_token([&](int e) { return lrow[e]; }, p.bias, p.E, p.k, p.mode, p.renorm, p.ids + (int64_t)t * p.k,
                 p.weights + (int64_t)t * p.k);
  }
}

template <int NH>
int launch_router(const RouterParams& p, cudaStream_t stream) {
  constexpr int NE = 32 * NH;
  const size_t smem = (size_t)kRouterStages * (kRouterTokens + NE) * kRow * 2 + kRouterStages * kChunk * 2 +
                      kRouterTokens * 4 + (size_t)kRouterTokens * (NE + 1) * 4;
  auto kernel = moe_router_kernel<NH>;
  if (smem > 48 * 1024) ZB_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  const unsigned grid = (unsigned)((p.T + kRouterTokens - 1) / kRouterTokens);
  kernel<<<grid, kRouterThreads, smem, stream>>>(p);
  return zb::check_launch("moe_router");
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
};

// Pass 1: the expert histogram of each 256-pair slice (order-free shared-memory atomics).
__global__ void __launch_bounds__(kPermThreads) moe_count_kernel(PermuteParams p) {
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
  __shared__ int32_t base[kMaxExperts];      // write cursor of this slice per expert
  __shared__ int32_t seg[kMaxExperts + 1];   // padded segment starts
  __shared__ int32_t total[kMaxExperts];
  __shared__ int32_t wcount[kPermThreads / 32][kMaxExperts];
  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  const int nslices = gridDim.x, me = blockIdx.x;
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
  if (ok) {
    int pos = seg[e] + base[e] + rank;
    for (int w = 0; w < warp; ++w) pos += wcount[w][e];
    p.sorted_pairs[pos] = i;
    p.position[i] = pos;
  } else if (live) {
    p.position[i] = -1;
  }
  // padding rows of every segment (expert e handled by slice e % nslices), then rows past the last segment
  for (int x = me; x < p.E; x += nslices) {
    for (int r = seg[x] + total[x] + tid; r < seg[x + 1]; r += kPermThreads) p.sorted_pairs[r] = -1;
  }
  for (int64_t r = seg[p.E] + (int64_t)me * kPermThreads + tid; r < p.capacity; r += (int64_t)nslices * kPermThreads)
    p.sorted_pairs[r] = -1;
  if (me == 0) {
    for (int x = tid; x < p.E; x += kPermThreads) p.counts[x] = total[x];
    for (int x = tid; x <= p.E; x += kPermThreads) p.offsets[x] = seg[x];
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
    for (int s0 = 0; s0 < p.k; s0 += 8) {  // up to 8 slot rows in flight, summed in slot order
      uint4 raw[8];
#pragma unroll
      for (int s = 0; s < 8; ++s)
        if (s0 + s < p.k) raw[s] = *reinterpret_cast<const uint4*>(p.y + (t * p.k + s0 + s) * p.D + c);
#pragma unroll
      for (int s = 0; s < 8; ++s) {
        if (s0 + s < p.k) {
          float v[8];
          zb::ld_bf16x8(reinterpret_cast<const __nv_bfloat16*>(&raw[s]), v);
#pragma unroll
          for (int j = 0; j < 8; ++j) acc[j] += v[j];
        }
      }
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
  const int nh = (E + 31) / 32;
  if (nh <= 1) return launch_router<1>(p, stream);
  if (nh <= 2) return launch_router<2>(p, stream);
  return launch_router<4>(p, stream);
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
  const unsigned slices = (unsigned)std::max<int64_t>(1, (P + kPermPairs - 1) / kPermPairs);
  moe_count_kernel<<<slices, kPermThreads, 0, stream>>>(p);
  if (int rc = zb::check_launch("moe_permute(count)")) return rc;
  moe_scatter_kernel<<<slices, kPermThreads, 0, stream>>>(p);
  return zb::check_launch("moe_permute(scatter)");
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

// The TTS sampler: next audio codes from per-codebook logits, on the device without a host round trip.
//
// Reference: sample_tts (model/src/zonos3/tts/sampler.py:159-372) as the server calls it once per decode step
// (servers/sgl scheduler -> sample_tts on the head's softcapped logits [B, C, V]). Per (request b, codebook c) row,
// in the reference's order:
//   1. ids that may not be sampled -> -inf: the audio padding id, every special id (>= codebook_size) but the
//      request's stop id, ordinary ids past the codebook's own size, the stop id while stop_blocked[b, c]
//      (sampler.py:238-251); then + stop_bias[b] on the stop id (:252-253);
//   2. repetition penalty over the request's recent ids of this codebook: a repeated id's logit is divided by the
//      penalty when positive, multiplied otherwise (apply_repetition_penalty, :83-108);
//   3. greedy (every temperature <= 0: argmax, first index of the maximum) or: / temperature, top-k (keep logits
//      >= the k-th largest), softmax, top-p (keep an id when the mass before it in a stable descending order --
//      larger probabilities, then equal ones of lower index -- is <= top_p), min-p (keep p >= min_p * max p),
//      renormalisation after each filter
//      (clamped at 1e-8), a row without mass falls back to its argmax, and one multinomial draw (:288-349).
// top_k / top_p / min_p are the batch's (min, max, max) as the reference reduces them on the host.
// The draw uses Philox4x32-10 (Salmon et al., SC'11) keyed by `seed`, counter (row, offset + *offset_dev when a
// device counter is given, so a captured decode step draws fresh numbers on every replay): a different random
// stream from torch.multinomial's, so sampled ids match the reference in distribution, not draw for draw.
//
// One CTA of 256 threads per row; the row's logits live in shared memory (V <= kMaxVocab). With a top-k of at most
// 512 the k-th largest logit comes from a 4-pass radix select and the survivors are sorted (sample_sorted_topk);
// otherwise the k-th largest logit and the top-p cut-off are found by bisection on the float bits with
// block-wide counts / sums.
#include "common.cuh"

namespace {

constexpr int kThreads = 256;
constexpr int kMaxVocab = 16384;

struct SamplerParams {
  const void* logits;  // [B, C, V]: row (b, c) at b * batch_stride + c * row_stride elements; bf16 or fp32
  int logits_fp32;
  float softcap;  // > 0: logits = softcap * tanh(logits / softcap) first (the head's soft cap)
  int64_t row_stride, batch_stride;
  int B, C, V;
  const float* temperatures;  // [B]
  int greedy;                 // every temperature <= 0
  int top_k;                  // 0 or >= V: off
  float top_p;                // off unless in (0, 1)
  float min_p;                // off unless > 0
  int codebook_size, audio_pad_id;
  const int32_t* stop_ids;        // [B]
  const int32_t* codebook_sizes;  // [C] or null
  const uint8_t* stop_blocked;    // [B, C] or null
  const float* stop_bias;         // [B] or null
  const int32_t* rep_ids;         // [B, C, W] or null (ids outside [0, V) ignored)
  int W;
  const float* rep_penalties;  // [B] or null
  uint64_t seed, offset;
  const uint64_t* offset_dev;  // [1] or null: added to `offset` (a step counter a captured graph advances)
  int text_vocab;
  int32_t* out;      // [B, C + 1]
  float* probs_out;  // [B * C, V] or null: the final distribution (one-hot on greedy rows)
};

// ---------------------------------------------------------------------------------------------------- Philox

__device__ __forceinline__ void philox_round(uint32_t (&c)[4], uint32_t k0, uint32_t k1) {
  const uint32_t m0 = 0xD2511F53u, m1 = 0xCD9E8D57u;  // Philox4x32 multipliers (Salmon et al. 2011)
  const uint32_t hi0 = __umulhi(m0, c[0]), lo0 = m0 * c[0];
  const uint32_t hi1 = __umulhi(m1, c[2]), lo1 = m1 * c[2];
  const uint32_t n0 = hi1 ^ c[1] ^ k0, n2 = hi0 ^ c[3] ^ k1;
  c[0] = n0;
  c[1] = lo1;
  c[2] = n2;
  c[3] = lo0;
}

// First 32-bit output of Philox4x32-10 for counter (ctr_lo, ctr_hi) under key `key`.
__device__ uint32_t philox(uint64_t key, uint64_t ctr_lo, uint64_t ctr_hi) {
  uint32_t c[4] = {(uint32_t)ctr_lo, (uint32_t)(ctr_lo >> 32), (uint32_t)ctr_hi, (uint32_t)(ctr_hi >> 32)};
  uint32_t k0 = (uint32_t)key, k1 = (uint32_t)(key >> 32);
  const uint32_t w0 = 0x9E3779B9u, w1 = 0xBB67AE85u;  // Weyl key increments (Salmon et al. 2011)
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    philox_round(c, k0, k1);
    k0 += w0;
    k1 += w1;
  }
  return c[0];
}

// ---------------------------------------------------------------------------------------------------- block ops

__device__ __forceinline__ float block_sum(float v, float* red) {
  v = zb::warp_sum(v);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  __syncthreads();  // red is reused
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = lane < kThreads / 32 ? red[lane] : 0.f;
  return zb::warp_sum(t);
}

__device__ __forceinline__ int block_count(int v, float* red) {
  for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  int* r = reinterpret_cast<int*>(red);
  __syncthreads();
  if (lane == 0) r[warp] = v;
  __syncthreads();
  int t = lane < kThreads / 32 ? r[lane] : 0;
  for (int off = 16; off > 0; off >>= 1) t += __shfl_xor_sync(0xffffffffu, t, off);
  return t;
}

// (value, index) of the maximum, lowest index among equal maxima (-inf rows: index 0).
__device__ __forceinline__ void block_argmax(const float* x, int V, float* red, float& best, int& best_i) {
  float b = -INFINITY;
  int bi = 0x7fffffff;
  for (int i = threadIdx.x; i < V; i += kThreads) {
    if (x[i] > b || (x[i] == b && i < bi)) {
      b = x[i];
      bi = i;
    }
  }
  for (int off = 16; off > 0; off >>= 1) {
    const float ob = __shfl_xor_sync(0xffffffffu, b, off);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
    if (ob > b || (ob == b && oi < bi)) {
      b = ob;
      bi = oi;
    }
  }
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  int* ri = reinterpret_cast<int*>(red) + 32;
  __syncthreads();
  if (lane == 0) {
    red[warp] = b;
    ri[warp] = bi;
  }
  __syncthreads();
  b = lane < kThreads / 32 ? red[lane] : -INFINITY;
  bi = lane < kThreads / 32 ? ri[lane] : 0x7fffffff;
  for (int off = 16; off > 0; off >>= 1) {
    const float ob = __shfl_xor_sync(0xffffffffu, b, off);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
    if (ob > b || (ob == b && oi < bi)) {
      b = ob;
      bi = oi;
    }
  }
  best = b;
  best_i = bi == 0x7fffffff ? 0 : bi;
}

// Order-preserving map of a float to an unsigned key (larger float -> larger key).
__device__ __forceinline__ uint32_t ordered(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

constexpr int kMaxCand = 1024;  // survivors of top-k that the sorted path holds (k <= kSortedTopK, plus ties)
constexpr int kSortedTopK = 512;

// Inclusive block-wide scan of one int per thread (warp totals through `wsum`, 8 ints).
__device__ __forceinline__ int block_scan_incl(int v, int* wsum) {
  const int lane = threadIdx.x % 32, warp = threadIdx.x / 32;
  for (int off = 1; off < 32; off <<= 1) {
    const int o = __shfl_up_sync(0xffffffffu, v, off);
    if (lane >= off) v += o;
  }
  __syncthreads();
  if (lane == 31) wsum[warp] = v;
  __syncthreads();
  for (int w = 0; w < warp; ++w) v += wsum[w];
  return v;
}
__device__ __forceinline__ float block_scan_incl_f(float v, float* wsum) {
  const int lane = threadIdx.x % 32, warp = threadIdx.x / 32;
  for (int off = 1; off < 32; off <<= 1) {
    const float o = __shfl_up_sync(0xffffffffu, v, off);
    if (lane >= off) v += o;
  }
  __syncthreads();
  if (lane == 31) wsum[warp] = v;
  __syncthreads();
  for (int w = 0; w < warp; ++w) v += wsum[w];
  return v;
}

// The tail of sample_sorted_topk in warp 0 alone (no block barriers), for `count` <= 64 candidates that hold every
// survivor of the top k (candidates in any order; those past the k-th largest are dropped here): the candidates,
// NS per lane (position j = 32 slot + lane), bitonic-sorted by (logit descending, index ascending) with shuffles;
// the survivors are the positions whose logit is >= the k-th largest (ties at the cut all kept); then the same
// softmax, top-p, min-p, empty-row fallback and draw as the block version, with warp scans in position order. The
// other warps only help zero the probability row when one is written.
template <int NS>  // 2: up to 64 candidates
__device__ bool sorted_tail_warp(const SamplerParams& p, const float* cand_v, const int* cand_i, int count, int row,
                                 int c, int32_t* out, float* probs) {
  static_assert(NS == 2, "the sort pairs slots only at stride 32");
  const int tid = threadIdx.x, lane = tid % 32;
  if (probs) {
    for (int i = tid; i < p.V; i += kThreads) probs[i] = 0.f;
    __syncthreads();
  }
  if (tid >= 32) return true;
  auto before = [](float va, int ia, float vb, int ib) { return va > vb || (va == vb && ia < ib); };
  float v[NS];
  int id[NS];
#pragma unroll
  for (int s = 0; s < NS; ++s) {
    const int j = 32 * s + lane;
    v[s] = j < count ? cand_v[j] : -INFINITY;
    id[s] = j < count ? cand_i[j] : 0x7fffffff;
  }
  auto cas = [&](float& va, int& ia, float& vb, int& ib, bool desc) {  // a is the lower position
    if (before(vb, ib, va, ia) == desc) {
      const float tv = va;
      const int ti = ia;
      va = vb;
      ia = ib;
      vb = tv;
      ib = ti;
    }
  };
#pragma unroll
  for (int size = 2; size <= 32 * NS; size <<= 1) {
#pragma unroll
    for (int stride = size / 2; stride > 0; stride >>= 1) {
      if (stride == 32) {  // partner in the other slot of the same lane: the run of 64 positions
        cas(v[0], id[0], v[1], id[1], (lane & size) == 0);
      } else {
#pragma unroll
        for (int s = 0; s < NS; ++s) {
          const int j = 32 * s + lane;
          const float ov = __shfl_xor_sync(0xffffffffu, v[s], stride);
          const int oi = __shfl_xor_sync(0xffffffffu, id[s], stride);
          const bool desc = (j & size) == 0;  // this run sorts in "before" order
          const bool take = (j & stride) == 0 ? before(ov, oi, v[s], id[s]) == desc   // lower: the run's pick
                                              : before(v[s], id[s], ov, oi) == desc;  // upper: the other one
          if (take) {
            v[s] = ov;
            id[s] = oi;
          }
        }
      }
    }
  }
  // survivors: positions < total, total = k plus the ties of the k-th largest logit that follow it
  const int k = min(p.top_k, count);
  const float kth = __shfl_sync(0xffffffffu, v[(k - 1) / 32], (k - 1) % 32);
  int total = 0;
#pragma unroll
  for (int s = 0; s < NS; ++s) total += __popc(__ballot_sync(0xffffffffu, 32 * s + lane < count && v[s] >= kth));
  auto scan = [&](const float* e, float* run) {  // inclusive cumulative sums in position order
    float carry = 0.f;
#pragma unroll
    for (int s = 0; s < NS; ++s) {
      float x = e[s];
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const float o = __shfl_up_sync(0xffffffffu, x, off);
        if (lane >= off) x += o;
      }
      run[s] = x + carry;
      carry += __shfl_sync(0xffffffffu, x, 31);
    }
  };
  auto wsum = [&](const float* e) {
    float t = 0.f;
#pragma unroll
    for (int s = 0; s < NS; ++s) t += e[s];
    return zb::warp_sum(t);
  };
  const float mx = __shfl_sync(0xffffffffu, v[0], 0);
  float e[NS];
#pragma unroll
  for (int s = 0; s < NS; ++s) e[s] = (32 * s + lane < total && mx != -INFINITY) ? expf(v[s] - mx) : 0.f;
  const float sum = wsum(e);
#pragma unroll
  for (int s = 0; s < NS; ++s) e[s] = sum > 0.f ? e[s] / sum : 0.f;
  if (p.top_p > 0.f && p.top_p < 1.f) {
    float run[NS];
    scan(e, run);
#pragma unroll
    for (int s = 0; s < NS; ++s)
      if (run[s] - e[s] > p.top_p) e[s] = 0.f;  // the mass before it
    const float ksum = fmaxf(wsum(e), 1e-8f);
#pragma unroll
    for (int s = 0; s < NS; ++s) e[s] = e[s] / ksum;
  }
  if (p.min_p > 0.f) {
    const float cut = p.min_p * __shfl_sync(0xffffffffu, e[0], 0);  // the largest probability sits first
#pragma unroll
    for (int s = 0; s < NS; ++s)
      if (e[s] < cut) e[s] = 0.f;
    const float ksum = fmaxf(wsum(e), 1e-8f);
#pragma unroll
    for (int s = 0; s < NS; ++s) e[s] = e[s] / ksum;
  }
  float mass = wsum(e);
  if (!(mass > 0.f)) {  // a row without mass: one-hot at the argmax (the first survivor)
#pragma unroll
    for (int s = 0; s < NS; ++s) e[s] = (s == 0 && lane == 0) ? 1.f : 0.f;
    mass = 1.f;
  }
  if (probs) {
#pragma unroll
    for (int s = 0; s < NS; ++s)
      if (32 * s + lane < total) probs[id[s]] = e[s];
  }
  const uint64_t counter = p.offset + (p.offset_dev ? *p.offset_dev : 0ull);
  const float u = (float)(philox(p.seed, (uint64_t)row, counter) >> 8) * (1.0f / 16777216.0f);
  const float target = u * mass;
  float run[NS];
  scan(e, run);
  int pick = 0;
  bool found = false;
#pragma unroll
  for (int s = 0; s < NS; ++s) {
    const unsigned m = __ballot_sync(0xffffffffu, target < run[s] && e[s] > 0.f);
    if (!found && m) {
      pick = 32 * s + __ffs(m) - 1;
      found = true;
    }
  }
  int chosen = 0;
#pragma unroll
  for (int s = 0; s < NS; ++s) {
    const int o = __shfl_sync(0xffffffffu, id[s], pick & 31);
    if (pick / 32 == s) chosen = o;
  }
  if (lane == 0) out[c] = chosen;
  return true;
}

// The sampling path after a small top-k (temperature already applied to x): the k-th largest logit by a 4-pass
// radix select, the survivors (logit >= it) compacted in index order and bitonic-sorted by (logit descending,
// index ascending) -- the order of the reference's stable descending sort --, then softmax, top-p with the
// reference's rule (inclusive cumulative sum minus the id's own probability > top_p drops it), min-p, the
// empty-row fallback and the draw, all on the short sorted list (sorted_tail_warp in one warp for at most 64
// survivors). Returns false (nothing written) when more than kMaxCand ids tie into the top k.
__device__ bool sample_sorted_topk(const SamplerParams& p, float* x, int row, int c, int32_t* out, float* probs,
                                   float* cand_v, int* cand_i, int* ints, float* red) {
  const int V = p.V, tid = threadIdx.x;
  int* hist = ints;         // [256]
  int* wsum = ints + 256;   // [8]
  int* sel = ints + 264;    // [2]
  int* wsum2 = ints + 272;  // [8], the other scan buffer
  uint32_t prefix = 0u, pmask = 0u;
  int kk = p.top_k;
  hist[tid] = 0;
  __syncthreads();
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int i = tid; i < V; i += kThreads) {
      const uint32_t key = ordered(x[i]);
      if ((key & pmask) == prefix) atomicAdd(&hist[(key >> shift) & 255u], 1);
    }
    __syncthreads();
    const int v = hist[255 - tid];
    hist[255 - tid] = 0;  // each bin is read by its own thread only: cleared for the next pass
    // inclusive scan over the digits from the top (scan buffers alternate between passes, so the barrier that
    // guards a buffer's reuse is the previous pass's last one)
    int sc = v;
    const int lane = tid % 32, warp = tid / 32;
    for (int off = 1; off < 32; off <<= 1) {
      const int o = __shfl_up_sync(0xffffffffu, sc, off);
      if (lane >= off) sc += o;
    }
    int* ws = (shift & 8) ? wsum2 : wsum;
    if (lane == 31) ws[warp] = sc;
    __syncthreads();
    for (int w = 0; w < warp; ++w) sc += ws[w];  // ids whose digit is >= 255 - tid
    if (sc >= kk && sc - v < kk) {
      sel[0] = 255 - tid;
      sel[1] = sc - v;
    }
    __syncthreads();  // sel is read by every thread before the next pass's scan can write it again
    prefix |= (uint32_t)sel[0] << shift;
    pmask |= 255u << shift;
    kk -= sel[1];
  }
  __syncthreads();  // sel and the scan buffers are free for the compaction's scan
  // compact the survivors in index order (contiguous chunks per thread)
  const int chunk = (V + kThreads - 1) / kThreads;
  const int cb = min(tid * chunk, V), ce = min(cb + chunk, V);
  int mine = 0;
  for (int i = cb; i < ce; ++i) mine += ordered(x[i]) >= prefix ? 1 : 0;
  const int incl = block_scan_incl(mine, wsum);
  __shared__ int total_s;
  if (tid == kThreads - 1) total_s = incl;  // the last thread's inclusive count is the total
  __syncthreads();
  const int total = total_s;
  if (total > kMaxCand) return false;
  int pos = incl - mine;
  for (int i = cb; i < ce; ++i) {
    if (ordered(x[i]) >= prefix) {
      cand_v[pos] = x[i];
      cand_i[pos] = i;
      ++pos;
    }
  }
  if (total <= 64) {
    __syncthreads();  // the compacted survivors are in shared memory
    return sorted_tail_warp<2>(p, cand_v, cand_i, total, row, c, out, probs);
  }
  int P = 1;
  while (P < total) P <<= 1;
  for (int r = total + tid; r < P; r += kThreads) {
    cand_v[r] = -INFINITY;
    cand_i[r] = 0x7fffffff;
  }
  __syncthreads();
  // bitonic sort: "a before b" when a.v > b.v, or equal values and a.i < b.i
  for (int size = 2; size <= P; size <<= 1) {
    for (int stride = size / 2; stride > 0; stride >>= 1) {
      for (int t = tid; t < P / 2; t += kThreads) {
        const int i = 2 * t - (t & (stride - 1)), j = i + stride;
        const bool desc = (i & size) == 0;  // this run sorts in "before" order
        const float vi = cand_v[i], vj = cand_v[j];
        const int ii = cand_i[i], ij = cand_i[j];
        const bool j_before_i = vj > vi || (vj == vi && ij < ii);
        if (j_before_i == desc) {
          cand_v[i] = vj;
          cand_v[j] = vi;
          cand_i[i] = ij;
          cand_i[j] = ii;
        }
      }
      __syncthreads();
    }
  }
  // softmax over the sorted survivors (4 consecutive positions per thread)
  const float mx = cand_v[0];
  const int q0 = 4 * tid;
  float e[4], part = 0.f;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int r = q0 + k;
    e[k] = (r < total && mx != -INFINITY) ? expf(cand_v[r] - mx) : 0.f;
    part += e[k];
  }
  const float sum = block_sum(part, red);
#pragma unroll
  for (int k = 0; k < 4; ++k) e[k] = sum > 0.f ? e[k] / sum : 0.f;
  if (p.top_p > 0.f && p.top_p < 1.f) {
    float loc = e[0] + e[1] + e[2] + e[3];
    float run = block_scan_incl_f(loc, reinterpret_cast<float*>(wsum)) - loc;
    float kept = 0.f;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      run += e[k];                       // the inclusive cumulative sum at this position
      if (run - e[k] > p.top_p) e[k] = 0.f;  // minus its own probability: the mass before it
      kept += e[k];
    }
    const float ksum = fmaxf(block_sum(kept, red), 1e-8f);
#pragma unroll
    for (int k = 0; k < 4; ++k) e[k] = e[k] / ksum;
  }
  if (p.min_p > 0.f) {
    __shared__ float top_s;
    if (tid == 0) top_s = e[0];  // the largest probability sits first
    __syncthreads();
    const float cut = p.min_p * top_s;
    float kept = 0.f;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      if (e[k] < cut) e[k] = 0.f;
      kept += e[k];
    }
    const float ksum = fmaxf(block_sum(kept, red), 1e-8f);
#pragma unroll
    for (int k = 0; k < 4; ++k) e[k] = e[k] / ksum;
  }
  float mass = block_sum(e[0] + e[1] + e[2] + e[3], red);
  if (!(mass > 0.f)) {  // a row without mass: one-hot at the argmax (the first survivor)
#pragma unroll
    for (int k = 0; k < 4; ++k) e[k] = q0 + k == 0 ? 1.f : 0.f;
    mass = 1.f;
  }
  if (probs) {
    for (int i = tid; i < V; i += kThreads) probs[i] = 0.f;
    __syncthreads();
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      if (q0 + k < total) probs[cand_i[q0 + k]] = e[k];
    }
  }
  // the draw over the sorted list
  const uint64_t counter = p.offset + (p.offset_dev ? *p.offset_dev : 0ull);
  const float u = (float)(philox(p.seed, (uint64_t)row, counter) >> 8) * (1.0f / 16777216.0f);
  const float target = u * mass;
  const float loc = e[0] + e[1] + e[2] + e[3];
  float run = block_scan_incl_f(loc, reinterpret_cast<float*>(wsum)) - loc;
  int pick = -1;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    run += e[k];
    if (pick < 0 && target < run && e[k] > 0.f) pick = q0 + k;
  }
  int* slot = sel;
  __syncthreads();
  if (tid == 0) *slot = 0x7fffffff;
  __syncthreads();
  if (pick >= 0) atomicMin(slot, pick);
  __syncthreads();
  if (tid == 0) out[c] = cand_i[*slot == 0x7fffffff ? 0 : *slot];
  return true;
}

__global__ void __launch_bounds__(kThreads) sample_tts_kernel(SamplerParams p) {
  zb::pdl_enter();
  extern __shared__ __align__(16) float x[];  // [V] logits, then probabilities
  __shared__ float red[64];
  __shared__ unsigned repeated[kMaxVocab / 32];
  const int row = blockIdx.x, b = row / p.C, c = row % p.C, V = p.V, tid = threadIdx.x;

  // 1. load, invalid ids, stop bias
  const int stop = p.stop_ids[b];
  const int limit = p.codebook_sizes ? p.codebook_sizes[c] : p.codebook_size;
  const bool blocked = p.stop_blocked && p.stop_blocked[(int64_t)b * p.C + c];
  const float bias = p.stop_bias ? p.stop_bias[b] : 0.f;
  const float inv_cap = p.softcap > 0.f ? 1.0f / p.softcap : 0.f;
  for (int i = tid; i < V; i += kThreads) {
    const int64_t at = (int64_t)b * p.batch_stride + (int64_t)c * p.row_stride + i;
    float v = p.logits_fp32 ? reinterpret_cast<const float*>(p.logits)[at]
                            : __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p.logits)[at]);
    if (p.softcap > 0.f) {
      // cap * tanh(x / cap) as torch evaluates it on the head's dtype: the division by a scalar as a multiply by
      // its reciprocal, each of the three ops rounded to bf16 for bf16 logits
      if (p.logits_fp32) {
        v = p.softcap * tanhf(v * inv_cap);
      } else {
        v = zb::bf16_round(p.softcap * zb::bf16_round(tanhf(zb::bf16_round(v * inv_cap))));
      }
    }
    const bool invalid = i == p.audio_pad_id || (i >= p.codebook_size && i != stop) ||
                         (i >= limit && i < p.codebook_size) || (blocked && i == stop);
    if (invalid) v = -INFINITY;
    if (i == stop) v += bias;
    x[i] = v;
  }
  // 2. repetition penalty
  if (p.rep_ids && p.rep_penalties && p.W > 0) {
    for (int i = tid; i < (V + 31) / 32; i += kThreads) repeated[i] = 0u;
    __syncthreads();
    const int32_t* ids = p.rep_ids + ((int64_t)b * p.C + c) * p.W;
    for (int w = tid; w < p.W; w += kThreads) {
      const int id = ids[w];
      if (id >= 0 && id < V) atomicOr(&repeated[id / 32], 1u << (id % 32));
    }
    __syncthreads();
    const float pen = fmaxf(p.rep_penalties[b], 1.f);
    for (int i = tid; i < V; i += kThreads) {
      if ((repeated[i / 32] >> (i % 32)) & 1u) x[i] = x[i] > 0.f ? x[i] / pen : x[i] * pen;
    }
  }
  __syncthreads();

  int32_t* out = p.out + (int64_t)b * (p.C + 1);
  if (c == 0 && tid == 0) out[p.C] = p.text_vocab;
  float* probs = p.probs_out ? p.probs_out + (int64_t)row * V : nullptr;
  if (p.greedy) {
    float best;
    int bi;
    block_argmax(x, V, red, best, bi);
    if (tid == 0) out[c] = bi;
    if (probs) {
      for (int i = tid; i < V; i += kThreads) probs[i] = i == bi ? 1.f : 0.f;
    }
    return;
  }

  // 3. temperature, top-k
  const float temp = fmaxf(p.temperatures[b], 1e-8f);
  for (int i = tid; i < V; i += kThreads) x[i] = x[i] / temp;
  __syncthreads();
  if (p.top_k > 0 && p.top_k <= kSortedTopK && p.top_k < V) {
    __shared__ float cand_v[kMaxCand];
    __shared__ int cand_i[kMaxCand];
    __shared__ int ints[280];
    if (sample_sorted_topk(p, x, row, c, out, probs, cand_v, cand_i, ints, red)) return;
  }
  if (p.top_k > 0 && p.top_k < V) {
    // the k-th largest logit: the largest key K with count(key >= K) >= k
    uint32_t lo = 0u, hi = 0xffffffffu;  // answer in [lo, hi]
    while (lo < hi) {
      const uint32_t mid = lo + (hi - lo) / 2 + 1;
      int cnt = 0;
      for (int i = tid; i < V; i += kThreads) cnt += ordered(x[i]) >= mid ? 1 : 0;
      if (block_count(cnt, red) >= p.top_k) lo = mid;
      else hi = mid - 1;
    }
    for (int i = tid; i < V; i += kThreads) {
      if (ordered(x[i]) < lo) x[i] = -INFINITY;
    }
    __syncthreads();
  }
  // the argmax after top-k (the fallback of a row without mass)
  float mx;
  int arg;
  block_argmax(x, V, red, mx, arg);
  // softmax
  float part = 0.f;
  for (int i = tid; i < V; i += kThreads) {
    const float e = mx == -INFINITY ? 0.f : expf(x[i] - mx);
    x[i] = e;
    part += e;
  }
  float total = block_sum(part, red);
  for (int i = tid; i < V; i += kThreads) x[i] = total > 0.f ? x[i] / total : 0.f;
  __syncthreads();
  // top-p: keep p_i when the mass strictly above p_i is <= top_p; the cut-off is the smallest value tau with
  // mass(> tau) <= top_p (bisection on the bits of non-negative floats)
  if (p.top_p > 0.f && p.top_p < 1.f) {
    uint32_t lo = 0u, hi = 0x7f800000u;
    while (lo < hi) {
      const uint32_t mid = lo + (hi - lo) / 2;
      float s = 0.f;
      for (int i = tid; i < V; i += kThreads) s += __float_as_uint(x[i]) > mid ? x[i] : 0.f;
      if (block_sum(s, red) <= p.top_p) hi = mid;
      else lo = mid + 1;
    }
    // ids equal to the cut-off value tau are kept in index order while the mass before them (everything above
    // tau, then the earlier ties) stays <= top_p: the reference's stable descending sort keeps ties in index order
    const float tau = __uint_as_float(lo);
    float above = 0.f;
    for (int i = tid; i < V; i += kThreads) above += x[i] > tau ? x[i] : 0.f;
    above = block_sum(above, red);
    const int chunk = (V + kThreads - 1) / kThreads;
    const int cb = min(tid * chunk, V), ce = min(cb + chunk, V);
    int ties = 0;
    for (int i = cb; i < ce; ++i) ties += x[i] == tau ? 1 : 0;
    int incl = ties;  // inclusive scan of the tie counts over the contiguous chunks
    const int lane = tid % 32, warp = tid / 32;
    for (int off = 1; off < 32; off <<= 1) {
      const int o = __shfl_up_sync(0xffffffffu, incl, off);
      if (lane >= off) incl += o;
    }
    int* wsum = reinterpret_cast<int*>(red) + 48;
    __syncthreads();
    if (lane == 31) wsum[warp] = incl;
    __syncthreads();
    int rank = incl - ties;
    for (int w = 0; w < warp; ++w) rank += wsum[w];
    for (int i = cb; i < ce; ++i) {
      if (x[i] == tau) {
        if (above + (float)rank * tau > p.top_p) x[i] = 0.f;
        ++rank;
      } else if (x[i] < tau) {
        x[i] = 0.f;
      }
    }
    __syncthreads();
    float kept = 0.f;
    for (int i = tid; i < V; i += kThreads) kept += x[i];
    const float sum = fmaxf(block_sum(kept, red), 1e-8f);
    for (int i = tid; i < V; i += kThreads) x[i] = x[i] / sum;
    __syncthreads();
  }
  if (p.min_p > 0.f) {
    float local = 0.f;
    for (int i = tid; i < V; i += kThreads) local = fmaxf(local, x[i]);
    local = zb::warp_max(local);
    __syncthreads();
    if (tid % 32 == 0) red[tid / 32] = local;
    __syncthreads();
    float top = 0.f;
    for (int w = 0; w < kThreads / 32; ++w) top = fmaxf(top, red[w]);
    const float cut = p.min_p * top;
    float kept = 0.f;
    for (int i = tid; i < V; i += kThreads) {
      if (x[i] < cut) x[i] = 0.f;
      kept += x[i];
    }
    const float sum = fmaxf(block_sum(kept, red), 1e-8f);
    for (int i = tid; i < V; i += kThreads) x[i] = x[i] / sum;
    __syncthreads();
  }
  // a row without mass: one-hot at the argmax
  float mass = 0.f;
  for (int i = tid; i < V; i += kThreads) mass += x[i];
  mass = block_sum(mass, red);
  if (!(mass > 0.f)) {
    for (int i = tid; i < V; i += kThreads) x[i] = i == arg ? 1.f : 0.f;
    mass = 1.f;
    __syncthreads();
  }
  if (probs) {
    for (int i = tid; i < V; i += kThreads) probs[i] = x[i];
  }
  // one draw: the first id whose inclusive prefix sum exceeds u * mass (contiguous chunks per thread)
  const uint64_t counter = p.offset + (p.offset_dev ? *p.offset_dev : 0ull);
  const float u = (float)(philox(p.seed, (uint64_t)row, counter) >> 8) * (1.0f / 16777216.0f);
  const float target = u * mass;
  const int chunk = (V + kThreads - 1) / kThreads;
  const int begin = min(tid * chunk, V), end = min(begin + chunk, V);
  float local = 0.f;
  for (int i = begin; i < end; ++i) local += x[i];
  // exclusive scan of the chunk sums
  float incl = local;
  const int lane = tid % 32, warp = tid / 32;
  for (int off = 1; off < 32; off <<= 1) {
    const float o = __shfl_up_sync(0xffffffffu, incl, off);
    if (lane >= off) incl += o;
  }
  __syncthreads();
  if (lane == 31) red[warp] = incl;
  __syncthreads();
  float before = 0.f;
  for (int w = 0; w < warp; ++w) before += red[w];
  float run = before + incl - local;
  int pick = -1;
  if (run <= target && target < run + local) {
    for (int i = begin; i < end; ++i) {
      run += x[i];
      if (target < run && x[i] > 0.f) {
        pick = i;
        break;
      }
    }
  }
  __syncthreads();
  int* slot = reinterpret_cast<int*>(red) + 40;
  if (tid == 0) *slot = 0x7fffffff;
  __syncthreads();
  if (pick >= 0) atomicMin(slot, pick);
  __syncthreads();
  if (tid == 0) out[c] = *slot == 0x7fffffff ? arg : *slot;  // rounding past the last id: the argmax
}

}  // namespace

ZB_API int zb_sample_tts(const void* logits, int logits_fp32, float softcap, int64_t row_stride, int64_t batch_stride,
                         int B, int C, int V,
                         const float* temperatures, int greedy, int top_k, float top_p, float min_p, int codebook_size,
                         int audio_pad_id, const int32_t* stop_ids, const int32_t* codebook_sizes,
                         const uint8_t* stop_blocked, const float* stop_bias, const int32_t* rep_ids, int W,
                         const float* rep_penalties, uint64_t seed, uint64_t offset, const uint64_t* offset_dev,
                         int text_vocab, int32_t* out, float* probs_out, cudaStream_t stream) {
  ZB_REQUIRE(B >= 0 && C > 0 && V > 0 && V <= kMaxVocab, "sample_tts: sizes B=%d C=%d V=%d (V <= %d)", B, C, V,
             kMaxVocab);
  if (B == 0) return zb::kOk;
  ZB_REQUIRE(logits && stop_ids && out && (greedy || temperatures), "sample_tts: null pointer");
  ZB_REQUIRE(row_stride >= V, "sample_tts: row_stride %lld < V %d", (long long)row_stride, V);
  ZB_REQUIRE(batch_stride >= (int64_t)(C - 1) * row_stride + V, "sample_tts: batch_stride %lld overlaps the rows",
             (long long)batch_stride);
  ZB_REQUIRE(0 < codebook_size && codebook_size < V && codebook_size <= audio_pad_id && audio_pad_id < V,
             "sample_tts: codebook_size %d / audio_pad_id %d for vocabulary %d", codebook_size, audio_pad_id, V);
  ZB_REQUIRE(W >= 0 && (W == 0 || rep_ids), "sample_tts: repetition window %d without ids", W);
  ZB_REQUIRE(softcap >= 0.f, "sample_tts: softcap %g", (double)softcap);
  SamplerParams p{logits, logits_fp32, softcap, row_stride, batch_stride, B, C, V, temperatures, greedy, top_k, top_p, min_p, codebook_size,
                  audio_pad_id, stop_ids, codebook_sizes, stop_blocked, stop_bias, rep_ids, W, rep_penalties, seed,
                  offset, offset_dev, text_vocab, out, probs_out};
  const size_t smem = (size_t)V * sizeof(float);
  if (smem > 48 * 1024) {
    ZB_CUDA(cudaFuncSetAttribute(sample_tts_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  }
  ZB_CUDA(zb::launch(sample_tts_kernel, dim3((unsigned)(B * C)), dim3(kThreads), smem, stream, 1, p));
  return zb::check_launch("sample_tts");
}

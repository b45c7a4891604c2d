// GQA decode attention over a slot-indexed KV cache, and the KV store that fills it.
//
// Reference: the global-attention layers' decode step — FlashAttention3's flash_attn_with_kvcache as the FA backend
// calls it (servers/sgl/src/zonos3_sgl/attention/fa.py:64-81, :171-212: one query row per request, causal, K/V
// looked up through the page table of token slots, cache_seqlens keys per request, softmax_scale = head_dim^-0.5)
// and MHAKVCache.store_kv / store_cache (servers/sgl/src/zonos3_sgl/kvcache/mha_pool.py:58-67,
// servers/sgl/src/zonos3_sgl/kernel/csrc/jit/store.cu:28-50: row i of k and v copied to slot out_loc[i]). The cache
// holds one token per page: k_cache / v_cache [slots, Hkv, hd] with `slot_stride` elements between two slots (the
// layer-first and the page-first pool layouts differ only in that stride).
//
// Head dim 128 (the model's attention) runs on the tensor cores: gqa_decode_tc_kernel below. Head dims 32 and 64
// (the tiny configurations) run on CUDA cores: a CTA per (request, KV head, split of the key range); 4 warps take
// 32-position tiles of the split in turn. A warp stages its tile's K and V rows in shared memory with cp.async (16-byte pieces, the slot of each row
// from the page table), then lane j scores position j against every query head of the group (fp32 dot products
// over the bf16 K row), the warp updates each head's running max and denominator (online softmax in base 2, the
// scale folded into log2(e)), and lanes, each owning hd / 32 dimensions, accumulate p * V for every head. The 4
// warps merge their (max, denominator, accumulator) through shared memory; with one split the CTA writes the
// normalised bf16 output, with several each split writes its partial to the workspace and a combine kernel merges
// them. fp32 throughout in this kernel (FA3 rounds P to bf16 before its P.V product, as the tensor-core kernel does;
// the difference is within bf16 tolerance).
#include <algorithm>

#include "common.cuh"
#include "tc.cuh"

namespace {

constexpr int kWarps = 4;
constexpr int kThreads = kWarps * 32;
constexpr int kTile = 32;  // key positions of a warp tile

// Dynamic shared memory of one CTA: the group's queries (fp32), each warp's K tile (rows padded by 16 bytes) and V
// tile (bf16), the warps' running max and denominator per head.
template <int HD, int G>
struct AttnSmem {
  static constexpr int KP = HD + 8;
  static constexpr size_t q = 0;
  static constexpr size_t k = q + (size_t)G * HD * 4;
  static constexpr size_t v = k + (size_t)kWarps * kTile * KP * 2;
  static constexpr size_t ml = v + (size_t)kWarps * kTile * HD * 2;
  static constexpr size_t total = ml + (size_t)2 * kWarps * G * 4;
  static_assert((size_t)kWarps * G * HD * 4 <= (size_t)kWarps * kTile * KP * 2, "warp merge fits the K tiles");
};

struct AttnParams {
  const __nv_bfloat16* q;  // [B, Hq, hd], request stride q_stride
  int64_t q_stride;
  const __nv_bfloat16* k_cache;  // slot s, head h at (s * slot_stride + h * hd)
  const __nv_bfloat16* v_cache;
  int64_t slot_stride;
  int64_t num_slots;          // slots of the cache; a table entry outside [0, num_slots) masks its key position
  const int32_t* page_table;  // [B, table_stride]: slot of each key position
  int64_t table_stride;
  const int32_t* seq_lens;  // [B] keys per request (0: the request's output is zero), clamped to max_seq_len
  int max_seq_len;          // columns of the page table
  int B, Hq, Hkv;
  float scale_log2;  // softmax_scale * log2(e)
  int splits;
  int split_len;  // key positions per split (a multiple of kTile)
  float* part;    // [B, Hq, splits, hd + 2]: accumulator, running max (base 2), denominator
  __nv_bfloat16* out;  // [B, Hq, hd], request stride out_stride
  int64_t out_stride;
  unsigned* status;  // device status word (a bounded wait that expired sets kStatusAttnDecodeTimeout)
  const __nv_bfloat16* gate;  // [B, Hq] gate logits (request stride gate_stride) or null
  int64_t gate_stride;
};

// out[b, h, d] = bf16(v), or with a gate bf16(bf16(v) * bf16(sigmoid(gate[b, h]))): the attention layer's output
// gate o * sigmoid(gater(x)) (zonos3.py:326, :383-385) at torch's bf16 rounding points.
__device__ __forceinline__ void store_out(const AttnParams& p, int64_t b, int h, int hd, int d, float v) {
  if (p.gate) {
    const float gl = __bfloat162float(p.gate[b * p.gate_stride + h]);
    v = zb::bf16_round(v) * zb::bf16_round(1.0f / (1.0f + expf(-gl)));
  }
  p.out[b * p.out_stride + (int64_t)h * hd + d] = __float2bfloat16_rn(v);
}

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(zb::smem_addr(dst)), "l"(src) : "memory");
}

template <int HD, int G>
__global__ void __launch_bounds__(kThreads) gqa_decode_kernel(AttnParams p) {
  zb::pdl_enter();
  using L = AttnSmem<HD, G>;
  constexpr int KP = L::KP;         // padded K row (bf16): conflict-free 16-byte row reads
  constexpr int DL = HD / 32;       // dimensions a lane owns in the P.V accumulation
  constexpr int CH = HD * 2 / 16;   // 16-byte pieces of a row
  extern __shared__ __align__(16) unsigned char smem_raw[];
  auto q_s = reinterpret_cast<float(*)[HD]>(smem_raw + L::q);
  auto k_s = reinterpret_cast<__nv_bfloat16(*)[kTile][KP]>(smem_raw + L::k);
  auto v_s = reinterpret_cast<__nv_bfloat16(*)[kTile][HD]>(smem_raw + L::v);
  auto m_s = reinterpret_cast<float(*)[G]>(smem_raw + L::ml);
  auto l_s = reinterpret_cast<float(*)[G]>(smem_raw + L::ml + (size_t)kWarps * G * 4);
  const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  const int len = min(max(p.seq_lens[b], 0), p.max_seq_len);
  const int begin = split * p.split_len, end = min(len, begin + p.split_len);

  for (int i = tid; i < G * HD; i += kThreads) {
    const int g = i / HD, d = i % HD;
    q_s[g][d] = __bfloat162float(p.q[(int64_t)b * p.q_stride + (int64_t)(kvh * G + g) * HD + d]);
  }
  __syncthreads();

  float m[G], l[G], acc[G][DL];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    m[g] = -INFINITY;
    l[g] = 0.f;
#pragma unroll
    for (int j = 0; j < DL; ++j) acc[g][j] = 0.f;
  }
  const int32_t* table = p.page_table + (int64_t)b * p.table_stride;
  for (int t0 = begin + warp * kTile; t0 < end; t0 += kWarps * kTile) {
    const int pos = t0 + lane;
    const int slot = pos < end ? table[pos] : -1;
    const bool valid = slot >= 0 && slot < p.num_slots;
    const unsigned live = __ballot_sync(0xffffffffu, valid);  // rows of the tile that hold a key
    // stage the tile: row r's 16-byte pieces, two rows per pass of the warp for HD = 128
    for (int i = lane; i < kTile * CH; i += 32) {
      const int r = i / CH, c = i % CH;
      const int rs = __shfl_sync(0xffffffffu, slot, r);  // every lane takes part in the shuffle
      if ((live >> r) & 1u) {
        const int64_t off = (int64_t)rs * p.slot_stride + (int64_t)kvh * HD + c * 8;
        cp_async16(&k_s[warp][r][c * 8], p.k_cache + off);
        cp_async16(&v_s[warp][r][c * 8], p.v_cache + off);
      }
    }
    asm volatile("cp.async.commit_group;\n cp.async.wait_group 0;" ::: "memory");
    __syncwarp();
    // scores of position `pos` for every head of the group
    float s[G];
#pragma unroll
    for (int g = 0; g < G; ++g) s[g] = 0.f;
    if (valid) {
#pragma unroll 4
      for (int c = 0; c < CH; ++c) {
        float kf[8];
        zb::ld_bf16x8(&k_s[warp][lane][c * 8], kf);
#pragma unroll
        for (int g = 0; g < G; ++g) {
          const float4 qa = *reinterpret_cast<const float4*>(&q_s[g][c * 8]);
          const float4 qb = *reinterpret_cast<const float4*>(&q_s[g][c * 8 + 4]);
          s[g] = fmaf(qa.x, kf[0], s[g]);
          s[g] = fmaf(qa.y, kf[1], s[g]);
          s[g] = fmaf(qa.z, kf[2], s[g]);
          s[g] = fmaf(qa.w, kf[3], s[g]);
          s[g] = fmaf(qb.x, kf[4], s[g]);
          s[g] = fmaf(qb.y, kf[5], s[g]);
          s[g] = fmaf(qb.z, kf[6], s[g]);
          s[g] = fmaf(qb.w, kf[7], s[g]);
        }
      }
    }
    // online softmax (base 2) and P.V
    float pr[G];
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const float x = valid ? s[g] * p.scale_log2 : -INFINITY;
      const float m_new = fmaxf(m[g], zb::warp_max(x));
      // 0 on the first live tile (m = -inf); 1 while no key has been seen (both -inf)
      const float corr = m_new == -INFINITY ? 1.f : exp2f(m[g] - m_new);
      pr[g] = valid ? exp2f(x - m_new) : 0.f;
      l[g] = l[g] * corr + zb::warp_sum(pr[g]);
      m[g] = m_new;
#pragma unroll
      for (int j = 0; j < DL; ++j) acc[g][j] *= corr;
    }
    const int rows = min(kTile, end - t0);
    for (int r = 0; r < rows; ++r) {
      if (!((live >> r) & 1u)) continue;  // a masked row was not staged (warp-uniform)
      float vf[DL];
      if constexpr (DL == 4) {
        zb::ld_bf16x4(&v_s[warp][r][lane * 4], vf);
      } else {
#pragma unroll
        for (int j = 0; j < DL; ++j) vf[j] = __bfloat162float(v_s[warp][r][lane * DL + j]);
      }
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float pg = __shfl_sync(0xffffffffu, pr[g], r);
#pragma unroll
        for (int j = 0; j < DL; ++j) acc[g][j] = fmaf(pg, vf[j], acc[g][j]);
      }
    }
    __syncwarp();  // the tile buffers are refilled next
  }

  // merge the warps: max, denominators and accumulators through shared memory (the K tiles are reused)
  if (lane == 0)
#pragma unroll
    for (int g = 0; g < G; ++g) {
      m_s[warp][g] = m[g];
      l_s[warp][g] = l[g];
    }
  __syncthreads();
  float* acc_s = reinterpret_cast<float*>(&k_s[0][0][0]);  // [kWarps][G][HD] fp32 (fits: 4*G*HD*4 <= K tiles)
#pragma unroll
  for (int g = 0; g < G; ++g)
#pragma unroll
    for (int j = 0; j < DL; ++j) acc_s[((size_t)warp * G + g) * HD + lane * DL + j] = acc[g][j];
  __syncthreads();
  for (int i = tid; i < G * HD; i += kThreads) {
    const int g = i / HD, d = i % HD;
    float M = -INFINITY;
    for (int w = 0; w < kWarps; ++w) M = fmaxf(M, m_s[w][g]);
    float L = 0.f, A = 0.f;
    if (M != -INFINITY) {
      for (int w = 0; w < kWarps; ++w) {
        const float f = exp2f(m_s[w][g] - M);
        L += f * l_s[w][g];
        A += f * acc_s[((size_t)w * G + g) * HD + d];
      }
    }
    const int h = kvh * G + g;
    if (p.splits == 1) {
      store_out(p, b, h, HD, d, L > 0.f ? A / L : 0.f);
    } else {
      float* part = p.part + (((int64_t)b * p.Hq + h) * p.splits + split) * (HD + 2);
      part[d] = A;
      if (d == 0) {
        part[HD] = M;
        part[HD + 1] = L;
      }
    }
  }
}

// Merge of the splits of one (request, head): out = sum_s 2^(m_s - M) acc_s / sum_s 2^(m_s - M) l_s.
template <int HD>
__global__ void __launch_bounds__(HD) gqa_combine_kernel(AttnParams p) {
  zb::pdl_enter();
  const int h = blockIdx.x, b = blockIdx.y, d = threadIdx.x;
  const float* part = p.part + ((int64_t)b * p.Hq + h) * p.splits * (HD + 2);
  float M = -INFINITY;
  for (int s = 0; s < p.splits; ++s) M = fmaxf(M, part[s * (HD + 2) + HD]);
  float L = 0.f, A = 0.f;
  if (M != -INFINITY) {
    for (int s = 0; s < p.splits; ++s) {
      const float f = exp2f(part[s * (HD + 2) + HD] - M);
      L += f * part[s * (HD + 2) + HD + 1];
      A += f * part[s * (HD + 2) + d];
    }
  }
  store_out(p, b, h, HD, d, L > 0.f ? A / L : 0.f);
}

template <int HD, int G>
int launch_attn(const AttnParams& p, cudaStream_t stream) {
  constexpr size_t smem = AttnSmem<HD, G>::total;
  auto kernel = gqa_decode_kernel<HD, G>;
  static bool configured[64] = {false};  // the shared-memory attribute, set once per device
  int dev = 0;
  ZB_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64 || !configured[dev]) {
    ZB_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    if (dev >= 0 && dev < 64) configured[dev] = true;
  }
  ZB_CUDA(zb::launch(kernel, dim3((unsigned)p.splits, (unsigned)p.Hkv, (unsigned)p.B), dim3(kThreads), smem, stream,
                     1, p));
  if (int rc = zb::check_launch("gqa_decode")) return rc;
  if (p.splits > 1) {
    ZB_CUDA(zb::launch(gqa_combine_kernel<HD>, dim3((unsigned)p.Hq, (unsigned)p.B), dim3(HD), 0, stream, 1, p));
    return zb::check_launch("gqa_decode(combine)");
  }
  return zb::kOk;
}

template <int HD>
int dispatch_group(const AttnParams& p, int G, cudaStream_t stream) {
  switch (G) {
    case 1: return launch_attn<HD, 1>(p, stream);
    case 2: return launch_attn<HD, 2>(p, stream);
    case 4: return launch_attn<HD, 4>(p, stream);
    case 8: return launch_attn<HD, 8>(p, stream);
    default: return zb::fail(zb::kUnsupported, "gqa_decode: %d query heads per KV head (1, 2, 4 or 8)", G);
  }
}

// ---------------------------------------------------------------------------------------------------------------
// Head dim 128: the tensor cores do both products. Warp-specialised, persistent CTAs (one per SM) walk their
// (request, KV head, split) units back to back:
//  - four loader warps read the page table one tile ahead and copy each 128-position tile's K and V rows
//    (thread r: row r's slot; a warp moves two 256-byte rows per instruction in 16-byte pieces) into a 3-stage
//    ring, 128B-swizzled; every loader thread's copies complete on the stage's mbarrier
//    (cp.async.mbarrier.arrive.noinc), so no thread waits for its own copies; they also stage each unit's
//    queries. (TMA tile::gather4 of the 128-byte rows measured 2.6x slower: request-bound.)
//  - four consumer warps (thread t = position t of the tile, = dimension t of the output): S^T = K Q^T
//    (M = 128 positions, N = 16: the group's heads zero-padded) lands in tensor memory; each thread reads its
//    position's scores, the tile max per head goes through shared memory, p = 2^(s log2e scale - m) is rounded to
//    bf16 (as FlashAttention-3 rounds P) into a K-major P^T operand, and O^T += V^T P^T (M = 128 dimensions,
//    N = 16; V read MN-major) accumulates in tensor memory. The running max is raised only when a tile's max
//    exceeds it by more than 2^8 (the stale max keeps every p <= 256 and cancels in the final division), so the
//    accumulator is rescaled (tensor-memory load, scale, store) only on such tiles.
// Consumer thread 0 issues the MMAs: O^T(t) then a commit to the stage's "empty" barrier (the loader refills it),
// then S^T(t + 1) once its stage is full, then a commit to the scores barrier.
namespace tcattn {

constexpr int kHD = 128;
constexpr int kTilePos = 128;  // key positions of a tile (tensor-memory lanes of S^T)
constexpr int kStages = 3;
constexpr int kN = 16;                         // MMA N: the group's query heads, zero-padded
constexpr int kConsumers = 4;                  // consumer warps (0-3: one per tensor-memory lane quarter)
constexpr int kLoaders = 4;                    // loader warps (4-7)
constexpr int kThreadsTma = 32 * (kConsumers + kLoaders);
constexpr uint32_t kBlkBytes = kTilePos * 128;  // one 64-dim block of a tile: 128 rows x 128 B
constexpr uint32_t kKBytes = 2 * kBlkBytes;     // K tile (K-major for S^T)
constexpr uint32_t kVBytes = 2 * kBlkBytes;     // V tile, same layout (MN-major for O^T)
constexpr uint32_t kStageBytes = kKBytes + kVBytes;
constexpr uint32_t kPBytes = kN * kTilePos * 2;  // P^T: 16 head rows x 128 positions, 2 K-major blocks
constexpr uint32_t kQBytes = kN * kHD * 2;       // Q: 16 head rows x 128 dims, 2 K-major blocks
constexpr uint32_t kBlk16 = kN * 128;            // one 64-wide K block of a 16-row operand
constexpr int kQBufs = kStages;                  // a unit's queries stay until its last S^T completed
constexpr uint32_t kOffP = kStages * kStageBytes;
constexpr uint32_t kOffQ = kOffP + 2 * kPBytes;
constexpr uint32_t kOffTail = kOffQ + kQBufs * kQBytes;
constexpr uint32_t kColS = 0, kColO = 16, kTmemCols = 32;
constexpr int kMaxUnits = 64;  // units one CTA walks at most (the grid grows past one CTA per SM beyond that)

struct Tail {
  int ulen[kMaxUnits];               // key count of each of this CTA's units (clamped to max_seq_len)
  unsigned mask[kStages][kLoaders];  // per stage: bit b of word w = position 32 w + b holds a key
  float red[2][kConsumers][kN];      // per-warp tile max of each head (double-buffered across tiles)
  float lsum[kConsumers][kN];        // per-warp denominators
  uint64_t full[kStages];            // every loader thread's copies of the stage landed (+ the mask's arrival)
  uint64_t empty[kStages];           // the stage's O^T update completed
  uint64_t sbar;                     // S^T completed
  uint32_t tmem;
  int abort;
};
constexpr size_t kSmem = kOffTail + sizeof(Tail) + 1024;  // + slack to 1024-align the base

// 16 bytes global -> shared; valid == false writes zeros and reads nothing.
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid = true) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(valid ? 16 : 0) : "memory");
}
// Arrives on `bar` once every cp.async this thread issued before has completed (counts as one expected arrival).
__device__ __forceinline__ void cp_async_arrive(uint32_t bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void consumer_sync() { asm volatile("bar.sync 1, %0;" ::"n"(kConsumers * 32) : "memory"); }

// Bounded wait that gives up at once after any earlier expiry in the CTA (flag in shared memory).
__device__ __forceinline__ bool wait(uint32_t bar, uint32_t parity, int* abort, unsigned* status) {
  if (*reinterpret_cast<volatile int*>(abort) != 0) return false;
  if (zb::mbar_wait_bounded(bar, parity, status, zb::kStatusAttnDecodeTimeout)) return true;
  *reinterpret_cast<volatile int*>(abort) = 1;
  return false;
}

}  // namespace tcattn

// Work unit = (request, KV head, split); unit u -> b = u / (Hkv * splits), kvh = u / splits % Hkv,
// split = u % splits. CTA c takes units c, c + gridDim.x, ... in order; a cursor walks their tiles.
struct Cursor {
  int u, j;  // unit (>= units: past the end) and tile within it
  int b, kvh, split, begin, end, ntiles;
};

// ulen: the key counts of this CTA's units, staged in shared memory.
__device__ __forceinline__ void unit_info(const AttnParams& p, const int* ulen, Cursor& c) {
  c.split = c.u % p.splits;
  c.kvh = c.u / p.splits % p.Hkv;
  c.b = c.u / (p.splits * p.Hkv);
  const int len = ulen[(c.u - (int)blockIdx.x) / (int)gridDim.x];
  c.begin = c.split * p.split_len;
  c.end = min(len, c.begin + p.split_len);
  c.ntiles = c.end > c.begin ? (c.end - c.begin + tcattn::kTilePos - 1) / tcattn::kTilePos : 0;
}
// From unit c.u on, the first unit with a tile (c.u >= units when none is left).
__device__ __forceinline__ void seek(const AttnParams& p, const int* ulen, Cursor& c, int units) {
  for (; c.u < units; c.u += gridDim.x) {
    unit_info(p, ulen, c);
    if (c.ntiles > 0) return;
  }
}
__device__ __forceinline__ void advance(const AttnParams& p, const int* ulen, Cursor& c, int units) {
  if (++c.j == c.ntiles) {
    c.j = 0;
    c.u += gridDim.x;
    seek(p, ulen, c, units);
  }
}

template <int G>
__global__ void __launch_bounds__(tcattn::kThreadsTma, 1)
    gqa_decode_tc_kernel(AttnParams p) {
  using namespace tcattn;
  namespace tc = zb::tc;
  zb::pdl_enter();
  extern __shared__ __align__(16) unsigned char smem_raw[];  // re-aligned to 1024 bytes below
  const uint32_t raw = zb::smem_addr(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  unsigned char* gbase = smem_raw + (base - raw);
  Tail& tl = *reinterpret_cast<Tail*>(gbase + kOffTail);
  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  const int units = p.B * p.Hkv * p.splits;
  auto full = [&](int s) { return zb::smem_addr(&tl.full[s]); };
  auto empty = [&](int s) { return zb::smem_addr(&tl.empty[s]); };
  const uint32_t sbar = zb::smem_addr(&tl.sbar);

  // This CTA's key counts in one parallel read; units without keys get their zero output (or empty partial) now.
  for (int i = tid; i < kMaxUnits; i += kThreadsTma) {
    const int u = (int)blockIdx.x + i * (int)gridDim.x;
    tl.ulen[i] = u < units ? min(max(p.seq_lens[u / (p.splits * p.Hkv)], 0), p.max_seq_len) : 0;
  }
  // P^T and Q buffers zeroed once (rows >= G stay zero)
  for (int i = tid; i < (int)((2 * kPBytes + kQBufs * kQBytes) / 16); i += kThreadsTma) {
    reinterpret_cast<uint4*>(gbase + kOffP)[i] = make_uint4(0, 0, 0, 0);
  }
  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) {
      zb::mbar_init(full(s), kLoaders * 32 + kLoaders);
      zb::mbar_init(empty(s), 1);
    }
    zb::mbar_init(sbar, 1);
    zb::fence_mbar_init();
    tl.abort = 0;
  }
  if (warp == 0) tc::alloc(zb::smem_addr(&tl.tmem), kTmemCols);
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  const int* ulen = tl.ulen;
  int total = 0;
  if (warp < kConsumers) {
    for (Cursor c{(int)blockIdx.x, 0}; c.u < units; c.u += gridDim.x) {
      unit_info(p, ulen, c);
      total += c.ntiles;
      if (c.ntiles > 0) continue;
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const int h = c.kvh * G + g;
        if (p.splits == 1) {
          store_out(p, c.b, h, kHD, tid, 0.f);
        } else {
          float* part = p.part + (((int64_t)c.b * p.Hq + h) * p.splits + c.split) * (kHD + 2);
          part[tid] = 0.f;
          if (tid == 0) {
            part[kHD] = -INFINITY;
            part[kHD + 1] = 0.f;
          }
        }
      }
    }
  }

  if (warp >= kConsumers) {
    // ------------------------------------------------------------------ loader warps
    const int r = tid - kConsumers * 32, lw = r / 32;  // this thread's tile row; loader warp index
    Cursor lc{(int)blockIdx.x, 0};
    seek(p, ulen, lc, units);
    auto read_slot = [&](const Cursor& c) {
      const int pos = c.begin + c.j * kTilePos + r;
      return c.u < units && pos < c.end ? p.page_table[(int64_t)c.b * p.table_stride + pos] : -1;
    };
    int ahead = read_slot(lc);
    int unit_no = 0;
    for (int j = 0; lc.u < units; ++j) {
      const int stage = j % kStages;
      if (j >= kStages) wait(empty(stage), (uint32_t)((j / kStages - 1) & 1), &tl.abort, p.status);
      const bool valid = ahead >= 0 && ahead < p.num_slots;
      const unsigned bits = __ballot_sync(0xffffffffu, valid);
      const int mine = valid ? ahead : -1;
      const uint32_t kb = base + (uint32_t)stage * kStageBytes, vb = kb + kKBytes;
      const int64_t head = (int64_t)lc.kvh * kHD;
#pragma unroll 4
      for (int it = 0; it < 16; ++it) {  // two rows per pass: 16 lanes x 16 bytes of each 256-byte row
        const int rl = 2 * it + lane / 16, c = lane % 16;
        const int rs = __shfl_sync(0xffffffffu, mine, rl);
        const bool ok = rs >= 0;  // a masked row is zero-filled: its p is 0, and 0 x V must stay 0
        const int64_t off = (int64_t)(ok ? rs : 0) * p.slot_stride + head + c * 8;
        const uint32_t o = (uint32_t)(c / 8) * kBlkBytes + tc::sw128(32 * lw + rl, c % 8);
        cp_async16(kb + o, p.k_cache + off, ok);
        cp_async16(vb + o, p.v_cache + off, ok);
      }
      if (lc.j == 0) {  // the unit's queries (rows < G) into its Q buffer
        if (r < G * 16) {
          const int qr = r / 16, c = r % 16;
          cp_async16(base + kOffQ + (uint32_t)(unit_no % kQBufs) * kQBytes + (uint32_t)(c / 8) * kBlk16 +
                         tc::sw128(qr, c % 8),
                     p.q + (int64_t)lc.b * p.q_stride + (int64_t)(lc.kvh * G + qr) * kHD + c * 8);
        }
        ++unit_no;
      }
      cp_async_arrive(full(stage));
      if (lane == 0) {  // the mask word, published by a plain (release) arrival of each loader warp
        tl.mask[stage][lw] = bits;
        zb::mbar_arrive(full(stage));
      }
      advance(p, ulen, lc, units);
      ahead = read_slot(lc);
    }
  } else {
    // ------------------------------------------------------------------ consumer warps
    const uint32_t tmem = tl.tmem;
    const uint32_t tlane = tmem + ((uint32_t)(32 * warp) << 16);
    constexpr uint32_t kIdS = tc::idesc_bf16(128, kN);
    constexpr uint32_t kIdO = tc::idesc_bf16(128, kN, /*a_mn=*/true);
    auto issue_s = [&](int t, int qbuf) {  // S^T(t) = K(t) Q^T
      const uint32_t kb = base + (uint32_t)(t % kStages) * kStageBytes;
      const uint32_t qb = base + kOffQ + (uint32_t)qbuf * kQBytes;
#pragma unroll
      for (int ks = 0; ks < kHD / 16; ++ks) {
        tc::mma(tmem + kColS, tc::desc_kmajor(kb + (ks / 4) * kBlkBytes + (ks % 4) * 32),
                tc::desc_kmajor(qb + (ks / 4) * kBlk16 + (ks % 4) * 32), kIdS, ks > 0);
      }
    };
    auto issue_o = [&](int t, bool accumulate) {  // O^T (+)= V(t)^T P(t)^T; V atoms: 16 KB apart along dims
      const uint32_t vb = base + (uint32_t)(t % kStages) * kStageBytes + kKBytes;
      const uint32_t pb = base + kOffP + (uint32_t)(t & 1) * kPBytes;
#pragma unroll
      for (int ks = 0; ks < kTilePos / 16; ++ks) {
        tc::mma(tmem + kColO, tc::desc_mnmajor(vb + ks * 2048, kBlkBytes, 1024),
                tc::desc_kmajor(pb + (ks / 4) * kBlk16 + (ks % 4) * 32), kIdO, accumulate || ks > 0);
      }
    };
    if (tid == 0 && total > 0) {
      wait(full(0), 0, &tl.abort, p.status);
      tc::fence_proxy_async();  // the loaders' copies (generic proxy) -> the tensor core's reads
      tc::fence_after();
      issue_s(0, 0);
      tc::commit(sbar);
    }

    Cursor cc{(int)blockIdx.x, 0};
    seek(p, ulen, cc, units);
    Cursor done = cc;  // the unit whose accumulator is read next
    int cunits = 0;
    float m_run[G], l_part[G];
#pragma unroll
    for (int g = 0; g < G; ++g) {
      m_run[g] = -INFINITY;
      l_part[g] = 0.f;
    }
    auto finish = [&](const Cursor& u, const float (&o)[G], const float (&m)[G]) {
      if (*reinterpret_cast<volatile int*>(&tl.abort) != 0) return;
#pragma unroll
      for (int g = 0; g < G; ++g) {
        float L = 0.f;
#pragma unroll
        for (int w = 0; w < kConsumers; ++w) L += tl.lsum[w][g];
        const int h = u.kvh * G + g;
        if (p.splits == 1) {
          store_out(p, u.b, h, kHD, tid, L > 0.f ? o[g] / L : 0.f);
        } else {
          float* part = p.part + (((int64_t)u.b * p.Hq + h) * p.splits + u.split) * (kHD + 2);
          part[tid] = L > 0.f ? o[g] : 0.f;
          if (tid == 0) {
            part[kHD] = m[g];
            part[kHD + 1] = L;
          }
        }
      }
    };
    auto close_unit = [&](float (&o)[G], float (&m)[G]) {
      uint32_t r[16];
      tc::ld16(tlane + kColO, r);
      tc::ld_wait();
#pragma unroll
      for (int g = 0; g < G; ++g) {
        o[g] = __uint_as_float(r[g]);
        m[g] = m_run[g];
        const float s = zb::warp_sum(l_part[g]);
        if (lane == 0) tl.lsum[warp][g] = s;
        m_run[g] = -INFINITY;
        l_part[g] = 0.f;
      }
    };

    for (int t = 0; t < total; ++t) {
      const int stage = t % kStages;
      // S^T(t) complete (and O^T(t - 1) before it); the stage's barrier also publishes its key mask
      wait(sbar, (uint32_t)(t & 1), &tl.abort, p.status);
      wait(full(stage), (uint32_t)((t / kStages) & 1), &tl.abort, p.status);
      tc::fence_after();
      const bool first = cc.j == 0;
      float o_prev[G], m_prev[G];
      if (first && t > 0) close_unit(o_prev, m_prev);
      uint32_t sr[16];
      tc::ld16(tlane + kColS, sr);
      tc::ld_wait();
      const bool valid = (tl.mask[stage][tid / 32] >> (tid % 32)) & 1u;
      float x[G];
#pragma unroll
      for (int g = 0; g < G; ++g) {
        x[g] = valid ? __uint_as_float(sr[g]) * p.scale_log2 : -INFINITY;
        const float wm = zb::warp_max(x[g]);
        if (lane == 0) tl.red[t & 1][warp][g] = wm;
      }
      consumer_sync();
      if (first && t > 0) {
        finish(done, o_prev, m_prev);
        done = cc;
      }
      bool rescale = false;
      float corr[G];
#pragma unroll
      for (int g = 0; g < G; ++g) {
        float mt = tl.red[t & 1][0][g];
#pragma unroll
        for (int w = 1; w < kConsumers; ++w) mt = fmaxf(mt, tl.red[t & 1][w][g]);
        corr[g] = 1.f;
        if (mt > m_run[g] + 8.f) {  // never true while both are -inf
          corr[g] = exp2f(m_run[g] - mt);  // 0 for the unit's first tile with a key
          m_run[g] = mt;
          rescale = true;
        }
      }
      if (rescale) {  // the same decision on every thread (same maxima, same history)
#pragma unroll
        for (int g = 0; g < G; ++g) l_part[g] *= corr[g];
        if (!first) {  // a unit's first O^T update overwrites the accumulator
          uint32_t o[16];
          tc::ld16(tlane + kColO, o);
          tc::ld_wait();
#pragma unroll
          for (int g = 0; g < G; ++g) o[g] = __float_as_uint(__uint_as_float(o[g]) * corr[g]);
          tc::st16(tlane + kColO, o);
          tc::st_wait();
        }
      }
      unsigned char* pbuf = gbase + kOffP + (t & 1) * kPBytes + (tid / 64) * kBlk16 + (tid % 8) * 2;
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float pv = x[g] == -INFINITY ? 0.f : exp2f(x[g] - m_run[g]);
        l_part[g] += pv;
        *reinterpret_cast<__nv_bfloat16*>(pbuf + tc::sw128(g, (tid % 64) / 8)) = __float2bfloat16_rn(pv);
      }
      advance(p, ulen, cc, units);
      const int next_q = cunits + (cc.j == 0 ? 1 : 0);  // Q buffer of tile t + 1's unit
      tc::fence_proxy_async();
      tc::fence_before();
      consumer_sync();
      tc::fence_after();
      if (tid == 0) {
        issue_o(t, !first);
        tc::commit(empty(stage));
        if (t + 1 < total) {
          wait(full((t + 1) % kStages), (uint32_t)(((t + 1) / kStages) & 1), &tl.abort, p.status);
          tc::fence_proxy_async();
          tc::fence_after();
          issue_s(t + 1, next_q % kQBufs);
          tc::commit(sbar);
        }
      }
      cunits = next_q;
    }

    if (total > 0) {
      wait(empty((total - 1) % kStages), (uint32_t)(((total - 1) / kStages) & 1), &tl.abort, p.status);
      tc::fence_after();
      float o_last[G], m_last[G];
      close_unit(o_last, m_last);
      consumer_sync();
      finish(done, o_last, m_last);
    }
    tc::fence_before();
    consumer_sync();
    if (warp == 0) {
      tc::fence_after();
      tc::dealloc(tmem, kTmemCols);
    }
  }
}

template <int G>
int launch_attn_tc(const AttnParams& p, cudaStream_t stream) {
  auto kernel = gqa_decode_tc_kernel<G>;
  static bool configured[64] = {false};  // the shared-memory attribute, set once per device
  int dev = 0;
  ZB_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64 || !configured[dev]) {
    ZB_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)tcattn::kSmem));
    if (dev >= 0 && dev < 64) configured[dev] = true;
  }
  // persistent: one CTA per SM (the ring takes most of its shared memory), each walking its units in turn
  const int64_t units = (int64_t)p.B * p.Hkv * p.splits;
  const int64_t per_cta_limit = (units + tcattn::kMaxUnits - 1) / tcattn::kMaxUnits;
  const unsigned grid = (unsigned)std::max<int64_t>(std::min<int64_t>(units, zb::sm_count()), per_cta_limit);
  ZB_CUDA(zb::launch(kernel, dim3(grid), dim3(tcattn::kThreadsTma), tcattn::kSmem, stream, 1, p));
  if (int rc = zb::check_launch("gqa_decode")) return rc;
  if (p.splits > 1) {
    ZB_CUDA(zb::launch(gqa_combine_kernel<128>, dim3((unsigned)p.Hq, (unsigned)p.B), dim3(128), 0, stream, 1, p));
    return zb::check_launch("gqa_decode(combine)");
  }
  return zb::kOk;
}

struct StoreParams {
  __nv_bfloat16* k_cache;
  __nv_bfloat16* v_cache;
  int64_t slot_stride;
  int64_t num_slots;
  const int32_t* slots;  // [N] destination slot of each row (outside [0, num_slots): not stored)
  const __nv_bfloat16* k;  // [N, row] with row stride k_stride
  const __nv_bfloat16* v;
  int64_t k_stride, v_stride;
  int N, row;  // row = Hkv * hd elements (a multiple of 8)
};

// A warp per (row, k or v): 16-byte pieces.
__global__ void __launch_bounds__(256) kv_store_kernel(StoreParams p) {
  zb::pdl_enter();
  const int64_t unit = (int64_t)blockIdx.x * 8 + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (unit >= 2 * (int64_t)p.N) return;
  const int64_t i = unit / 2;
  const bool is_v = unit % 2;
  const int slot = p.slots[i];
  if (slot < 0 || slot >= p.num_slots) return;
  const uint4* src = reinterpret_cast<const uint4*>((is_v ? p.v + i * p.v_stride : p.k + i * p.k_stride));
  uint4* dst = reinterpret_cast<uint4*>((is_v ? p.v_cache : p.k_cache) + (int64_t)slot * p.slot_stride);
  for (int c = lane; c < p.row / 8; c += 32) dst[c] = src[c];
}

}  // namespace

ZB_API int zb_gqa_decode(const uint16_t* q, int64_t q_stride, const uint16_t* k_cache, const uint16_t* v_cache,
                         int64_t slot_stride, int64_t num_slots, const int32_t* page_table, int64_t table_stride,
                         const int32_t* seq_lens, int max_seq_len, int B, int Hq, int Hkv, int hd,
                         float softmax_scale, int splits, int split_len, float* workspace, int64_t workspace_bytes,
                         uint16_t* out, int64_t out_stride, const uint16_t* gate, int64_t gate_stride,
                         cudaStream_t stream) {
  ZB_REQUIRE(B >= 0 && Hq > 0 && Hkv > 0 && Hq % Hkv == 0, "gqa_decode: bad heads Hq=%d Hkv=%d", Hq, Hkv);
  if (hd != 32 && hd != 64 && hd != 128) {
    return zb::fail(zb::kUnsupported, "gqa_decode: head dim %d (32, 64 or 128)", hd);
  }
  if (B == 0) return zb::kOk;
  ZB_REQUIRE(q && k_cache && v_cache && page_table && seq_lens && out, "gqa_decode: null pointer");
  const int tile = hd == 128 ? tcattn::kTilePos : kTile;
  ZB_REQUIRE(splits >= 1 && split_len > 0 && split_len % tile == 0,
             "gqa_decode: splits %d >= 1 and split_len %d a positive multiple of %d", splits, split_len, tile);
  ZB_REQUIRE(max_seq_len >= 0 && max_seq_len <= table_stride && (int64_t)splits * split_len >= max_seq_len &&
                 num_slots >= 0,
             "gqa_decode: max_seq_len %d must fit the table row (%lld) and the splits (%d x %d)", max_seq_len,
             (long long)table_stride, splits, split_len);
  const int64_t need = splits > 1 ? (int64_t)B * Hq * splits * (hd + 2) * 4 : 0;
  ZB_REQUIRE(splits == 1 || (workspace && workspace_bytes >= need),
             "gqa_decode: %d splits need a workspace of %lld bytes", splits, (long long)need);
  ZB_REQUIRE(q_stride >= (int64_t)Hq * hd && out_stride >= (int64_t)Hq * hd && slot_stride >= (int64_t)Hkv * hd &&
                 slot_stride % 8 == 0,
             "gqa_decode: strides (q %lld, out %lld, slot %lld)", (long long)q_stride, (long long)out_stride,
             (long long)slot_stride);
  ZB_REQUIRE_ALIGNED(k_cache, 16, "gqa_decode k_cache");
  ZB_REQUIRE_ALIGNED(v_cache, 16, "gqa_decode v_cache");
  AttnParams p{reinterpret_cast<const __nv_bfloat16*>(q), q_stride, reinterpret_cast<const __nv_bfloat16*>(k_cache),
               reinterpret_cast<const __nv_bfloat16*>(v_cache), slot_stride, num_slots, page_table, table_stride,
               seq_lens, max_seq_len, B, Hq, Hkv, softmax_scale * 1.4426950408889634f, splits, split_len, workspace,
               reinterpret_cast<__nv_bfloat16*>(out), out_stride, zb::device_status_ptr(),
               reinterpret_cast<const __nv_bfloat16*>(gate), gate_stride};
  ZB_REQUIRE(!gate || gate_stride >= Hq, "gqa_decode: gate_stride %lld < %d heads", (long long)gate_stride, Hq);
  const int G = Hq / Hkv;
  if (hd == 128) {
    ZB_REQUIRE(q_stride % 8 == 0, "gqa_decode: q_stride %lld must be a multiple of 8", (long long)q_stride);
    ZB_REQUIRE(num_slots >= 1, "gqa_decode: an empty cache (num_slots %lld)", (long long)num_slots);
    ZB_REQUIRE_ALIGNED(q, 16, "gqa_decode q");
    switch (G) {
      case 1: return launch_attn_tc<1>(p, stream);
      case 2: return launch_attn_tc<2>(p, stream);
      case 4: return launch_attn_tc<4>(p, stream);
      case 8: return launch_attn_tc<8>(p, stream);
      default: return zb::fail(zb::kUnsupported, "gqa_decode: %d query heads per KV head (1, 2, 4 or 8)", G);
    }
  }
  return hd == 64 ? dispatch_group<64>(p, G, stream) : dispatch_group<32>(p, G, stream);
}

ZB_API int zb_kv_store(uint16_t* k_cache, uint16_t* v_cache, int64_t slot_stride, int64_t num_slots,
                       const int32_t* slots, const uint16_t* k, int64_t k_stride, const uint16_t* v, int64_t v_stride,
                       int N, int Hkv, int hd, cudaStream_t stream) {
  ZB_REQUIRE(N >= 0 && Hkv > 0 && hd > 0 && (Hkv * hd) % 8 == 0, "kv_store: bad sizes N=%d Hkv=%d hd=%d", N, Hkv, hd);
  if (N == 0) return zb::kOk;
  ZB_REQUIRE(k_cache && v_cache && slots && k && v, "kv_store: null pointer");
  ZB_REQUIRE(slot_stride >= (int64_t)Hkv * hd && slot_stride % 8 == 0 && k_stride % 8 == 0 && v_stride % 8 == 0 &&
                 k_stride >= (int64_t)Hkv * hd && v_stride >= (int64_t)Hkv * hd,
             "kv_store: strides must cover a row and be multiples of 8 elements");
  for (const void* ptr : {(const void*)k_cache, (const void*)v_cache, (const void*)k, (const void*)v}) {
    ZB_REQUIRE_ALIGNED(ptr, 16, "kv_store tensors");
  }
  StoreParams p{reinterpret_cast<__nv_bfloat16*>(k_cache), reinterpret_cast<__nv_bfloat16*>(v_cache), slot_stride,
                num_slots, slots, reinterpret_cast<const __nv_bfloat16*>(k), reinterpret_cast<const __nv_bfloat16*>(v), k_stride,
                v_stride, N, Hkv * hd};
  ZB_CUDA(zb::launch(kv_store_kernel, dim3((unsigned)((2 * (int64_t)N + 7) / 8)), dim3(256), 0, stream, 1, p));
  return zb::check_launch("kv_store");
}

// ---------------------------------------------------------------------------------------------------------------
// The attention layer's decode prologue in one kernel: from the fused projection rows [N, Hq*hd | Hkv*hd | Hkv*hd]
// (q | k | v, then anything after, row stride proj_stride), per token t and head: q = bf16(RMSNorm(q_h, eps)),
// q = bf16(q * bf16(|temp_h|)), k = bf16(RMSNorm(k_g, eps)), both rotated by interleaved RoPE at positions[t]
// (pairs (2i, 2i+1), inverse frequency 1 / theta^(2i / hd)), q written to q_out [N, Hq, hd], k and v written to
// slot out_loc[t] of the caches (a slot outside [0, num_slots) stores nothing). Follows Attention.forward
// (servers/sgl/src/zonos3_sgl/models/zonos3.py:340-375: rms_norm, |temp|, rotary with is_neox=False, store_kv).
// A warp per (token, head), lane l owning dims 4l .. 4l+3 (two rotation pairs).
namespace {

struct PrologueParams {
  const __nv_bfloat16* proj;
  int64_t proj_stride;
  const __nv_bfloat16* temp;  // [Hq]
  const int32_t* positions;   // [N]
  float theta, eps;
  __nv_bfloat16* q_out;  // [N, Hq, 128]
  __nv_bfloat16* k_cache;
  __nv_bfloat16* v_cache;
  int64_t slot_stride, num_slots;
  const int32_t* out_loc;  // [N]
  int N, Hq, Hkv;
};

__global__ void __launch_bounds__(256) gqa_prologue_kernel(PrologueParams p) {
  zb::pdl_enter();
  constexpr int HD = 128;
  const int heads = p.Hq + 2 * p.Hkv;
  const int64_t unit = (int64_t)blockIdx.x * 8 + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (unit >= (int64_t)p.N * heads) return;
  const int t = (int)(unit / heads), h = (int)(unit % heads);
  const int64_t slot = p.out_loc[t];
  const bool store = slot >= 0 && slot < p.num_slots;
  const __nv_bfloat16* src = p.proj + (int64_t)t * p.proj_stride + (int64_t)h * HD + 4 * lane;
  float x[4];
  zb::ld_bf16x4(src, x);
  if (h >= p.Hq + p.Hkv) {  // v: copied into the cache
    if (store) {
      *reinterpret_cast<uint2*>(p.v_cache + slot * p.slot_stride + (int64_t)(h - p.Hq - p.Hkv) * HD + 4 * lane) =
          *reinterpret_cast<const uint2*>(src);
    }
    return;
  }
  const float ss = zb::warp_sum(x[0] * x[0] + x[1] * x[1] + x[2] * x[2] + x[3] * x[3]);
  const float r = rsqrtf(ss / HD + p.eps);
  const bool is_q = h < p.Hq;
  const float tq = is_q ? zb::bf16_round(fabsf(__bfloat162float(p.temp[h]))) : 1.f;
  float y[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    y[k] = zb::bf16_round(x[k] * r);
    if (is_q) y[k] = zb::bf16_round(y[k] * tq);
  }
  const float pos = (float)p.positions[t];
  uint32_t word[2];
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    const int i = 2 * lane + k;  // rotation pair (dims 2i, 2i+1)
    const float inv_freq = 1.0f / powf(p.theta, (float)(2 * i) / HD);
    float sn, cs;
    sincosf(pos * inv_freq, &sn, &cs);
    const float a = y[2 * k], b = y[2 * k + 1];
    const __nv_bfloat162 rot = __floats2bfloat162_rn(a * cs - b * sn, a * sn + b * cs);
    word[k] = *reinterpret_cast<const uint32_t*>(&rot);
  }
  const uint2 packed = make_uint2(word[0], word[1]);
  if (is_q) {
    *reinterpret_cast<uint2*>(p.q_out + ((int64_t)t * p.Hq + h) * HD + 4 * lane) = packed;
  } else if (store) {
    *reinterpret_cast<uint2*>(p.k_cache + slot * p.slot_stride + (int64_t)(h - p.Hq) * HD + 4 * lane) = packed;
  }
}

}  // namespace

ZB_API int zb_gqa_prologue_decode(const uint16_t* proj, int64_t proj_stride, const uint16_t* temp,
                                  const int32_t* positions, float rope_theta, float eps, uint16_t* q_out,
                                  uint16_t* k_cache, uint16_t* v_cache, int64_t slot_stride, int64_t num_slots,
                                  const int32_t* out_loc, int N, int Hq, int Hkv, int hd, cudaStream_t stream) {
  ZB_REQUIRE(N >= 0 && Hq > 0 && Hkv > 0, "gqa_prologue_decode: sizes N=%d Hq=%d Hkv=%d", N, Hq, Hkv);
  if (hd != 128) return zb::fail(zb::kUnsupported, "gqa_prologue_decode: head dim %d (128)", hd);
  if (N == 0) return zb::kOk;
  ZB_REQUIRE(proj && temp && positions && q_out && k_cache && v_cache && out_loc, "gqa_prologue_decode: null pointer");
  ZB_REQUIRE(proj_stride >= (int64_t)(Hq + 2 * Hkv) * hd && proj_stride % 4 == 0 && slot_stride >= (int64_t)Hkv * hd &&
                 slot_stride % 4 == 0,
             "gqa_prologue_decode: strides (proj %lld, slot %lld)", (long long)proj_stride, (long long)slot_stride);
  for (const void* ptr : {(const void*)proj, (const void*)q_out, (const void*)k_cache, (const void*)v_cache}) {
    ZB_REQUIRE_ALIGNED(ptr, 8, "gqa_prologue_decode tensors");
  }
  PrologueParams p{reinterpret_cast<const __nv_bfloat16*>(proj), proj_stride,
                   reinterpret_cast<const __nv_bfloat16*>(temp), positions, rope_theta, eps,
                   reinterpret_cast<__nv_bfloat16*>(q_out), reinterpret_cast<__nv_bfloat16*>(k_cache),
                   reinterpret_cast<__nv_bfloat16*>(v_cache), slot_stride, num_slots, out_loc, N, Hq, Hkv};
  const int64_t units = (int64_t)N * (Hq + 2 * Hkv);
  ZB_CUDA(zb::launch(gqa_prologue_kernel, dim3((unsigned)((units + 7) / 8)), dim3(256), 0, stream, 1, p));
  return zb::check_launch("gqa_prologue_decode");
}

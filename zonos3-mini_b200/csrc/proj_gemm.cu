// Dense projections of the decode step on 5th-generation tensor cores (tcgen05 + TMEM + TMA), sm_100a:
//
//   Y[t, n] = X[t, :] . W[n, :]        X [T, K] bf16 (tokens), W [N, K] bf16 (a Linear weight), fp32 accumulation
//
// with two epilogues:
//   plain        Y rounded once to bf16 (the layer's F.linear: DeltaNet and attention wo, the attention projection,
//                the codebook head; servers/sgl/src/zonos3_sgl/models/gdn.py:447, zonos3.py:326-390, :1341-1360);
//   DeltaNet     the in_proj GEMM (gdn.py:399) fused with the decode prologue that OriginalGDN runs on its output
//   decode       (gdn.py:403-434: FLA causal_conv1d_update + l2norm + the gate and beta; lm.py:561-573): per token,
//                the qkv channels go through the width-4 causal conv continuing the token's conv history (which it
//                shifts in place), SiLU, and the per-head L2 norm of q and k; z is stored for the gated norm; the a /
//                b columns become g = -exp(A_log) * softplus(a + dt_bias) and beta = sigmoid(b). The in_proj output
//                never reaches global memory. Rounding points follow the unfused path: in_proj output bf16, conv
//                output bf16, normalised q / k bf16.
//
// Kernel: persistent CTA pairs (clusters of 2, one CTA per SM) on 256-token x BN-column tiles with the pair-wide
// tcgen05.mma.cta_group::2 (M = 256: each CTA holds 128 tokens of X and BN/2 rows of W, and the fp32 accumulator of
// its 128 tokens x BN columns in its own TMEM):
//   warp 0      TMA producer of its CTA: per stage of two k-blocks, one 3-D tensor copy of X [2 x 128 x 64] and one
//               of W [2 x BN/2 x 64], 128B-swizzled, plain loads without multicast (a copy spanning two k-blocks
//               of the same rows streams at about twice the rate of two [rows x 64] copies); both CTAs' bytes
//               complete on the leader's full barrier;
//   warp 1      TMEM (two BN-column accumulators); on the leader one lane issues the M=256 MMAs and commits;
//   warps 2-9   epilogue: lane quarter (warp % 4) of the CTA's 128 tokens, column half (warp - 2) / 4.
// Work items are (token tile, column tile, K slice). With S > 1 slices (split-K, for the narrow projections whose
// column tiles alone would leave most SMs idle) every CTA writes its fp32 partial tile to the workspace and takes a
// ticket (an acq_rel atomic on the tile's counter); the CTA that draws the last ticket sums the S partials in slice
// order (so the result does not depend on which CTA came last), runs the epilogue, resets the counter and drops the
// partials' L2 lines (discard.global.L2, no write-back). Nothing waits on another CTA outside its own pair. Every
// mbarrier wait is bounded (~1 s): on expiry the kernel sets a status bit, stops issuing, drains, frees TMEM and
// returns (a tile's counter may then stay non-zero: the caller re-zeroes the workspace after such a status).
#include <algorithm>

#include "tc_pair.cuh"

namespace {

constexpr int BK = 64;    // K elements of one swizzled 128-byte row
constexpr int KD = 2;     // k-blocks per stage, moved by one 3-D tensor copy per operand
constexpr int SBK = BK * KD;
constexpr int kEpiWarps = 8;
constexpr int kThreads = (2 + kEpiWarps) * 32;
constexpr uint32_t X_BLOCK = 128 * BK * 2;  // 16 KB: this CTA's 128 tokens of one k-block
constexpr uint32_t X_BYTES = KD * X_BLOCK;
constexpr int kMaxStages = 8;
constexpr int kW = 4;  // conv width of the release DeltaNet

template <int BN>
struct Cfg {
  static_assert(BN == 64 || BN == 128 || BN == 256, "column tile");
  static constexpr uint32_t W_BLOCK = (BN / 2) * BK * 2;  // this CTA's half of the tile's weight rows, one k-block
  static constexpr uint32_t W_BYTES = KD * W_BLOCK;
  static constexpr uint32_t STAGE_BYTES = X_BYTES + W_BYTES;
  static constexpr int STAGES = (200 * 1024) / STAGE_BYTES;  // 3 (BN 256), 4 (128), 5 (64)
  static constexpr uint32_t TMEM_COLS = 2 * BN;  // double-buffered accumulator (a power of two >= 128)
  static constexpr int CHUNKS = BN / 64;         // 32-column chunks of an epilogue warp's column half
};

enum Epi : int { kPlain = 0, kGdnDecode = 1 };
// Column tile of the fused DeltaNet in_proj: 64 columns per epilogue warp, so a 128-channel head spans the two
// column halves (they swap their sums of squares) and the 8224-column in_proj makes 65 tiles, 130 CTAs.
constexpr int kGdnBlockN = 128;

struct ProjParams {
  int T, N, K;
  int m_tiles, n_tiles, splits;
  int total_items;
  unsigned* tickets;  // [m_tiles * n_tiles * 2] (splits > 1)
  float* partial;     // [m_tiles * n_tiles * 2][splits][128][BN] fp32 (splits > 1)
  // plain
  __nv_bfloat16* out;
  int64_t out_stride;
  // DeltaNet decode prologue
  const __nv_bfloat16* conv_w;  // [3 * inner, W]
  const float* A_log;           // [H]
  const float* dt_bias;         // [H]
  const int64_t* slots;         // [T] conv-state row of each token (outside [0, conv_rows): padding)
  __nv_bfloat16* conv_state;    // [conv_rows, 3 * inner, W - 1]
  int64_t conv_rows;
  __nv_bfloat16* q;  // [T, inner] each
  __nv_bfloat16* k;
  __nv_bfloat16* v;
  __nv_bfloat16* z;
  float* g;  // [T, H]
  float* beta;
  int H, D;
  unsigned* status;
};

struct Shared {
  uint64_t full[kMaxStages];
  uint64_t empty[kMaxStages];
  uint64_t tmem_full[2];
  uint64_t tmem_empty[2];
  uint64_t drain;
  uint64_t xbar[2];       // DeltaNet prologue: the epilogue warps' sum-of-squares exchange, by item parity
  uint32_t tmem_base;
  int abort;
  int last;
  float ss_x[2][2][128];  // [item parity][column half][token]
};
constexpr uint32_t kSharedBytes = (sizeof(Shared) + 127) / 128 * 128;

__device__ __forceinline__ float silu(float x) { return x / (1.0f + expf(-x)); }
__device__ __forceinline__ float softplus(float x) { return x > 20.f ? x : log1pf(expf(x)); }

__device__ __forceinline__ unsigned atomic_add_acq_rel(unsigned* p, unsigned v) {
  unsigned old;
  asm volatile("atom.add.acq_rel.gpu.global.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}
__device__ __forceinline__ void discard_l2(const void* p) {
  asm volatile("discard.global.L2 [%0], 128;" ::"l"(p) : "memory");
}
__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}
__device__ __forceinline__ void epilogue_bar() { asm volatile("bar.sync 1, %0;" ::"n"(kEpiWarps * 32) : "memory"); }

// Element i of bf16 values packed two per 32-bit word (low half first): as a float, or its 16 raw bits.
__device__ __forceinline__ float bf16_at(const uint32_t* r, int i) {
  return __uint_as_float((i & 1) ? (r[i >> 1] & 0xffff0000u) : (r[i >> 1] << 16));
}
__device__ __forceinline__ uint32_t raw16_at(const uint32_t* r, int i) {
  return (i & 1) ? (r[i >> 1] >> 16) : (r[i >> 1] & 0xffffu);
}
__device__ __forceinline__ uint32_t pack2(float a, float b) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}

template <int BN, int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    proj_gemm_kernel(const __grid_constant__ CUtensorMap tmap_x, const __grid_constant__ CUtensorMap tmap_w,
                     ProjParams p) {
  zb::pdl_enter();
  using C = Cfg<BN>;
  constexpr int STAGES = C::STAGES;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  // stage buffers 1024-byte aligned (the swizzle atom); the dynamic shared-memory base is the same in both CTAs of
  // the pair, so every buffer sits at the same offset in both
  const uint32_t raw_addr = zb::smem_addr(smem_raw);
  unsigned char* stages = smem_raw + ((1024 - (raw_addr & 1023)) & 1023);
  Shared* sh = reinterpret_cast<Shared*>(stages + STAGES * C::STAGE_BYTES);
  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  const uint32_t rank = blockIdx.x & 1;
  const bool leader = rank == 0;
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  volatile int* abort_flag = &sh->abort;
  const int k_blocks = p.K / SBK;  // stages of KD k-blocks

  if (tid == 0) {
    for (int s = 0; s < STAGES; ++s) {
      zb::mbar_init(zb::smem_addr(&sh->full[s]), 1);
      zb::mbar_init(zb::smem_addr(&sh->empty[s]), 1);
    }
    for (int a = 0; a < 2; ++a) {
      zb::mbar_init(zb::smem_addr(&sh->tmem_full[a]), 1);
      zb::mbar_init(zb::smem_addr(&sh->tmem_empty[a]), 2 * kEpiWarps);  // the epilogue warps of both CTAs
    }
    zb::mbar_init(zb::smem_addr(&sh->drain), 1);
    for (int a = 0; a < 2; ++a) zb::mbar_init(zb::smem_addr(&sh->xbar[a]), kEpiWarps);
    sh->abort = 0;
    zb::fence_mbar_init();
  }
  if (warp == 1) zb::tcp::tmem_alloc<true>(zb::smem_addr(&sh->tmem_base), C::TMEM_COLS);
  zb::tcp::fence_before();
  __syncthreads();
  zb::cluster_arrive_relaxed();  // both CTAs' barriers are initialised before either signals the other's
  zb::cluster_wait();
  zb::tcp::fence_after();
  const uint32_t tmem_base = sh->tmem_base;

  // item -> (token tile m, column tile n, K slice s), token tile fastest
  auto decode = [&](int item, int& m, int& n, int& s) {
    m = item % p.m_tiles;
    const int r = item / p.m_tiles;
    s = r % p.splits;
    n = r / p.splits;
  };
  auto k_range = [&](int s, int& kb0, int& kb1) {
    kb0 = (int)((int64_t)s * k_blocks / p.splits);
    kb1 = (int)((int64_t)(s + 1) * k_blocks / p.splits);
  };

  if (warp == 0) {
    if (lane == 0) {  // producer of this CTA's halves; bytes complete on the leader's full barrier
      uint32_t q = 0;
      for (int item = pair; item < p.total_items && !*abort_flag; item += npairs) {
        int m, n, s, kb0, kb1;
        decode(item, m, n, s);
        k_range(s, kb0, kb1);
        const int x_row = m * 256 + (int)rank * 128;
        const int w_row = n * BN + (int)rank * (BN / 2);
        for (int kb = kb0; kb < kb1; ++kb, ++q) {
          const int st = q % STAGES;
          if (!zb::mbar_wait_bounded(zb::smem_addr(&sh->empty[st]), ((q / STAGES) & 1) ^ 1, p.status,
                                     zb::kStatusGemmTimeout)) {
            *abort_flag = 1;
            break;
          }
          const uint32_t full_local = zb::smem_addr(&sh->full[st]);
          if (leader) zb::mbar_arrive_expect_tx(full_local, 2 * C::STAGE_BYTES);
          const uint32_t full_leader = zb::mapa_shared(full_local, 0);
          const uint32_t dst = zb::smem_addr(stages + st * C::STAGE_BYTES);
          zb::tcp::tma_load_kblocks<true>(dst, &tmap_x, x_row, kb * KD, full_leader);
          zb::tcp::tma_load_kblocks<true>(dst + X_BYTES, &tmap_w, w_row, kb * KD, full_leader);
        }
      }
      if (leader) {  // drain: wait (bounded) for the copies still in flight before the CTA may exit
        for (uint32_t d = 0; d < (uint32_t)STAGES && d < q; ++d) {
          const uint32_t qq = q - 1 - d;
          zb::mbar_wait_bounded(zb::smem_addr(&sh->full[qq % STAGES]), (qq / STAGES) & 1, nullptr, 0, 200000000ull);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {  // the pair's MMA issuer
      uint32_t q = 0;
      int it = 0;
      for (int item = pair; item < p.total_items && !*abort_flag; item += npairs, ++it) {
        const int acc = it & 1;
        const uint32_t use = it >> 1;
        if (!zb::mbar_wait_bounded(zb::smem_addr(&sh->tmem_empty[acc]), (use & 1) ^ 1, p.status,
                                   zb::kStatusGemmTimeout)) {
          *abort_flag = 1;
          break;
        }
        zb::tcp::fence_after();
        int m, n, s, kb0, kb1;
        decode(item, m, n, s);
        k_range(s, kb0, kb1);
        const uint32_t d_tmem = tmem_base + acc * BN;
        bool ok = true;
        for (int kb = kb0; kb < kb1; ++kb, ++q) {
          const int st = q % STAGES;
          if (!zb::mbar_wait_bounded(zb::smem_addr(&sh->full[st]), (q / STAGES) & 1, p.status,
                                     zb::kStatusGemmTimeout)) {
            *abort_flag = 1;
            ok = false;
            break;
          }
          zb::tcp::fence_after();
          const uint32_t x_addr = zb::smem_addr(stages + st * C::STAGE_BYTES);
          const uint32_t w_addr = x_addr + X_BYTES;
#pragma unroll
          for (int j = 0; j < KD; ++j) {
#pragma unroll
            for (int kk = 0; kk < BK / 16; ++kk) {
              zb::tcp::mma<true>(d_tmem, zb::tcp::desc_sw128(x_addr + j * X_BLOCK + kk * 32),
                                 zb::tcp::desc_sw128(w_addr + j * C::W_BLOCK + kk * 32), zb::tcp::idesc(256, BN),
                                 (kb > kb0 || j > 0 || kk > 0) ? 1u : 0u);
            }
          }
          zb::tcp::commit<true>(zb::smem_addr(&sh->empty[st]), 0x3);  // stage st of both CTAs is free
        }
        if (!ok) break;
        zb::tcp::commit<true>(zb::smem_addr(&sh->tmem_full[acc]), 0x3);
      }
      // every MMA issued by this thread has completed before TMEM is released
      zb::tcp::commit<true>(zb::smem_addr(&sh->drain), 0x1);
      zb::mbar_wait_bounded(zb::smem_addr(&sh->drain), 0, nullptr, 0, 200000000ull);
    }
  } else {
    const int quarter = warp % 4, chalf = (warp - 2) / 4;
    const int row_local = quarter * 32 + lane;  // this thread's token inside the CTA's 128
    int it = 0;
    for (int item = pair; item < p.total_items; item += npairs, ++it) {
      const int acc = it & 1;
      const uint32_t use = it >> 1;
      int m, n, s;
      decode(item, m, n, s);
      const int64_t t = (int64_t)m * 256 + rank * 128 + row_local;
      const bool valid = t < p.T;
      const int col0 = n * BN + chalf * (BN / 2);  // first output column of this warp's half
      const bool split = p.splits > 1;
      // DeltaNet prologue: the token's conv-history row of this half's channels, fetched into L2 while the MMAs run
      // (a slot outside [0, conv_rows) is a padding token: zero history, never written)
      bool has_hist = false;
      __nv_bfloat16* hist = nullptr;
      if constexpr (EPI == kGdnDecode) {
        const int inner = p.H * p.D;
        if (valid && col0 < 3 * inner) {
          const int64_t slot = p.slots[t];
          has_hist = slot >= 0 && slot < p.conv_rows;
          if (has_hist) {
            hist = p.conv_state + (slot * 3 * inner + col0) * (kW - 1);
            prefetch_l2(hist, (BN / 2) * (kW - 1) * 2);
          }
        }
      }
      const bool ok = __all_sync(0xffffffffu, !*abort_flag && zb::mbar_wait_bounded(zb::smem_addr(&sh->tmem_full[acc]),
                                                                                    use & 1, p.status,
                                                                                    zb::kStatusGemmTimeout));
      if (!ok && !split) {  // the tcgen05.ld below are warp-collective: the whole warp leaves
        *abort_flag = 1;
        break;
      }
      zb::tcp::fence_after();
      const uint32_t t_row = tmem_base + ((uint32_t)(quarter * 32) << 16) + acc * BN + chalf * (BN / 2);
      const int tile = m * p.n_tiles + n;
      float* part_row = p.partial + ((int64_t)(tile * 2 + (int)rank) * p.splits * 128 + row_local) * BN +
                        chalf * (BN / 2);  // slice sl at + sl * 128 * BN
      if (split) {
        // this slice's partial tile -> workspace, then the ticket. The epilogue warps meet at named barriers here,
        // so they leave on an expired wait together: the decision is taken once, by one thread, between barriers.
        if (ok) {
#pragma unroll 1
          for (int c = 0; c < C::CHUNKS; ++c) {
            float y[32];
            zb::tcp::tmem_ld32(t_row + c * 32, y);
            if (valid) {
              float4* dst = reinterpret_cast<float4*>(part_row + (int64_t)s * 128 * BN + c * 32);
#pragma unroll
              for (int j = 0; j < 8; ++j)
                __stcg(dst + j, make_float4(y[4 * j], y[4 * j + 1], y[4 * j + 2], y[4 * j + 3]));
            }
          }
        } else {
          *abort_flag = 1;
        }
        zb::tcp::fence_before();
        __syncwarp();
        if (lane == 0) zb::tcp::mbar_arrive_cluster(zb::mapa_shared(zb::smem_addr(&sh->tmem_empty[acc]), 0));
        __threadfence();
        epilogue_bar();
        if (warp == 2 && lane == 0) {
          int decision = -1;  // -1: leave (a wait expired), 0: another slice completes the tile, 1: this CTA does
          if (!*abort_flag) {
            unsigned* ticket = p.tickets + tile * 2 + rank;
            const unsigned prior = atomic_add_acq_rel(ticket, 1u);
            decision = prior == (unsigned)(p.splits - 1);
            if (decision) *reinterpret_cast<volatile unsigned*>(ticket) = 0u;  // every slice has arrived: reset
          }
          sh->last = decision;
        }
        epilogue_bar();
        const int decision = sh->last;
        epilogue_bar();  // every epilogue thread has read sh->last before the next item may rewrite it
        if (decision < 0) break;
        if (decision == 0) continue;
        __threadfence();
      }
      // the tile's values, 32 columns at a time: from TMEM, or the slices' partial sums in slice order
      auto load = [&](int c, float (&y)[32]) {
        if (!split) {
          zb::tcp::tmem_ld32(t_row + c * 32, y);
          return;
        }
#pragma unroll
        for (int j = 0; j < 32; ++j) y[j] = 0.f;
        if (!valid) return;
        for (int sl = 0; sl < p.splits; ++sl) {
          const float* src = part_row + (int64_t)sl * 128 * BN + c * 32;
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const float4 u = __ldcg(reinterpret_cast<const float4*>(src) + j);
            y[4 * j] += u.x;
            y[4 * j + 1] += u.y;
            y[4 * j + 2] += u.z;
            y[4 * j + 3] += u.w;
          }
          discard_l2(src);
        }
      };

      if constexpr (EPI == kPlain) {
#pragma unroll 1
        for (int c = 0; c < C::CHUNKS; ++c) {
          float y[32];
          load(c, y);
          const int c0 = col0 + c * 32;
          if (valid) {
            __nv_bfloat16* dst = p.out + t * p.out_stride + c0;
#pragma unroll
            for (int j = 0; j < 4; ++j)
              if (c0 + 8 * j < p.N) *reinterpret_cast<uint4*>(dst + 8 * j) = zb::pack_bf16x8(y + 8 * j);
          }
        }
      } else {
        // DeltaNet decode prologue. Regions of the in_proj columns: [0, 3 inner) q | k | v, [3 inner, 4 inner) z,
        // then a | b (one column per head each). A warp's column half never straddles two regions.
        const int inner = p.H * p.D;
        const bool exch = p.D > BN / 2;  // a head spans both column halves: the halves swap sums of squares
        float total = 0.f;               // this half's sum of squares (q / k: one head when !exch)
        uint32_t packed[C::CHUNKS * 16];  // conv outputs (bf16 pairs) of the warp's columns
        float ss[C::CHUNKS];
        const bool conv = col0 < 3 * inner;
        const int part = col0 / inner;
        if (conv) {
          // q / k / v channels: causal conv over (history, this token), SiLU; history shifted in place
#pragma unroll
          for (int c = 0; c < C::CHUNKS; ++c) {
            float y[32];
            load(c, y);
            float css = 0.f;
#pragma unroll
            for (int g16 = 0; g16 < 2; ++g16) {
              const int chl = c * 32 + g16 * 16;  // first of 16 channels (96 contiguous history bytes)
              uint32_t hr[24];                    // history [ch][W-1] as bf16 pairs
              if (has_hist) {
                const uint4* hp = reinterpret_cast<const uint4*>(hist + chl * (kW - 1));
#pragma unroll
                for (int u = 0; u < 6; ++u) {
                  const uint4 t4 = hp[u];
                  hr[4 * u] = t4.x, hr[4 * u + 1] = t4.y, hr[4 * u + 2] = t4.z, hr[4 * u + 3] = t4.w;
                }
              } else {
#pragma unroll
                for (int u = 0; u < 24; ++u) hr[u] = 0u;
              }
              uint32_t xb[16];  // this token's inputs (bf16 bits)
              float out[16];
#pragma unroll
              for (int g8 = 0; g8 < 2; ++g8) {
                uint32_t wr[16];  // taps [ch][W] of 8 channels
                const uint4* wp = reinterpret_cast<const uint4*>(p.conv_w + (int64_t)(col0 + chl + g8 * 8) * kW);
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                  const uint4 t4 = __ldg(wp + u);
                  wr[4 * u] = t4.x, wr[4 * u + 1] = t4.y, wr[4 * u + 2] = t4.z, wr[4 * u + 3] = t4.w;
                }
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                  const int ch = g8 * 8 + j;
                  const float xin = zb::bf16_round(y[g16 * 16 + ch]);  // the in_proj output is bf16
                  float a = 0.f;
#pragma unroll
                  for (int e = 0; e < kW - 1; ++e) a = fmaf(bf16_at(wr, j * kW + e), bf16_at(hr, ch * 3 + e), a);
                  a = fmaf(bf16_at(wr, j * kW + kW - 1), xin, a);
                  out[ch] = zb::bf16_round(silu(a));  // the conv output is an activation of the model dtype
                  css = fmaf(out[ch], out[ch], css);
                  xb[ch] = __float_as_uint(xin) >> 16;
                }
              }
              if (has_hist) {  // new history per channel: old entries 1 .. W-2, then this token's input
                uint32_t nr[24];
#pragma unroll
                for (int w = 0; w < 24; ++w) {
                  uint32_t half[2];
#pragma unroll
                  for (int hh = 0; hh < 2; ++hh) {
                    const int i = 2 * w + hh;  // element (channel i / 3, entry i % 3)
                    half[hh] = (i % 3 == 2) ? xb[i / 3] : raw16_at(hr, i + 1);
                  }
                  nr[w] = half[0] | (half[1] << 16);
                }
                uint4* hp = reinterpret_cast<uint4*>(hist + chl * (kW - 1));
#pragma unroll
                for (int u = 0; u < 6; ++u) hp[u] = make_uint4(nr[4 * u], nr[4 * u + 1], nr[4 * u + 2], nr[4 * u + 3]);
              }
#pragma unroll
              for (int j = 0; j < 8; ++j) packed[c * 16 + g16 * 8 + j] = pack2(out[2 * j], out[2 * j + 1]);
            }
            ss[c] = css;
            total += css;
          }
        } else if (col0 < 4 * inner) {
          // z: stored for the gated norm
#pragma unroll 1
          for (int c = 0; c < C::CHUNKS; ++c) {
            float y[32];
            load(c, y);
            if (valid) {
              __nv_bfloat16* dst = p.z + t * inner + (col0 - 3 * inner) + c * 32;
#pragma unroll
              for (int j = 0; j < 4; ++j) *reinterpret_cast<uint4*>(dst + 8 * j) = zb::pack_bf16x8(y + 8 * j);
            }
          }
        } else {
          // a | b: the log decay g and the write strength beta of each head
#pragma unroll 1
          for (int c = 0; c < C::CHUNKS; ++c) {
            float y[32];
            load(c, y);
            if (!valid) continue;
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const int col = col0 - 4 * inner + c * 32 + j;
              const float x = zb::bf16_round(y[j]);
              if (col < p.H) {
                p.g[t * p.H + col] = -expf(p.A_log[col]) * softplus(x + p.dt_bias[col]);
              } else if (col < 2 * p.H) {
                p.beta[t * p.H + col - p.H] = 1.f / (1.f + expf(-x));
              }
            }
          }
        }
        float partner = 0.f;
        if (exch) {  // every epilogue warp of the CTA takes part, whatever its region
          const int buf = it & 1;
          sh->ss_x[buf][chalf][row_local] = total;
          __syncwarp();
          if (lane == 0) zb::mbar_arrive(zb::smem_addr(&sh->xbar[buf]));
          const bool seen = __all_sync(0xffffffffu, zb::mbar_wait_bounded(zb::smem_addr(&sh->xbar[buf]),
                                                                          (it >> 1) & 1, p.status,
                                                                          zb::kStatusGemmTimeout));
          if (!seen) {
            *abort_flag = 1;
            break;
          }
          partner = sh->ss_x[buf][chalf ^ 1][row_local];
        }
        if (conv && valid) {
          __nv_bfloat16* dst = (part == 0 ? p.q : part == 1 ? p.k : p.v) + t * inner + (col0 - part * inner);
          const int per_head = p.D / 32;  // chunks of one head when it lies inside the half
#pragma unroll
          for (int c = 0; c < C::CHUNKS; ++c) {
            float scale = 1.f;
            if (part < 2) {
              float tot = total + partner;
              if (!exch) {
                const int h0 = c / per_head * per_head;
                tot = 0.f;
#pragma unroll
                for (int cc = 0; cc < C::CHUNKS; ++cc)
                  if (cc >= h0 && cc < h0 + per_head) tot += ss[cc];
              }
              scale = rsqrtf(tot + 1e-6f);
            }
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              uint32_t o[4];
#pragma unroll
              for (int u = 0; u < 4; ++u) {
                const uint32_t pk = packed[c * 16 + j * 4 + u];
                o[u] = pack2(__uint_as_float(pk << 16) * scale, __uint_as_float(pk & 0xffff0000u) * scale);
              }
              *reinterpret_cast<uint4*>(dst + c * 32 + j * 8) = make_uint4(o[0], o[1], o[2], o[3]);
            }
          }
        }
      }
      if (!split) {
        zb::tcp::fence_before();
        __syncwarp();
        if (lane == 0) zb::tcp::mbar_arrive_cluster(zb::mapa_shared(zb::smem_addr(&sh->tmem_empty[acc]), 0));
      }
    }
  }
  zb::tcp::fence_before();
  __syncthreads();
  zb::cluster_arrive_relaxed();  // neither CTA frees TMEM or exits while the pair may still use it
  zb::cluster_wait();
  if (warp == 1) {
    zb::tcp::fence_after();
    zb::tcp::tmem_dealloc<true>(tmem_base, C::TMEM_COLS);
  }
}

// ------------------------------------------------------------------------------------------ host side

template <int BN>
constexpr size_t smem_bytes() {
  return 1024 + Cfg<BN>::STAGES * Cfg<BN>::STAGE_BYTES + kSharedBytes;
}

struct Plan {
  int block_n, splits, m_tiles, n_tiles;
  int64_t ticket_bytes, partial_bytes;
};

int k_blocks_of(int K) { return K / SBK; }

// Column tile and K slices: the explicit choice when given (block_n 64 / 128 / 256, splits >= 1), else the widest
// tile that still gives every pair of SMs a tile, and one K slice (split-K measured slower at the decode shapes: the
// partial tiles' round trip through L2 costs more than the idle SMs it recovers).
Plan plan_for(int T, int N, int K, int block_n, int splits, int pairs) {
  Plan pl{};
  pl.m_tiles = (T + 255) / 256;
  if (block_n == 0) {
    block_n = 256;
    while (block_n > 64 && (int64_t)pl.m_tiles * ((N + block_n - 1) / block_n) * 2 <= pairs) block_n /= 2;
  }
  pl.block_n = block_n;
  pl.n_tiles = (N + block_n - 1) / block_n;
  const int64_t tiles = (int64_t)pl.m_tiles * pl.n_tiles;
  if (splits == 0) splits = 1;
  pl.splits = splits;
  pl.ticket_bytes = splits > 1 ? (tiles * 2 * 4 + 255) / 256 * 256 : 0;
  pl.partial_bytes = splits > 1 ? tiles * 2 * splits * 128 * block_n * 4 : 0;
  return pl;
}

template <int BN>
int pairs_for();

template <int BN, int EPI>
int launch(const CUtensorMap& mx, const CUtensorMap& mw, ProjParams p, cudaStream_t stream, const char* what) {
  auto kernel = proj_gemm_kernel<BN, EPI>;
  constexpr size_t kSmem = smem_bytes<BN>();
  static_assert(kSmem <= 227 * 1024, "shared memory of one CTA");
  static int configured[64] = {0};
  int dev = 0;
  ZB_CUDA(cudaGetDevice(&dev));
  const bool cacheable = dev >= 0 && dev < 64;
  if (!cacheable || !configured[dev]) {
    ZB_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmem));
    if (cacheable) configured[dev] = 1;
  }
  const int pairs = pairs_for<BN>();  // the persistent loop assumes every pair is resident at once
  if (pairs < 1) return zb::fail(zb::kUnsupported, "%s: no CTA pair fits on this GPU", what);
  const int units = std::min(p.total_items, pairs);
  if (units <= 0) return zb::kOk;
  ZB_CUDA(zb::launch(kernel, dim3((unsigned)(2 * units)), dim3(kThreads), kSmem, stream, 2u, mx, mw, p));
  return zb::check_launch(what);
}

// Pairs resident at once for the column tile (cached per device; the same for both epilogues: one CTA per SM).
template <int BN>
int pairs_for() {
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  if (dev >= 0 && dev < 64 && cached[dev]) return cached[dev];
  auto kernel = proj_gemm_kernel<BN, kPlain>;
  constexpr size_t kSmem = smem_bytes<BN>();
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmem) != cudaSuccess) return 0;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kSmem;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int pairs = 0;
  if (cudaOccupancyMaxActiveClusters(&pairs, kernel, &cfg) != cudaSuccess) return 0;
  if (dev >= 0 && dev < 64) cached[dev] = pairs;
  return pairs;
}

// Host-side plan without a device (workspace sizing): 74 pairs, the B200's 148 SMs.
constexpr int kDefaultPairs = 74;

int check_plan(const Plan& pl, int K, void* workspace, int64_t workspace_bytes, const char* what) {
  if (pl.block_n != 64 && pl.block_n != 128 && pl.block_n != 256)
    return zb::fail(zb::kUnsupported, "%s: column tile %d (64, 128 or 256)", what, pl.block_n);
  ZB_REQUIRE(pl.splits >= 1 && pl.splits <= k_blocks_of(K), "%s: %d K slices for %d k-blocks", what, pl.splits,
             k_blocks_of(K));
  if (pl.splits > 1) {
    ZB_REQUIRE(workspace != nullptr, "%s: split-K needs a workspace", what);
    ZB_REQUIRE(workspace_bytes >= pl.ticket_bytes + pl.partial_bytes, "%s: workspace %lld bytes < %lld", what,
               (long long)workspace_bytes, (long long)(pl.ticket_bytes + pl.partial_bytes));
    ZB_REQUIRE_ALIGNED(workspace, 256, "workspace");
  }
  return zb::kOk;
}

template <int EPI>
int dispatch(const Plan& pl, const CUtensorMap& mx, const CUtensorMap& mw, ProjParams& p, cudaStream_t stream,
             const char* what) {
  switch (pl.block_n) {
    case 64: return launch<64, EPI>(mx, mw, p, stream, what);
    case 128: return launch<128, EPI>(mx, mw, p, stream, what);
    default: return launch<256, EPI>(mx, mw, p, stream, what);
  }
}

// Plans against the pairs resident at once (every tile keeps one CTA per SM, so the widest tile's count serves all).
Plan resolve_plan(int T, int N, int K, int block_n, int splits) {
  int pairs = pairs_for<256>();
  if (pairs <= 0) pairs = kDefaultPairs;
  return plan_for(T, N, K, block_n, splits, pairs);
}

int common_checks(const void* x, int64_t x_stride, int T, int K, const void* w, int N, const char* what) {
  ZB_REQUIRE(x && w, "%s: null pointer", what);
  ZB_REQUIRE(T >= 0 && N > 0 && K > 0, "%s: bad sizes T=%d N=%d K=%d", what, T, N, K);
  if (K % SBK != 0) return zb::fail(zb::kUnsupported, "%s: K=%d must be a multiple of %d", what, K, SBK);
  ZB_REQUIRE(x_stride >= K && x_stride % 8 == 0, "%s: x row stride %lld (>= K, a multiple of 8)", what,
             (long long)x_stride);
  ZB_REQUIRE_ALIGNED(x, 16, "x");
  ZB_REQUIRE_ALIGNED(w, 16, "weight");
  return zb::kOk;
}

}  // namespace

ZB_API int64_t zb_proj_gemm_workspace_bytes(int T, int N, int K, int block_n, int splits) {
  if (T <= 0 || N <= 0 || K < SBK) return 0;
  const Plan pl = resolve_plan(T, N, K, block_n, splits);
  return pl.ticket_bytes + pl.partial_bytes;
}

ZB_API int zb_proj_gemm(const uint16_t* x, int64_t x_stride, int T, int K, const uint16_t* weight, int N,
                        uint16_t* out, int64_t out_stride, int block_n, int splits, void* workspace,
                        int64_t workspace_bytes, cudaStream_t stream) {
  if (int rc = common_checks(x, x_stride, T, K, weight, N, "proj_gemm")) return rc;
  ZB_REQUIRE(out != nullptr, "proj_gemm: null output");
  ZB_REQUIRE(N % 8 == 0 && out_stride >= N && out_stride % 8 == 0,
             "proj_gemm: N=%d (a multiple of 8) and out row stride %lld (>= N, a multiple of 8)", N,
             (long long)out_stride);
  ZB_REQUIRE_ALIGNED(out, 16, "out");
  if (T == 0) return zb::kOk;
  const Plan pl = resolve_plan(T, N, K, block_n, splits);
  if (int rc = check_plan(pl, K, workspace, workspace_bytes, "proj_gemm")) return rc;
  CUtensorMap mx, mw;
  if (int rc = zb::tcp::make_map_kblocks(&mx, x, T, K, x_stride, 128, KD, "proj_gemm")) return rc;
  if (int rc = zb::tcp::make_map_kblocks(&mw, weight, N, K, K, (uint32_t)(pl.block_n / 2), KD, "proj_gemm")) return rc;
  ProjParams p{};
  p.T = T;
  p.N = N;
  p.K = K;
  p.m_tiles = pl.m_tiles;
  p.n_tiles = pl.n_tiles;
  p.splits = pl.splits;
  p.total_items = pl.m_tiles * pl.n_tiles * pl.splits;
  p.tickets = reinterpret_cast<unsigned*>(workspace);
  p.partial = reinterpret_cast<float*>(static_cast<char*>(workspace) + pl.ticket_bytes);
  p.out = reinterpret_cast<__nv_bfloat16*>(out);
  p.out_stride = out_stride;
  p.status = zb::device_status_ptr();
  return dispatch<kPlain>(pl, mx, mw, p, stream, "proj_gemm");
}

ZB_API int zb_gdn_in_proj_decode(const uint16_t* x, int64_t x_stride, int T, int K, const uint16_t* in_proj,
                                 const uint16_t* conv_weight, const float* A_log, const float* dt_bias,
                                 const int64_t* slots, uint16_t* conv_state, int64_t conv_rows, int H, int D,
                                 uint16_t* q, uint16_t* k, uint16_t* v, uint16_t* z, float* g, float* beta,
                                 int splits, void* workspace, int64_t workspace_bytes, cudaStream_t stream) {
  const char* what = "gdn_in_proj_decode";
  ZB_REQUIRE(H > 0 && H <= 64, "%s: H=%d (1..64)", what, H);
  if (D != 64 && D != 128) return zb::fail(zb::kUnsupported, "%s: head dim %d (64 or 128)", what, D);
  const int inner = H * D;
  if (inner % 128 != 0) return zb::fail(zb::kUnsupported, "%s: H*D=%d must be a multiple of 128", what, inner);
  const int N = 4 * inner + 2 * H;
  if (int rc = common_checks(x, x_stride, T, K, in_proj, N, what)) return rc;
  ZB_REQUIRE(conv_weight && A_log && dt_bias && slots && conv_state && q && k && v && z && g && beta,
             "%s: null pointer", what);
  for (const void* ptr : {(const void*)conv_weight, (const void*)conv_state, (const void*)q, (const void*)k,
                          (const void*)v, (const void*)z}) {
    ZB_REQUIRE_ALIGNED(ptr, 16, "gdn_in_proj_decode tensors");
  }
  if (T == 0) return zb::kOk;
  const Plan pl = resolve_plan(T, N, K, kGdnBlockN, splits);
  if (int rc = check_plan(pl, K, workspace, workspace_bytes, what)) return rc;
  CUtensorMap mx, mw;
  if (int rc = zb::tcp::make_map_kblocks(&mx, x, T, K, x_stride, 128, KD, what)) return rc;
  if (int rc = zb::tcp::make_map_kblocks(&mw, in_proj, N, K, K, kGdnBlockN / 2, KD, what)) return rc;
  ProjParams p{};
  p.T = T;
  p.N = N;
  p.K = K;
  p.m_tiles = pl.m_tiles;
  p.n_tiles = pl.n_tiles;
  p.splits = pl.splits;
  p.total_items = pl.m_tiles * pl.n_tiles * pl.splits;
  p.tickets = reinterpret_cast<unsigned*>(workspace);
  p.partial = reinterpret_cast<float*>(static_cast<char*>(workspace) + pl.ticket_bytes);
  p.conv_w = reinterpret_cast<const __nv_bfloat16*>(conv_weight);
  p.A_log = A_log;
  p.dt_bias = dt_bias;
  p.slots = slots;
  p.conv_state = reinterpret_cast<__nv_bfloat16*>(conv_state);
  p.conv_rows = conv_rows;
  p.q = reinterpret_cast<__nv_bfloat16*>(q);
  p.k = reinterpret_cast<__nv_bfloat16*>(k);
  p.v = reinterpret_cast<__nv_bfloat16*>(v);
  p.z = reinterpret_cast<__nv_bfloat16*>(z);
  p.g = g;
  p.beta = beta;
  p.H = H;
  p.D = D;
  p.status = zb::device_status_ptr();
  return launch<kGdnBlockN, kGdnDecode>(mx, mw, p, stream, what);
}

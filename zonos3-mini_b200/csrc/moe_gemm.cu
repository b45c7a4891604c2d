// Grouped expert GEMMs of the MoE layer on 5th-generation tensor cores (tcgen05 + TMEM + TMA), sm_100a.
//
//   GEMM1 (gate/up + SwiGLU): H[r, n] = bf16( silu(bf16(A[r].Wg[e,n])) * bf16(A[r].Wu[e,n]) )
//   GEMM2 (down + routing weight): Y[pair(r), n] = bf16( (H[r].W2[e,n]) * weight[pair(r)] )
// A rows are the permuted (token, slot) pairs, grouped by expert and padded to 128-row tiles (zb_moe_permute);
// expert e owns rows [offsets[e], offsets[e+1]). The k slots of a token are summed afterwards (zb_moe_combine).
// Reference: fused_experts_impl (servers/sgl/src/zonos3_sgl/layers/moe/fused_moe/fused_moe_impl.py:127-289)
// with fused_moe_kernel (servers/sgl/src/zonos3_sgl/kernel/triton/fused_moe.py:54-192) and silu_and_mul; weight
// layouts gate_up_proj [E, 2I, D] (gate rows first) and down_proj [E, D, I] (zonos3.py:450-637); the math of
// lm.py:618-639. Rounding points follow the server: GEMM1 output bf16, SwiGLU bf16, GEMM2 * weight bf16.
//
// Kernel structure: persistent CTA pairs (clusters of 2, one CTA per SM, 6 warps each) computing 256 x 256 output
// tiles with the pair-wide tcgen05.mma.cta_group::2 (M = 256: each CTA holds 128 rows of A and 128 of the 256 B
// rows, and its 128 accumulator rows in its own TMEM), so every SM stages half of the B tile it used to:
//   warp 0      TMA producer of its CTA: per k-block, its A tile [128 x 64] and its B half [128 x 64], both
//               128B-swizzled, into a 6-stage ring (32 KB per stage); both CTAs' copies complete bytes on the
//               leader CTA's full barrier (plain tensor loads, no multicast);
//   warp 1      TMEM (512 columns = two 128x256 fp32 accumulators, allocated pair-wide); on the leader CTA one
//               lane issues the M=256 MMAs (K=16 each) and commits to both CTAs' barriers;
//   warps 2-9   epilogue of each CTA: tcgen05.ld of its accumulator rows (two warps per 32-lane TMEM quarter,
//               each half of the columns), SwiGLU or the routing-weight scale, bf16 stores, then an arrival on
//               the leader's accumulator-empty barrier; the accumulator is double-buffered so the epilogue of one
//               tile overlaps the MMAs of the next.
// Expert row groups are padded to 128 rows; a 256-row tile whose second half belongs to the next expert computes
// it and the epilogue drops those rows. Decode-sized batches (a few dozen rows per expert) run a single-CTA shape of
// the same kernel instead: tcgen05.mma.cta_group::1 with M = 128, N = 256 (the CTA loads its 128 A rows and all
// 256 B rows, 48 KB per stage, 4 stages), because there the pair's M = 256 spends its tensor time on padding
// rows: the 256 x 256 x K products per weight tile bound those GEMMs, not the weight stream. Given the experts' row
// counts, the single-CTA shape also loads only the rows a tile holds (32-row boxes); the MMA still reads 128 A rows,
// and the rows past the last box are stale shared memory whose accumulator rows are padding rows of the segment. Work items are (expert, n-tile, m-tile) with the m-tile fastest, so the
// pairs running at one time share weight tiles through L2. Every mbarrier wait is bounded (~1 s): on expiry the
// kernel sets a status bit, stops issuing, drains (bounded), frees TMEM and returns.
#include <algorithm>

#include "tc_pair.cuh"

namespace {

constexpr int BM = 128, BN = 256, BK = 64;
constexpr int kEpilogueWarps = 8;               // two per TMEM lane quarter, each half of the columns
constexpr uint32_t kStageOutBytes = 32 * 64;     // per epilogue warp: 32 rows x 32 bf16 output columns
constexpr int kThreads = (2 + kEpilogueWarps) * 32;
constexpr uint32_t A_BYTES = BM * BK * 2;      // 16 KB: this CTA's A rows
constexpr uint32_t BOX_BYTES = BM * BK * 2;    // 16 KB: one 128-row B box
// the two shapes: a CTA pair (M = 256 over the pair, each CTA one of the two B boxes of the 256-wide tile) or one
// CTA (M = 128, both B boxes)
template <bool PAIR>
struct Shape {
  static constexpr int CTAS = PAIR ? 2 : 1;
  static constexpr int ROWS = CTAS * BM;                       // A rows of a tile
  static constexpr uint32_t B_BYTES = PAIR ? BOX_BYTES : 2 * BOX_BYTES;  // this CTA's B rows
  static constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = PAIR ? 6 : 4;
};
constexpr int kMaxStages = 6;
constexpr int kTmemCols = 512;
constexpr int kMaxExperts = 128;

// kFused: the SwiGLU GEMM (phase 0) and the down GEMM (phase 1) in one persistent launch of the single-CTA shape;
// a down tile of expert e starts once every SwiGLU tile of e has published its H columns (per-expert counters).
enum Mode : int { kSwiGLU = 0, kDown = 1, kFused = 2 };

struct GemmParams {
  const int32_t* offsets;  // [E + 1] padded row offsets (multiples of BM)
  const int32_t* counts;   // [E] routed rows of each expert, or null (every tile loads all 128 rows)
  int E;
  int K;                   // reduction length (multiple of BK)
  int n_tiles;             // output column tiles per expert
  int64_t b_rows_per_expert;  // rows of B per expert (2I for GEMM1, D for GEMM2)
  int b_second_offset;     // row offset of the second 128-row B box (I for GEMM1, 128 for GEMM2)
  int b_tile_step;         // B row advance per n-tile (128 for GEMM1, 256 for GEMM2)
  __nv_bfloat16* out;      // GEMM1: H [rows, I]; GEMM2: Y [pairs, D]
  int64_t out_stride;
  int out_cols;            // valid output columns (GEMM2: D, a multiple of 128; the last tile may be half)
  const int32_t* sorted_pairs;  // GEMM2
  const float* weights;         // GEMM2: [pairs]
  int64_t pair_limit;           // GEMM2: pairs >= this are dropped (the rows of `out`)
  unsigned* status;
  // kFused: the down GEMM's geometry (phase 1); the fields above describe the SwiGLU GEMM (phase 0)
  int K1, n_tiles1;
  int64_t b_rows1;
  int b_second1, b_step1;
  __nv_bfloat16* out1;
  int64_t out_stride1;
  int out_cols1;
  unsigned* flags;  // [E + 1]: per expert, SwiGLU epilogue warps done; [E]: CTAs done (zero between launches)
};

// The geometry of one phase's work items.
struct Phase {
  int mode, K, n_tiles;
  int64_t b_rows;
  int b_second, b_step;
  __nv_bfloat16* out;
  int64_t out_stride;
  int out_cols;
};
__device__ __forceinline__ Phase phase_of(const GemmParams& p, int MODE, int ph) {
  if (MODE == kFused && ph == 1)
    return Phase{kDown, p.K1, p.n_tiles1, p.b_rows1, p.b_second1, p.b_step1, p.out1, p.out_stride1, p.out_cols1};
  return Phase{MODE == kFused ? (int)kSwiGLU : MODE, p.K, p.n_tiles, p.b_rows_per_expert, p.b_second_offset,
               p.b_tile_step, p.out, p.out_stride, p.out_cols};
}

using zb::tcp::mbar_arrive_cluster;
using zb::tcp::tmem_ld32;

// SiLU with the fast exponential and division: the product silu(gate) * up is rounded to bf16, where their
// few-ulp fp32 error is far below the rounding step.
__device__ __forceinline__ float silu(float x) { return __fdividef(x, 1.0f + __expf(-x)); }

struct Shared {
  uint64_t full[kMaxStages];
  uint64_t empty[kMaxStages];
  uint64_t tmem_full[2];
  uint64_t tmem_empty[2];
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
  int item_start[kMaxExperts + 1];  // first work item of each expert (pair tiles x n-tiles)
  int item_start1[kMaxExperts + 1]; // kFused: the same for the down GEMM's items (after all SwiGLU items)
  int row_off[kMaxExperts + 1];     // padded row offsets
  int count[kMaxExperts];           // routed rows (counts, or the padded sizes)
};
constexpr uint32_t kSharedBytes = (sizeof(Shared) + 127) / 128 * 128;

// Waits until *counter >= target (acquire), for at most ~1 s; on expiry records kStatusGemmTimeout and returns false.
__device__ bool wait_counter(const unsigned* counter, unsigned target, unsigned* status) {
  const uint64_t start = zb::globaltimer_ns();
  for (;;) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(counter) : "memory");
    if (v >= target) return true;
    if (zb::globaltimer_ns() - start > 1000000000ull) {
      if (status) atomicOr(status, zb::kStatusGemmTimeout);
      return false;
    }
    __nanosleep(128);
  }
}

template <int MODE, bool PAIR>
__global__ void __launch_bounds__(kThreads, 1)
    moe_gemm_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_a32,
                    const __grid_constant__ CUtensorMap tmap_b, const __grid_constant__ CUtensorMap tmap_a1,
                    const __grid_constant__ CUtensorMap tmap_a1_32, const __grid_constant__ CUtensorMap tmap_b1,
                    GemmParams p) {
  zb::pdl_enter();
  using Sh = Shape<PAIR>;
  constexpr int STAGES = Sh::STAGES, CTAS = Sh::CTAS, ROWS = Sh::ROWS;
  constexpr uint32_t STAGE_BYTES = Sh::STAGE_BYTES;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  // stage buffers first, 1024-byte aligned (the 128B swizzle pattern repeats every 1024 bytes); the dynamic
  // shared-memory base is the same in both CTAs, so every buffer sits at the same offset in the pair
  const uint32_t raw_addr = zb::smem_addr(smem_raw);
  const uint32_t pad = (1024 - (raw_addr & 1023)) & 1023;
  unsigned char* stages = smem_raw + pad;
  Shared* sh = reinterpret_cast<Shared*>(stages + STAGES * STAGE_BYTES);
  // [kEpilogueWarps][32 rows x 64 B], 128-byte aligned after the barrier block
  unsigned char* out_stage = stages + STAGES * STAGE_BYTES + kSharedBytes;
  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  const uint32_t rank = PAIR ? (blockIdx.x & 1) : 0;  // cluster of 2 along x: rank 0 leads the pair
  const bool leader = rank == 0;
  const int pair = PAIR ? blockIdx.x >> 1 : blockIdx.x, npairs = PAIR ? gridDim.x >> 1 : gridDim.x;
  volatile int* abort_flag = &sh->abort;

  if (tid == 0) {
    for (int s = 0; s < STAGES; ++s) {
      zb::mbar_init(zb::smem_addr(&sh->full[s]), 1);
      zb::mbar_init(zb::smem_addr(&sh->empty[s]), 1);
    }
    for (int a = 0; a < 2; ++a) {
      zb::mbar_init(zb::smem_addr(&sh->tmem_full[a]), 1);
      zb::mbar_init(zb::smem_addr(&sh->tmem_empty[a]), CTAS * kEpilogueWarps);  // the epilogue warps of the CTAs
    }
    zb::mbar_init(zb::smem_addr(&sh->drain), 1);
    sh->abort = 0;
    zb::fence_mbar_init();
  }
  for (int e = tid; e <= p.E; e += kThreads) sh->row_off[e] = p.offsets[e];
  for (int e = tid; e < p.E; e += kThreads)
    sh->count[e] = p.counts ? p.counts[e] : p.offsets[e + 1] - p.offsets[e];
  __syncthreads();
  if (tid == 0) {  // work items per expert: ceil(128-row tiles / CTAS) tiles x n-tiles
    int acc = 0;
    for (int e = 0; e < p.E; ++e) {
      sh->item_start[e] = acc;
      const int m128 = (sh->row_off[e + 1] - sh->row_off[e]) / BM;
      acc += (m128 + CTAS - 1) / CTAS * p.n_tiles;
    }
    sh->item_start[p.E] = acc;
    if (MODE == kFused) {
      for (int e = 0; e < p.E; ++e) {
        sh->item_start1[e] = acc;
        acc += (sh->row_off[e + 1] - sh->row_off[e]) / BM * p.n_tiles1;
      }
      sh->item_start1[p.E] = acc;
    }
  }
  if (warp == 1) zb::tcp::tmem_alloc<PAIR>(zb::smem_addr(&sh->tmem_base), kTmemCols);
  zb::tcp::fence_before();
  __syncthreads();
  zb::cluster_arrive_relaxed();  // both CTAs' barriers are initialised before either signals the other's
  zb::cluster_wait();
  zb::tcp::fence_after();
  const uint32_t tmem_base = sh->tmem_base;
  const int E = p.E;
  const int items0 = sh->item_start[E];
  const int total_items = MODE == kFused ? sh->item_start1[E] : items0;

  // item -> (phase, expert, n-tile, first row of the 256-row pair tile)
  auto decode = [&](int item, int& ph, int& e, int& n, int& row0) {
    ph = (MODE == kFused && item >= items0) ? 1 : 0;
    const int* starts = ph ? sh->item_start1 : sh->item_start;
    const int ntl = ph ? p.n_tiles1 : p.n_tiles;
    int lo = 0, hi = E;  // largest e with starts[e] <= item
    while (hi - lo > 1) {
      const int mid = (lo + hi) / 2;
      if (starts[mid] <= item) lo = mid; else hi = mid;
    }
    e = lo;
    while (e + 1 < E && starts[e + 1] <= item) ++e;  // skip experts without tiles
    const int m_tiles = (starts[e + 1] - starts[e]) / ntl;
    const int local = item - starts[e];
    n = local / m_tiles;
    row0 = sh->row_off[e] + (local % m_tiles) * ROWS;
  };

  if (warp == 0) {
    if (lane == 0) {  // producer of this CTA's halves; bytes complete on the leader's full barrier
      uint32_t q = 0;
      for (int item = pair; item < total_items && !*abort_flag; item += npairs) {
        int ph, e, n, row0;
        decode(item, ph, e, n, row0);
        const Phase g = phase_of(p, MODE, ph);
        const CUtensorMap* ma = ph ? &tmap_a1 : &tmap_a;
        const CUtensorMap* ma32 = ph ? &tmap_a1_32 : &tmap_a32;
        const CUtensorMap* mb = ph ? &tmap_b1 : &tmap_b;
        const int k_blocks = g.K / BK;
        const int a_row = row0 + (int)rank * BM;
        const int b_row = (int)(e * g.b_rows) + n * g.b_step + (rank ? g.b_second : 0);
        const int b_row2 = b_row + g.b_second;  // the second B box (one CTA only)
        if (MODE == kFused && ph == 1) {
          // the down tile reads H rows of expert e: wait (bounded) until every SwiGLU tile of e has published them
          const unsigned target = (unsigned)(kEpilogueWarps * p.n_tiles * ((sh->row_off[e + 1] - sh->row_off[e]) / BM));
          if (!wait_counter(p.flags + e, target, p.status)) {
            *abort_flag = 1;
            break;
          }
          asm volatile("fence.proxy.async.global;" ::: "memory");  // the tensor loads below see those rows
        }
        // single CTA: 32-row A boxes covering the tile's routed rows (>= 1 for every tile of a segment)
        const int a_boxes = PAIR ? 4 : (min(max(sh->count[e] - (row0 - sh->row_off[e]), 0), BM) + 31) / 32;
        const uint32_t tx_bytes = CTAS * STAGE_BYTES - (uint32_t)(4 - a_boxes) * (A_BYTES / 4);
        for (int kb = 0; kb < k_blocks; ++kb, ++q) {
          const int s = q % STAGES;
          const uint32_t parity = ((q / STAGES) & 1) ^ 1;
          if (!zb::mbar_wait_bounded(zb::smem_addr(&sh->empty[s]), parity, p.status, zb::kStatusGemmTimeout)) {
            *abort_flag = 1;
            break;
          }
          const uint32_t full_local = zb::smem_addr(&sh->full[s]);
          if (leader) zb::mbar_arrive_expect_tx(full_local, tx_bytes);
          const uint32_t full_leader = PAIR ? zb::mapa_shared(full_local, 0) : full_local;
          const uint32_t a_dst = zb::smem_addr(stages + s * STAGE_BYTES);
          if (a_boxes == 4) {
            zb::tcp::tma_load_2d<PAIR>(a_dst, ma, kb * BK, a_row, full_leader);
          } else {
            for (int j = 0; j < a_boxes; ++j)
              zb::tcp::tma_load_2d<PAIR>(a_dst + j * (A_BYTES / 4), ma32, kb * BK, a_row + 32 * j, full_leader);
          }
          zb::tcp::tma_load_2d<PAIR>(a_dst + A_BYTES, mb, kb * BK, b_row, full_leader);
          if (!PAIR) zb::tcp::tma_load_2d<PAIR>(a_dst + A_BYTES + BOX_BYTES, mb, kb * BK, b_row2, full_leader);
        }
      }
      if (leader) {  // drain: wait (bounded) for the copies still in flight before the CTA may exit
        for (uint32_t d = 0; d < STAGES && d < q; ++d) {
          const uint32_t qq = q - 1 - d;
          zb::mbar_wait_bounded(zb::smem_addr(&sh->full[qq % STAGES]), (qq / STAGES) & 1, nullptr, 0, 200000000ull);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {  // the pair's MMA issuer
      uint32_t q = 0;
      int it = 0;
      for (int item = pair; item < total_items && !*abort_flag; item += npairs, ++it) {
        const int acc = it & 1;
        const uint32_t use = it >> 1;
        if (!zb::mbar_wait_bounded(zb::smem_addr(&sh->tmem_empty[acc]), (use & 1) ^ 1, p.status,
                                   zb::kStatusGemmTimeout)) {
          *abort_flag = 1;
          break;
        }
        zb::tcp::fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        int ph, e_, n_, row0_;
        decode(item, ph, e_, n_, row0_);
        const int k_blocks = phase_of(p, MODE, ph).K / BK;
        bool ok = true;
        for (int kb = 0; kb < k_blocks; ++kb, ++q) {
          const int s = q % STAGES;
          if (!zb::mbar_wait_bounded(zb::smem_addr(&sh->full[s]), (q / STAGES) & 1, p.status,
                                     zb::kStatusGemmTimeout)) {
            *abort_flag = 1;
            ok = false;
            break;
          }
          zb::tcp::fence_after();
          const uint32_t a_addr = zb::smem_addr(stages + s * STAGE_BYTES);
          const uint32_t b_addr = a_addr + A_BYTES;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            zb::tcp::mma<PAIR>(d_tmem, zb::tcp::desc_sw128(a_addr + kk * 32), zb::tcp::desc_sw128(b_addr + kk * 32),
                               zb::tcp::idesc(ROWS, BN), (kb > 0 || kk > 0) ? 1u : 0u);
          }
          zb::tcp::commit<PAIR>(zb::smem_addr(&sh->empty[s]), 0x3);  // stage s (of both CTAs of a pair) is free
        }
        if (!ok) break;
        zb::tcp::commit<PAIR>(zb::smem_addr(&sh->tmem_full[acc]), 0x3);
      }
      // every MMA issued by this thread has completed before TMEM is released
      zb::tcp::commit<PAIR>(zb::smem_addr(&sh->drain), 0x1);
      zb::mbar_wait_bounded(zb::smem_addr(&sh->drain), 0, nullptr, 0, 200000000ull);
    }
  } else {
    // epilogue warps 2..9: TMEM lane quarter (warp % 4) of this CTA's 128 accumulator rows, column half
    // (warp - 2) / 4 of the tile
    const int quarter = warp % 4, chalf = (warp - 2) / 4;
    const int row_in_tile = (int)rank * BM + quarter * 32 + lane;
    int it = 0;
    for (int item = pair; item < total_items; item += npairs, ++it) {
      const int acc = it & 1;
      const uint32_t use = it >> 1;
      // the tile's rows (and, for the down projection, their pairs and routing weights) are looked up while the
      // MMAs still run
      int ph, e, n, row0;
      decode(item, ph, e, n, row0);
      const Phase g = phase_of(p, MODE, ph);
      const int64_t row = row0 + row_in_tile;
      const bool valid = row < sh->row_off[e + 1];  // rows past the expert's group belong to the next expert
      int pr = -1;
      float w = 0.f;
      if (g.mode == kDown) {
        pr = valid ? p.sorted_pairs[row] : -1;
        if (pr >= p.pair_limit) pr = -1;  // never write past the rows of `out`
        w = pr >= 0 ? p.weights[pr] : 0.f;
      }
      bool ok = !*abort_flag &&
                zb::mbar_wait_bounded(zb::smem_addr(&sh->tmem_full[acc]), use & 1, p.status, zb::kStatusGemmTimeout);
      // the tcgen05.ld below are warp-collective: every lane takes the same branch
      if (!__all_sync(0xffffffffu, ok)) {
        *abort_flag = 1;
        break;
      }
      zb::tcp::fence_after();
      const uint32_t t_row = tmem_base + ((uint32_t)(quarter * 32) << 16) + acc * BN;
      if (g.mode == kSwiGLU) {
        __nv_bfloat16* dst = g.out + row * g.out_stride + (int64_t)n * 128;
#pragma unroll 1
        for (int c = chalf * 64; c < chalf * 64 + 64; c += 32) {
          float gate[32], up[32];
          tmem_ld32(t_row + c, gate);
          tmem_ld32(t_row + 128 + c, up);
          if (valid) {
#pragma unroll
            for (int j = 0; j < 32; j += 8) {
              float h[8];
#pragma unroll
              for (int i = 0; i < 8; ++i)
                h[i] = silu(zb::bf16_round(gate[j + i])) * zb::bf16_round(up[j + i]);
              *reinterpret_cast<uint4*>(dst + c + j) = zb::pack_bf16x8(h);
            }
          }
        }
        if (MODE == kFused) {  // publish this warp's H columns of expert e to the down tiles (release)
          __threadfence();
          asm volatile("fence.proxy.async.global;" ::: "memory");
          __syncwarp();
          if (lane == 0) asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(p.flags + e) : "memory");
        }
      } else {
        // rows go to scattered pair slots: each 32-column chunk of the warp's 32 rows is staged in shared memory
        // (16-byte units swizzled by row so that neither the row-wise writes nor the column-wise reads conflict)
        // and written back as 64-byte row segments, four lanes per row
        unsigned char* stg = out_stage + (warp - 2) * kStageOutBytes;
        const int sub = lane & 3, rsub = lane >> 2;
#pragma unroll 1
        for (int c = chalf * (BN / 2); c < chalf * (BN / 2) + BN / 2 && n * BN + c < g.out_cols; c += 32) {
          float y[32];
          tmem_ld32(t_row + c, y);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            float o[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) o[i] = y[8 * j + i] * w;
            const int unit = 4 * (lane & 1) + (j ^ ((lane >> 1) & 3));
            *reinterpret_cast<uint4*>(stg + (lane >> 1) * 128 + unit * 16) = zb::pack_bf16x8(o);
          }
          __syncwarp();
#pragma unroll
          for (int it = 0; it < 4; ++it) {
            const int r = it * 8 + rsub;  // row of the warp handled by this lane; segment `sub`
            const int rp = __shfl_sync(0xffffffffu, pr, r);
            const int unit = 4 * (r & 1) + (sub ^ ((r >> 1) & 3));
            const uint4 v = *reinterpret_cast<const uint4*>(stg + (r >> 1) * 128 + unit * 16);
            if (rp >= 0)
              *reinterpret_cast<uint4*>(g.out + (int64_t)rp * g.out_stride + (int64_t)n * BN + c + 8 * sub) = v;
          }
          __syncwarp();
        }
      }
      zb::tcp::fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(zb::mapa_shared(zb::smem_addr(&sh->tmem_empty[acc]), 0));
    }
  }
  zb::tcp::fence_before();
  __syncthreads();
  zb::cluster_arrive_relaxed();  // neither CTA frees TMEM or exits while the pair may still use it
  zb::cluster_wait();
  if (warp == 1) {
    zb::tcp::fence_after();
    zb::tcp::tmem_dealloc<PAIR>(tmem_base, kTmemCols);
  }
  if (MODE == kFused && tid == 0) {  // the last CTA to finish zeroes the counters for the next launch
    __threadfence();
    if (atomicAdd(p.flags + E, 1u) == gridDim.x - 1)
      for (int e = 0; e <= E; ++e) reinterpret_cast<volatile unsigned*>(p.flags)[e] = 0u;
  }
}

// ------------------------------------------------------------------------------------------ host side

int make_map(CUtensorMap* map, const void* base, int64_t rows, int64_t cols, int64_t row_stride_elems,
             uint32_t box_rows = 128) {
  return zb::tcp::make_map(map, base, rows, cols, row_stride_elems, box_rows, "moe_gemm");
}

template <bool PAIR>
constexpr size_t smem_bytes() {
  return 1024 + Shape<PAIR>::STAGES * Shape<PAIR>::STAGE_BYTES + kSharedBytes + kEpilogueWarps * kStageOutBytes;
}

// The single-CTA shape for batches whose permuted layout (capacity rows over E experts) averages at most 96 routed
// rows per expert (decode), the pair shape otherwise.
bool use_pair(int64_t capacity, int E) {
  const int64_t routed = capacity - (int64_t)E * (BM - 1);  // about the pairs the capacity was sized for
  return routed > (int64_t)E * 96;
}

// The tensor maps of a launch: A (128- and 32-row boxes) and B of the GEMM, and for kFused those of the down GEMM.
struct Maps {
  CUtensorMap a, a32, b, a1, a1_32, b1;
};

template <int MODE, bool PAIR>
int launch(const Maps& m, const GemmParams& p, int64_t capacity, cudaStream_t stream) {
  auto kernel = moe_gemm_kernel<MODE, PAIR>;
  constexpr size_t kSmemBytes = smem_bytes<PAIR>();
  static_assert(kSmemBytes <= 227 * 1024, "shared memory of one CTA");
  static int configured[64] = {0};
  int dev = 0;
  ZB_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64 || !configured[dev]) {
    ZB_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes));
    if (dev >= 0 && dev < 64) configured[dev] = 1;
  }
  // the persistent loop assumes every CTA (pair) is resident at once: as many as the GPU co-schedules (a pair
  // needs two SMs of one GPC), cached per device
  static int resident[64] = {0};
  int max_units = dev >= 0 && dev < 64 ? resident[dev] : 0;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = Shape<PAIR>::CTAS;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  if (max_units == 0) {
    if constexpr (PAIR) {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(2);
      cfg.blockDim = dim3(kThreads);
      cfg.dynamicSmemBytes = kSmemBytes;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      ZB_CUDA(cudaOccupancyMaxActiveClusters(&max_units, kernel, &cfg));
    } else {
      int per_sm = 0, sms = 0;
      ZB_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kThreads, kSmemBytes));
      ZB_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
      max_units = per_sm * sms;
    }
    if (max_units < 1) return zb::fail(zb::kUnsupported, "moe_gemm: no CTA (pair) fits on this GPU");
    if (dev >= 0 && dev < 64) resident[dev] = max_units;
  }
  // tiles: at most capacity / tile rows plus one per expert (kFused: of both GEMMs). kFused waits on other CTAs'
  // tiles, so it relies on every CTA of the grid being resident at once (the grid never exceeds max_units).
  const int64_t upper_items =
      (capacity / Shape<PAIR>::ROWS + p.E) * (p.n_tiles + (MODE == kFused ? p.n_tiles1 : 0));
  const int units = (int)std::min<int64_t>(upper_items, max_units);
  if (units <= 0) return zb::kOk;
  ZB_CUDA(zb::launch(kernel, dim3((unsigned)(Shape<PAIR>::CTAS * units)), dim3(kThreads), kSmemBytes, stream,
                     (unsigned)Shape<PAIR>::CTAS, m.a, m.a32, m.b, m.a1, m.a1_32, m.b1, p));
  return zb::check_launch(MODE == kSwiGLU ? "moe_gemm_swiglu" : MODE == kDown ? "moe_gemm_down" : "moe_gemm_fused");
}

int check_common(const void* a, const int32_t* offsets, int E, int64_t capacity) {
  ZB_REQUIRE(a && offsets, "moe_gemm: null pointer");
  ZB_REQUIRE(E > 0 && E <= kMaxExperts, "moe_gemm: E=%d (1..%d)", E, kMaxExperts);
  ZB_REQUIRE(capacity > 0 && capacity % BM == 0, "moe_gemm: capacity %lld must be a positive multiple of %d",
             (long long)capacity, BM);
  ZB_REQUIRE_ALIGNED(a, 16, "A");
  return zb::kOk;
}

}  // namespace

ZB_API int zb_moe_gemm_swiglu(const uint16_t* x_perm, int64_t capacity, const uint16_t* gate_up, int E, int D, int I,
                              const int32_t* offsets, const int32_t* counts, uint16_t* h, cudaStream_t stream) {
  if (int rc = check_common(x_perm, offsets, E, capacity)) return rc;
  ZB_REQUIRE(gate_up && h, "moe_gemm_swiglu: null pointer");
  if (D % BK != 0 || I % 128 != 0)
    return zb::fail(zb::kUnsupported, "moe_gemm_swiglu: D=%d must be a multiple of 64 and I=%d of 128", D, I);
  ZB_REQUIRE_ALIGNED(gate_up, 16, "gate_up");
  ZB_REQUIRE_ALIGNED(h, 16, "h");
  Maps m;
  if (int rc = make_map(&m.a, x_perm, capacity, D, D)) return rc;
  if (int rc = make_map(&m.a32, x_perm, capacity, D, D, 32)) return rc;
  if (int rc = make_map(&m.b, gate_up, (int64_t)E * 2 * I, D, D)) return rc;
  m.a1 = m.a, m.a1_32 = m.a32, m.b1 = m.b;
  GemmParams p{offsets, counts, E, D, I / 128, 2 * (int64_t)I, I, 128, reinterpret_cast<__nv_bfloat16*>(h), I, I,
               nullptr, nullptr, 0, zb::device_status_ptr()};
  return use_pair(capacity, E) ? launch<kSwiGLU, true>(m, p, capacity, stream)
                                : launch<kSwiGLU, false>(m, p, capacity, stream);
}

namespace zb {

// The down projection with its pair rows bounded: a pair id >= pair_limit (a row `y` does not have) is dropped.
int moe_gemm_down_bounded(const uint16_t* h, int64_t capacity, const uint16_t* down, int E, int D, int I,
                          const int32_t* offsets, const int32_t* counts, const int32_t* sorted_pairs,
                          const float* weights, uint16_t* y, int64_t pair_limit, cudaStream_t stream) {
  if (int rc = check_common(h, offsets, E, capacity)) return rc;
  ZB_REQUIRE(down && sorted_pairs && weights && y, "moe_gemm_down: null pointer");
  if (I % BK != 0 || D % 128 != 0)
    return zb::fail(zb::kUnsupported, "moe_gemm_down: I=%d must be a multiple of 64 and D=%d of 128", I, D);
  ZB_REQUIRE_ALIGNED(down, 16, "down");
  ZB_REQUIRE_ALIGNED(y, 16, "y");
  Maps m;
  if (int rc = make_map(&m.a, h, capacity, I, I)) return rc;
  if (int rc = make_map(&m.a32, h, capacity, I, I, 32)) return rc;
  if (int rc = make_map(&m.b, down, (int64_t)E * D, I, I)) return rc;
  m.a1 = m.a, m.a1_32 = m.a32, m.b1 = m.b;
  GemmParams p{offsets, counts, E, I, (D + BN - 1) / BN, (int64_t)D, 128, BN, reinterpret_cast<__nv_bfloat16*>(y), D,
               D, sorted_pairs, weights, pair_limit, zb::device_status_ptr()};
  return use_pair(capacity, E) ? launch<kDown, true>(m, p, capacity, stream)
                                : launch<kDown, false>(m, p, capacity, stream);
}

}  // namespace zb

ZB_API int zb_moe_gemm_down(const uint16_t* h, int64_t capacity, const uint16_t* down, int E, int D, int I,
                            const int32_t* offsets, const int32_t* counts, const int32_t* sorted_pairs,
                            const float* weights, uint16_t* y, cudaStream_t stream) {
  // a permutation of capacity rows holds pair ids below capacity (zb_moe_permute never writes more)
  return zb::moe_gemm_down_bounded(h, capacity, down, E, D, I, offsets, counts, sorted_pairs, weights, y, capacity,
                                   stream);
}

ZB_API int zb_moe_gemms(const uint16_t* x_perm, int64_t capacity, const uint16_t* gate_up, const uint16_t* down,
                        int E, int D, int I, const int32_t* offsets, const int32_t* counts,
                        const int32_t* sorted_pairs, const float* weights, uint16_t* h, uint16_t* y, uint32_t* flags,
                        cudaStream_t stream) {
  if (int rc = check_common(x_perm, offsets, E, capacity)) return rc;
  if (use_pair(capacity, E)) {  // prefill-sized batches: the two pair-shape launches
    if (int rc = zb_moe_gemm_swiglu(x_perm, capacity, gate_up, E, D, I, offsets, counts, h, stream)) return rc;
    return zb_moe_gemm_down(h, capacity, down, E, D, I, offsets, counts, sorted_pairs, weights, y, stream);
  }
  ZB_REQUIRE(gate_up && down && sorted_pairs && weights && h && y && flags, "moe_gemms: null pointer");
  if (D % BK != 0 || I % BK != 0 || I % 128 != 0 || D % 128 != 0)
    return zb::fail(zb::kUnsupported, "moe_gemms: D=%d and I=%d must be multiples of 128", D, I);
  for (const void* ptr : {(const void*)gate_up, (const void*)down, (const void*)h, (const void*)y}) {
    ZB_REQUIRE_ALIGNED(ptr, 16, "moe_gemms tensors");
  }
  Maps m;
  if (int rc = make_map(&m.a, x_perm, capacity, D, D)) return rc;
  if (int rc = make_map(&m.a32, x_perm, capacity, D, D, 32)) return rc;
  if (int rc = make_map(&m.b, gate_up, (int64_t)E * 2 * I, D, D)) return rc;
  if (int rc = make_map(&m.a1, h, capacity, I, I)) return rc;
  if (int rc = make_map(&m.a1_32, h, capacity, I, I, 32)) return rc;
  if (int rc = make_map(&m.b1, down, (int64_t)E * D, I, I)) return rc;
  GemmParams p{offsets, counts, E, D, I / 128, 2 * (int64_t)I, I, 128, reinterpret_cast<__nv_bfloat16*>(h), I, I,
               sorted_pairs, weights, capacity, zb::device_status_ptr()};
  p.K1 = I;
  p.n_tiles1 = (D + BN - 1) / BN;
  p.b_rows1 = D;
  p.b_second1 = 128;
  p.b_step1 = BN;
  p.out1 = reinterpret_cast<__nv_bfloat16*>(y);
  p.out_stride1 = D;
  p.out_cols1 = D;
  p.flags = flags;
  return launch<kFused, false>(m, p, capacity, stream);
}

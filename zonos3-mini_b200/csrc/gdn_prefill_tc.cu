// Gated-DeltaNet chunked prefill for d_k = d_v = 128 on 5th-generation tensor cores (tcgen05 + TMEM), sm_100a.
//
// Same algorithm and rounding class as the d = 64 kernel in gdn_prefill.cu (WY / UT form, chunk C = 64, fp32 state,
// every fp32 operand of a product split into bf16 hi + lo); reference: FLA chunk_gated_delta_rule_fwd as called by
// OriginalGDN._run_packed (servers/sgl/src/zonos3_sgl/models/gdn.py:418-434), equal to the per-token recurrence of
// model/src/zonos3/reference/lm.py:576-582. With S the K-first state (S^T = the reference's V-first M), per chunk:
//   A_ts = beta_t e^{G_t - G_s} k_t.k_s (s < t),  T = (I + A)^{-1},  P_ts = scale e^{G_t - G_s} q_t.k_s (s <= t)
//   Y = diag(beta)(V - diag(gamma) K S0),  U = T Y,  O = scale diag(gamma) Q S0 + P U
//   S_C = gamma_C S0 + (diag(f) K)^T U,  f_t = e^{G_C - G_t}
//
// Two kernels. The state-independent part of every chunk runs first, all (chunk, head) pairs in parallel:
//   gdn_prefill_prep_kernel (one CTA of 4 warps per chunk and head): decay scan (G, gamma, f), [K;Q] K^T on tcgen05
//   (M = 128 rows of K then Q, N = 64, K = 128, accumulator in TMEM), A and P from it, T = (I + A)^{-1} in fp32
//   (16 x 16 diagonal blocks by substitution, then the off-diagonal blocks row-block by row-block), and T and P
//   split into bf16 hi + lo in the 128B-swizzled K-major layout the tensor cores read; one 33 KB record per
//   (chunk, head) goes to a workspace with one bulk copy.
// Then the sequential state pass, gdn_prefill_state_kernel: one CTA (8 warps) per (sequence, head) walks its chunks
// in order. Every product is a tcgen05.mma with the accumulator in tensor memory; the operands that change with the
// state (S^T, Y^T, U^T; rows = value index) are the A operand read from TMEM, the state-independent ones (K, Q, T,
// P, (fK)^T) are B operands in swizzled shared memory. TMEM columns (512, lane = value index v):
//   [  0,128) S^T fp32 master            [128,192) S^T bf16 hi (packed pairs)   [192,256) S^T bf16 lo
//   [256,320) (K S0)^T                   [320,384) (Q S0)^T, then O^T            [384,448) U^T
//   [448,480) Y^T / U^T bf16 hi          [480,512) Y^T / U^T bf16 lo
// Per chunk:  M2  S^T [K;Q]^T  (S hi, S lo)   (A: TMEM, B: K and Q rows)  -> (K S0)^T, (Q S0)^T
//             threads: Y^T hi/lo from M2 and V into TMEM; O^T *= scale gamma_t
//             M3  Y^T T^T  (hh, hl, lh)                                   -> U^T
//             threads: U^T hi/lo into TMEM
//             M4  S^T += U^T (fK)  and  O^T += U^T P^T  (hh, hl, lh each); meanwhile the threads build the next
//                 chunk's (fK)^T hi/lo from its K rows (ldmatrix.trans / stmatrix, double-buffered tiles)
//             threads: S^T master -> hi/lo for the next chunk's M2, master *= the next chunk's gamma_C (so M4 can
//             accumulate onto it); then M2 of the next chunk is issued and this chunk's O^T is written as bf16 rows
//             (staged in shared memory, 256-byte row stores) while it runs
// K, Q and the prep record (one bulk copy) of a chunk load one chunk ahead (double-buffered); V has one buffer and
// loads after the Y step of the chunk before; cp.async rows past the sequence end are zero-filled. Every mbarrier
// wait is bounded (~1 s); on expiry the kernel records kStatusPrefillTimeout, stops, frees TMEM and returns.
//
// Chunk records are addressed by id = cu[s] / 64 + s + c for chunk c of sequence s: ids of one sequence are
// consecutive and those of the next start higher, so ids lie in [0, ceil(N / 64) + num_seqs).
#include "common.cuh"

namespace {

constexpr int C = 64;          // chunk length
constexpr int D = 128;         // d_k = d_v
constexpr int LC = C + 4;      // fp32 row length of the inverse workspace

// prep record (workspace, per (chunk id, head)); the tiles are 128B-swizzled as if based at a 1024-aligned address
constexpr uint32_t kRecTh = 0, kRecTl = 8192, kRecPh = 16384, kRecPl = 24576;
constexpr uint32_t kRecG = 32768, kRecGam = kRecG + 256, kRecBet = kRecG + 512, kRecEf = kRecG + 768;
constexpr uint32_t kRecBytes = kRecG + 1024;  // 33,792

// ---- prep kernel
constexpr int kPrepThreads = 128;
constexpr uint32_t kPrepKQ = 0;                       // KQ tile (32 KB); after M1 the record staging over it
constexpr uint32_t kPrepTf = kRecBytes;               // fp32 [C][LC]: A, then T
constexpr uint32_t kPrepYs = kPrepTf + C * LC * 4;    // fp32 [3][16][16]: sums of the off-diagonal blocks
constexpr uint32_t kPrepSmall = kPrepYs + 3 * 256 * 4;
struct PrepSmall {
  float graw[C];
  float braw[C];
  float rf[C];       // e^{G_t - G_{16 (t / 16)}}
  float cf[4 * C];   // [row block i][s]: e^{G_{16 i} - G_s} for s < 16 (i + 1)
  int fast;          // factored decays usable for this chunk
  uint64_t bar;
  uint32_t tmem_base;
};
constexpr uint32_t kPrepSmem = 1024 + kPrepSmall + sizeof(PrepSmall);

// ---- state kernel
constexpr int kEpiThreads = 256;             // warps 0-7: loads and the TMEM / shared-memory steps
constexpr int kThreads = kEpiThreads + 32;   // warp 8: issues the tensor-core MMAs
constexpr uint32_t kColMaster = 0, kColSh = 128, kColSl = 192, kColKS = 256, kColQS = 320, kColU = 384,
                   kColYh = 448, kColYl = 480;
constexpr uint32_t kKQBytes = 2 * 128 * 128;           // 2 k-atoms of [128 rows][128 B]
constexpr uint32_t kVBytes = C * D * 2;                // row-major [t][v]
constexpr uint32_t kFKTBytes = D * 128;                // [dk][t], one k-atom
constexpr uint32_t kRecSlot = (kRecBytes + 1023) / 1024 * 1024;
constexpr uint32_t kOffKQ = 0;                         // [2]
constexpr uint32_t kOffV = kOffKQ + 2 * kKQBytes;      // one buffer: the next chunk's V loads after this Y step
constexpr uint32_t kOffRec = kOffV + kVBytes;          // [2]
constexpr uint32_t kOffFKT = kOffRec + 2 * kRecSlot;   // [2] x (hi, lo)
constexpr uint32_t kOffSmall = kOffFKT + 4 * kFKTBytes;
struct Small {
  uint64_t bar_rec[2];
  uint64_t bar_m2, bar_m3, bar_m4, bar_m4o;
  uint32_t tmem_base;
  int abort;
};
constexpr uint32_t kSmemBytes = 1024 + kOffSmall + sizeof(Small);

struct PrepParams {
  const __nv_bfloat16* q;  // [N, H, D]
  const __nv_bfloat16* k;
  const float* g;          // [N, H]
  const float* beta;
  const int32_t* cu_seqlens;
  int num_seqs;
  int H;
  float scale;
  unsigned char* records;  // [ids, H] x kRecBytes
  unsigned* status;
};

struct StateParams {
  const __nv_bfloat16* q;
  const __nv_bfloat16* k;
  const __nv_bfloat16* v;
  const int32_t* cu_seqlens;
  const float* init_state;     // [*, H, D(v), D(k)] or null
  const int64_t* state_slots;  // optional row of init/final per sequence
  float* final_state;
  __nv_bfloat16* out;          // [N, H, D]
  const unsigned char* records;
  int H;
  float scale;
  unsigned* status;
};

// ------------------------------------------------------------------------------------------ PTX wrappers

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(valid ? 16 : 0) : "memory");
}
__device__ __forceinline__ void cp_async4(uint32_t dst, const void* src, bool valid) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(dst), "l"(src), "r"(valid ? 4 : 0) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem] B[smem]^T
__device__ __forceinline__ void mma_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// D[tmem] (+)= A[tmem] B[smem]^T
__device__ __forceinline__ void mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

// 128B-swizzled K-major operand descriptor (8-row groups 1024 bytes apart).
__device__ __forceinline__ uint64_t desc_sw128(uint32_t addr) {
  uint64_t d = 0;
  d |= (uint64_t)((addr >> 4) & 0x3FFF);
  d |= (uint64_t)1 << 16;
  d |= (uint64_t)(1024 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// kind::f16, bf16 A and B (K-major), fp32 accumulator, M = 128.
__host__ __device__ constexpr uint32_t idesc_m128(int n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
}

__device__ __forceinline__ void tmem_ld32_nowait(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
      "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
      "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// (x0, x1) = hi + lo, each a packed bf16 pair (x0 in the low half); two-wide conversions
__device__ __forceinline__ void split_pair(float x0, float x1, uint32_t& hi, uint32_t& lo) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(x0, x1);
  const float2 hf = __bfloat1622float2(h);
  const __nv_bfloat162 l = __floats2bfloat162_rn(x0 - hf.x, x1 - hf.y);
  hi = *reinterpret_cast<const uint32_t*>(&h);
  lo = *reinterpret_cast<const uint32_t*>(&l);
}

// four 8x8 b16 matrices, transposed on load: lane l addresses row (l % 8) of matrix (l / 8)
__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr)
               : "memory");
}
// four 8x8 b16 matrices stored (lane l addresses row (l % 8) of matrix (l / 8))
__device__ __forceinline__ void stsm_x4(uint32_t addr, const uint32_t (&r)[4]) {
  asm volatile("stmatrix.sync.aligned.m8n8.x4.shared.b16 [%0], {%1,%2,%3,%4};" ::"r"(addr), "r"(r[0]), "r"(r[1]),
               "r"(r[2]), "r"(r[3])
               : "memory");
}

// byte offset of 16-byte chunk `ch` (8 columns) of `row`
__device__ __forceinline__ uint32_t sw128_chunk(int row, int ch) {
  return (uint32_t)(row * 128 + (((ch ^ row) & 7) << 4));
}

// bulk copy shared -> global (this CTA's bulk group)
__device__ __forceinline__ void bulk_s2g(void* dst, uint32_t src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst), "r"(src), "r"(bytes)
               : "memory");
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem), "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// K / Q rows of chunk c of the sequence at t_begin (len tokens) into a KQ tile: rows 0-63 K, 64-127 Q, 2 k-atoms
// of 128B-swizzled rows; rows past the end are zero-filled.
__device__ __forceinline__ void load_kq(uint32_t kq, const __nv_bfloat16* kp, const __nv_bfloat16* qp,
                                        int64_t t_begin, int64_t len, int c, int64_t row_stride, int h, int tid,
                                        int nthreads) {
  for (int i = tid; i < 2 * C * 16; i += nthreads) {
    const int r = i >> 4, cidx = i & 15;
    const int t = r & (C - 1);
    const int64_t tok = (int64_t)c * C + t;
    const bool ok = tok < len;
    const __nv_bfloat16* src = (r < C ? kp : qp) + (t_begin + (ok ? tok : 0)) * row_stride + (int64_t)h * D + cidx * 8;
    cp_async16(kq + (cidx >> 3) * (128 * 128) + sw128_chunk(r, cidx & 7), src, ok);
  }
}

// A row t (is_a: beta_t e^{G_t - G_s} (K K^T)_ts for s < t, fp32 into Tf) or P row t (scale e^{G_t - G_s} (Q K^T)_ts
// for s <= t, split into the record's P hi / lo tiles) from the 64 accumulator columns of this thread's TMEM lane.
// kFactored: decays from the factors rf / cf; otherwise one fast exponential per element (its relative error, a
// few 1e-6 for exponents down to -40, is below the ~2^-17 of the bf16 hi + lo operands it feeds).
template <bool kFactored>
__device__ __forceinline__ void decay_epilogue(bool is_a, int t, const uint32_t (&r0)[32], const uint32_t (&r1)[32],
                                               const float* G, const float* bet, const float* rf, const float* cf,
                                               float scale, float* Tf, unsigned char* base) {
  const float Gt = G[t];
  const float* cfr = cf + C * (t >> 4);
  auto decay = [&](int s) { return kFactored ? cfr[s] : __expf(Gt - G[s]); };
  if (is_a) {
    const float rowf = bet[t] * (kFactored ? rf[t] : 1.f);
    float* dst = Tf + t * LC;
#pragma unroll
    for (int s = 0; s < C; s += 4) {
      float4 a;
      float* av = &a.x;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int ss = s + e;
        const float x = __uint_as_float(ss < 32 ? r0[ss] : r1[ss - 32]);
        av[e] = ss < t ? rowf * decay(ss) * x : 0.f;
      }
      *reinterpret_cast<float4*>(dst + s) = a;
    }
  } else {
    const float rowf = scale * (kFactored ? rf[t] : 1.f);
#pragma unroll
    for (int ch = 0; ch < 8; ++ch) {
      uint32_t hv[4], lv[4];
#pragma unroll
      for (int e = 0; e < 8; e += 2) {
        const int s0 = 8 * ch + e;
        const float x0 = __uint_as_float(s0 < 32 ? r0[s0] : r1[s0 - 32]);
        const float x1 = __uint_as_float(s0 + 1 < 32 ? r0[s0 + 1] : r1[s0 + 1 - 32]);
        const float p0 = s0 <= t ? rowf * decay(s0) * x0 : 0.f;
        const float p1 = s0 + 1 <= t ? rowf * decay(s0 + 1) * x1 : 0.f;
        split_pair(p0, p1, hv[e / 2], lv[e / 2]);
      }
      *reinterpret_cast<uint4*>(base + kRecPh + sw128_chunk(t, ch)) = make_uint4(hv[0], hv[1], hv[2], hv[3]);
      *reinterpret_cast<uint4*>(base + kRecPl + sw128_chunk(t, ch)) = make_uint4(lv[0], lv[1], lv[2], lv[3]);
    }
  }
}

__global__ void __launch_bounds__(kPrepThreads) gdn_prefill_prep_kernel(PrepParams p) {
  zb::pdl_enter();
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  const uint32_t raw_addr = zb::smem_addr(smem_raw);
  const uint32_t pad = (1024 - (raw_addr & 1023)) & 1023;
  unsigned char* base = smem_raw + pad;
  const uint32_t sbase = raw_addr + pad;
  PrepSmall& sm = *reinterpret_cast<PrepSmall*>(base + kPrepSmall);
  float* Tf = reinterpret_cast<float*>(base + kPrepTf);
  float* Ys = reinterpret_cast<float*>(base + kPrepYs);
  float* G = reinterpret_cast<float*>(base + kRecG);
  float* gam = reinterpret_cast<float*>(base + kRecGam);
  float* bet = reinterpret_cast<float*>(base + kRecBet);
  float* ef = reinterpret_cast<float*>(base + kRecEf);

  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  const int id = blockIdx.x, h = blockIdx.y;
  // sequence of this chunk id: the last s with cu[s] / 64 + s <= id
  if (p.num_seqs <= 0) return;
  int lo = 0, hi = p.num_seqs - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (p.cu_seqlens[mid] / C + mid <= id) lo = mid; else hi = mid - 1;
  }
  const int seq = lo;
  const int64_t t_begin = p.cu_seqlens[seq], len = p.cu_seqlens[seq + 1] - t_begin;
  const int c = id - (int)(t_begin / C) - seq;
  if (c < 0 || (int64_t)c * C >= len) return;  // an unused id (uniform over the CTA)
  const int64_t row_stride = (int64_t)p.H * D;

  load_kq(sbase + kPrepKQ, p.k, p.q, t_begin, len, c, row_stride, h, tid, kPrepThreads);
  if (tid < 2 * C) {
    const int t = tid & (C - 1);
    const int64_t tok = (int64_t)c * C + t;
    const bool ok = tok < len;
    cp_async4(zb::smem_addr(tid < C ? &sm.graw[t] : &sm.braw[t]),
              (tid < C ? p.g : p.beta) + (t_begin + (ok ? tok : 0)) * p.H + h, ok);
  }
  cp_async_commit();
  const uint32_t bar = zb::smem_addr(&sm.bar);
  if (tid == 0) {
    zb::mbar_init(bar, 1);
    zb::fence_mbar_init();
  }
  if (warp == 0) tmem_alloc(zb::smem_addr(&sm.tmem_base), 64);
  cp_async_wait_all();
  fence_proxy_async();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;

  // ---- M1: [K;Q] K^T -> TMEM lanes 0-63 (K K^T), 64-127 (Q K^T)
  if (tid == 0) {
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      const uint32_t off = sbase + kPrepKQ + (ks >> 2) * (128 * 128) + (ks & 3) * 32;
      mma_ss(tmem, desc_sw128(off), desc_sw128(off), idesc_m128(64), ks > 0);
    }
    mma_commit(bar);
  }
  // ---- decay scan (the record's vectors sit after the KQ tile, outside what M1 reads)
  if (warp == 0) {
    const float a0 = sm.graw[2 * lane], a1 = sm.graw[2 * lane + 1];
    float incl = a0 + a1;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const float o = __shfl_up_sync(0xffffffffu, incl, off);
      if (lane >= off) incl += o;
    }
    const float g0 = incl - a1, g1 = incl;
    const float gC = __shfl_sync(0xffffffffu, incl, 31);
    G[2 * lane] = g0;
    G[2 * lane + 1] = g1;
    gam[2 * lane] = expf(g0);
    gam[2 * lane + 1] = expf(g1);
    ef[2 * lane] = expf(gC - g0);
    ef[2 * lane + 1] = expf(gC - g1);
    bet[2 * lane] = sm.braw[2 * lane];
    bet[2 * lane + 1] = sm.braw[2 * lane + 1];
    // factored decays: e^{G_t - G_s} = e^{G_t - G_{16i}} e^{G_{16i} - G_s} for t in row block i and s <= t. With
    // every g <= 0 (G non-increasing) and at most 80 of decay inside any 16-token block, both factors lie in
    // [0, e^80] and the product is the decay to rounding; otherwise the per-element path is used.
    __syncwarp();
    const float blk_range = G[(lane & 3) * 16] - G[(lane & 3) * 16 + 15];
    const bool fast = __all_sync(0xffffffffu, a0 <= 0.f && a1 <= 0.f && blk_range <= 80.f);
    if (lane == 0) sm.fast = fast ? 1 : 0;
    if (fast) {
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int t = 2 * lane + u;
        sm.rf[t] = expf(G[t] - G[t & ~15]);
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int e = 32 * u + lane, i = e >> 6, sidx = e & 63;
        sm.cf[e] = sidx < 16 * (i + 1) ? expf(G[16 * i] - G[sidx]) : 0.f;
      }
    }
  }
  __syncthreads();
  bool ok = zb::mbar_wait_bounded(bar, 0, p.status, zb::kStatusPrefillTimeout);
  tc_fence_after();
  // ---- A (rows 0-63) into the fp32 workspace; P hi / lo (rows 64-127) into the record (over the dead KQ tile)
  {
    uint32_t r0[32], r1[32];
    const uint32_t tl = tmem + ((uint32_t)(32 * warp) << 16);
    tmem_ld32_nowait(tl, r0);
    tmem_ld32_nowait(tl + 32, r1);
    tmem_ld_wait();
    const int t = tid & (C - 1);
    if (sm.fast)
      decay_epilogue<true>(tid < C, t, r0, r1, G, bet, sm.rf, sm.cf, p.scale, Tf, base);
    else
      decay_epilogue<false>(tid < C, t, r0, r1, G, bet, sm.rf, sm.cf, p.scale, Tf, base);
  }
  __syncthreads();

  // ---- T = (I + A)^{-1}. Diagonal 16 x 16 blocks by forward substitution (thread = block b, column j)
  if (tid < 64) {
    const int b = tid >> 4, j = tid & 15;
    float x[16];
#pragma unroll
    for (int r = 0; r < 16; ++r) x[r] = r == j ? 1.f : 0.f;
#pragma unroll
    for (int r = 0; r < 16; ++r)
#pragma unroll
      for (int r2 = r + 1; r2 < 16; ++r2) x[r2] -= Tf[(16 * b + r2) * LC + 16 * b + r] * x[r];
#pragma unroll
    for (int r = 0; r < 16; ++r) Tf[(16 * b + r) * LC + 16 * b + j] = x[r];
  }
  __syncthreads();
  // ---- off-diagonal blocks row-block by row-block: for i = 1..3 and every j < i, Y_ij = sum_{k=j}^{i-1} A_ik T_kj,
  // then T_ij = -T_ii Y_ij, written over A_ij (row-block i of A is not read again). Work unit: 4 columns of one row
  // of one block (a strip); all 128 threads share each step.
  for (int i = 1; i < 4; ++i) {
    for (int st = tid; st < 64 * i; st += kPrepThreads) {
      const int j = st >> 6, r = (st >> 2) & 15, cq = st & 3;
      const float* arow = Tf + (16 * i + r) * LC;
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int k = j; k < i; ++k) {
#pragma unroll
        for (int m = 0; m < 16; ++m) {
          const float a = arow[16 * k + m];
          const float4 tv = *reinterpret_cast<const float4*>(Tf + (16 * k + m) * LC + 16 * j + 4 * cq);
          acc.x = fmaf(a, tv.x, acc.x);
          acc.y = fmaf(a, tv.y, acc.y);
          acc.z = fmaf(a, tv.z, acc.z);
          acc.w = fmaf(a, tv.w, acc.w);
        }
      }
      *reinterpret_cast<float4*>(Ys + j * 256 + r * 16 + 4 * cq) = acc;
    }
    __syncthreads();
    for (int st = tid; st < 64 * i; st += kPrepThreads) {
      const int j = st >> 6, r = (st >> 2) & 15, cq = st & 3;
      const float* trow = Tf + (16 * i + r) * LC + 16 * i;
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int m = 0; m < 16; ++m) {
        const float tv = trow[m];
        const float4 y = *reinterpret_cast<const float4*>(Ys + j * 256 + m * 16 + 4 * cq);
        acc.x = fmaf(tv, y.x, acc.x);
        acc.y = fmaf(tv, y.y, acc.y);
        acc.z = fmaf(tv, y.z, acc.z);
        acc.w = fmaf(tv, y.w, acc.w);
      }
      *reinterpret_cast<float4*>(Tf + (16 * i + r) * LC + 16 * j + 4 * cq) =
          make_float4(-acc.x, -acc.y, -acc.z, -acc.w);
    }
    __syncthreads();
  }
  // ---- T hi / lo into the record: Tf below and on the diagonal blocks, zero above them (8 columns per store)
  for (int e = tid; e < C * 8; e += kPrepThreads) {
    const int t = e >> 3, ch = e & 7;
    const bool zero = (ch >> 1) > (t >> 4);
    uint32_t hv[4], lv[4];
#pragma unroll
    for (int u = 0; u < 8; u += 2) {
      const float v0 = zero ? 0.f : Tf[t * LC + 8 * ch + u];
      const float v1 = zero ? 0.f : Tf[t * LC + 8 * ch + u + 1];
      split_pair(v0, v1, hv[u / 2], lv[u / 2]);
    }
    *reinterpret_cast<uint4*>(base + kRecTh + sw128_chunk(t, ch)) = make_uint4(hv[0], hv[1], hv[2], hv[3]);
    *reinterpret_cast<uint4*>(base + kRecTl + sw128_chunk(t, ch)) = make_uint4(lv[0], lv[1], lv[2], lv[3]);
  }
  fence_proxy_async();  // record staging (generic writes) -> bulk copy
  tc_fence_before();
  __syncthreads();
  if (tid == 0 && ok) {
    bulk_s2g(p.records + ((int64_t)id * p.H + h) * kRecBytes, sbase, kRecBytes);
    bulk_wait_all();
  }
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 64);
  }
}

__global__ void __launch_bounds__(kThreads, 1) gdn_prefill_state_kernel(StateParams p) {
  zb::pdl_enter();
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  const uint32_t raw_addr = zb::smem_addr(smem_raw);
  const uint32_t pad = (1024 - (raw_addr & 1023)) & 1023;
  unsigned char* base = smem_raw + pad;
  const uint32_t sbase = raw_addr + pad;
  Small& sm = *reinterpret_cast<Small*>(base + kOffSmall);

  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  const bool epi = tid < kEpiThreads;               // warps 0-7
  const bool mma_thread = warp == kEpiThreads / 32 && lane == 0;
  const int quarter = warp & 3;             // TMEM lane quarter of this warp
  const int half = (warp >> 2) & 1;         // warps 0-3 and 4-7 split columns
  const int row = 32 * quarter + lane;      // this thread's TMEM lane (value index)
  const uint32_t lane_off = (uint32_t)(32 * quarter) << 16;
  const int seq = blockIdx.x, h = blockIdx.y;
  const int64_t t_begin = p.cu_seqlens[seq], t_end = p.cu_seqlens[seq + 1];
  const int64_t len = t_end - t_begin;
  const int nchunks = (int)((len + C - 1) / C);
  const int64_t row_stride = (int64_t)p.H * D;
  const int64_t slot = p.state_slots ? p.state_slots[seq] : seq;
  const int64_t id0 = t_begin / C + seq;  // record id of chunk 0
  const uint32_t bar_m2 = zb::smem_addr(&sm.bar_m2), bar_m3 = zb::smem_addr(&sm.bar_m3);
  const uint32_t bar_m4 = zb::smem_addr(&sm.bar_m4), bar_m4o = zb::smem_addr(&sm.bar_m4o);

  if (tid == 0) {
    zb::mbar_init(zb::smem_addr(&sm.bar_rec[0]), 1);
    zb::mbar_init(zb::smem_addr(&sm.bar_rec[1]), 1);
    zb::mbar_init(bar_m2, 1);
    zb::mbar_init(bar_m3, 1);
    zb::mbar_init(bar_m4, 1);
    zb::mbar_init(bar_m4o, 1);
    sm.abort = 0;
    zb::fence_mbar_init();
  }
  if (warp == 0) tmem_alloc(zb::smem_addr(&sm.tmem_base), 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;
  const uint32_t tl = tmem + lane_off;  // this warp's lane quarter

  // ---- loads: K / Q rows of chunk c into KQ[c & 1] (cp.async, one group) with its prep record (one bulk copy);
  // V rows into the single V buffer (cp.async, its own group)
  int last_issued = -1;  // thread 0: chunk of the last record copy
  auto load_kqrec = [&](int c) {
    const int b = c & 1;
    if (tid >= kEpiThreads) return;
    load_kq(sbase + kOffKQ + b * kKQBytes, p.k, p.q, t_begin, len, c, row_stride, h, tid, kEpiThreads);
    cp_async_commit();
    if (tid == 0) {
      last_issued = c;
      const uint32_t bar = zb::smem_addr(&sm.bar_rec[b]);
      zb::mbar_arrive_expect_tx(bar, kRecBytes);
      zb::bulk_g2s(sbase + kOffRec + b * kRecSlot, p.records + ((id0 + c) * p.H + h) * kRecBytes, kRecBytes, bar);
    }
  };
  auto load_v = [&](int c) {
    if (tid >= kEpiThreads) return;
    for (int i = tid; i < C * 16; i += kEpiThreads) {
      const int t = i >> 4, cidx = i & 15;
      const int64_t tok = (int64_t)c * C + t;
      const bool ok = tok < len;
      cp_async16(sbase + kOffV + t * 256 + cidx * 16,
                 p.v + (t_begin + (ok ? tok : 0)) * row_stride + (int64_t)h * D + cidx * 8, ok);
    }
    cp_async_commit();
  };
  auto wait_bar = [&](uint32_t bar, uint32_t parity) {
    if (!zb::mbar_wait_bounded(bar, parity, p.status, zb::kStatusPrefillTimeout)) sm.abort = 1;
  };
  auto wait_rec = [&](int c) { wait_bar(zb::smem_addr(&sm.bar_rec[c & 1]), (uint32_t)((c >> 1) & 1)); };
  auto rec_vec = [&](int c, uint32_t off) {
    return reinterpret_cast<const float*>(base + kOffRec + (c & 1) * kRecSlot + off);
  };
  // M2 of chunk c: (K S0)^T, (Q S0)^T
  auto issue_m2 = [&](int c) {
    if (!mma_thread) return;
    const uint32_t kq = sbase + kOffKQ + (c & 1) * kKQBytes;
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      const uint32_t off = (ks >> 2) * (128 * 128) + (ks & 3) * 32;
      mma_ts(tmem + kColKS, tmem + kColSh + 8 * ks, desc_sw128(kq + off), idesc_m128(128), ks > 0);
    }
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      const uint32_t off = (ks >> 2) * (128 * 128) + (ks & 3) * 32;
      mma_ts(tmem + kColKS, tmem + kColSl + 8 * ks, desc_sw128(kq + off), idesc_m128(128), 1);
    }
    mma_commit(bar_m2);
  };
  // (fK)^T hi / lo of chunk c into FKT[c & 1] from the K rows of KQ[c & 1]: ldmatrix.trans gives each lane the
  // (t, t+1) pair of one key, stmatrix writes the [dk][t] tiles; per warp item: t-block tb (8 rows) x 32 keys
  auto build_fkt = [&](int c) {
    const uint32_t kqa = sbase + kOffKQ + (c & 1) * kKQBytes;
    const uint32_t fh = sbase + kOffFKT + (c & 1) * 2 * kFKTBytes, fl = fh + kFKTBytes;
    const float* ef = rec_vec(c, kRecEf);
    const int mi = lane >> 3, r8 = lane & 7;
#pragma unroll
    for (int it = warp; it < 32; it += kEpiThreads / 32) {
      const int tb = it & 7, dk0 = 32 * (it >> 3);
      const int dkb = dk0 + 8 * mi;
      uint32_t kv[4];
      ldsm_x4_trans(kqa + (dkb >> 6) * (128 * 128) + sw128_chunk(8 * tb + r8, (dkb & 63) >> 3), kv);
      const int t = 8 * tb + 2 * (lane & 3);
      const float f0 = ef[t], f1 = ef[t + 1];
      uint32_t hv[4], lv[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 kf = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&kv[j]));
        split_pair(f0 * kf.x, f1 * kf.y, hv[j], lv[j]);
      }
      const uint32_t drow = sw128_chunk(dk0 + 8 * mi + r8, tb);
      stsm_x4(fh + drow, hv);
      stsm_x4(fl + drow, lv);
    }
    fence_proxy_async();  // (fK)^T tiles -> tensor-core reads
  };

  // output rows of chunk c from their staging tile (over (fK)^T hi of buffer c & 1): 16 threads per 256-byte row
  auto write_rows = [&](int c) {
    if (!epi) return;
    const unsigned char* ostage = base + kOffFKT + (c & 1) * 2 * kFKTBytes;
    for (int e = tid; e < C * 16; e += kEpiThreads) {
      const int t = e >> 4, ch = e & 15;
      if ((int64_t)c * C + t < len)
        *reinterpret_cast<uint4*>(p.out + (t_begin + (int64_t)c * C + t) * row_stride + (int64_t)h * D + ch * 8) =
            *reinterpret_cast<const uint4*>(ostage + t * 256 + ch * 16);
    }
  };

  // ---- prologue: chunk 0's loads; S^T hi / lo = split(S0) for M2, master = gamma_C S0 (the decay of chunk 0
  // applied ahead of M4); (fK)^T of chunk 0; M2 of chunk 0; chunk 1's K / Q and record
  if (epi) {
    if (nchunks > 0) {
      load_kqrec(0);
      load_v(0);
      cp_async_wait_all();
      wait_rec(0);
      fence_proxy_async();
    }
    const float gamC = nchunks > 0 ? rec_vec(0, kRecGam)[C - 1] : 1.f;
#pragma unroll
    for (int part = 0; part < 2; ++part) {
      const int k0 = 64 * half + 32 * part;
      uint32_t m[32];
#pragma unroll
      for (int j = 0; j < 32; j += 4) {
        float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
        if (p.init_state)
          s = *reinterpret_cast<const float4*>(p.init_state + ((slot * p.H + h) * D + row) * (int64_t)D + k0 + j);
        m[j] = __float_as_uint(s.x);
        m[j + 1] = __float_as_uint(s.y);
        m[j + 2] = __float_as_uint(s.z);
        m[j + 3] = __float_as_uint(s.w);
      }
      uint32_t hi[16], lo[16];
#pragma unroll
      for (int j = 0; j < 32; j += 2) split_pair(__uint_as_float(m[j]), __uint_as_float(m[j + 1]), hi[j / 2], lo[j / 2]);
      tmem_st16(tl + kColSh + 32 * half + 16 * part, hi);
      tmem_st16(tl + kColSl + 32 * half + 16 * part, lo);
#pragma unroll
      for (int j = 0; j < 32; ++j) m[j] = __float_as_uint(__uint_as_float(m[j]) * gamC);
      tmem_st32(tl + kColMaster + k0, m);
    }
    if (nchunks > 0) build_fkt(0);
    tmem_st_wait();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (nchunks > 0 && !sm.abort) {
    issue_m2(0);
    if (nchunks > 1) load_kqrec(1);
  }

  // ---- chunks. Per chunk c the tensor-core chain is M2 -> M3 -> M4 -> M2(c + 1), issued by warp 8; warps 0-7 do
  // the Y, U and state-split steps between them, build (fK)^T of chunk c + 1 during M4 and write chunk c's output
  // rows during M2(c + 1). Every __syncthreads below is reached by all nine warps.
  for (int c = 0; c < nchunks; ++c) {
    if (sm.abort) break;
    const int b = c & 1;
    const bool has_next = c + 1 < nchunks;
    const uint32_t ph = (uint32_t)(c & 1);
    const uint32_t rec = sbase + kOffRec + b * kRecSlot;
    const float* gam = rec_vec(c, kRecGam);
    const float* bet = rec_vec(c, kRecBet);
    const __nv_bfloat16* Vs = reinterpret_cast<const __nv_bfloat16*>(base + kOffV);

    // ---- after M2: Y^T hi / lo into TMEM and O^T *= scale gamma_t; warps 0-3 columns t 0..31, warps 4-7 t 32..63
    if (epi) {
      wait_bar(bar_m2, ph);
      tc_fence_after();
      const int t0 = 32 * half;
      uint32_t r[32];
      tmem_ld32_nowait(tl + kColKS + t0, r);
      tmem_ld_wait();
      uint32_t hv[16], lv[16];
#pragma unroll
      for (int j = 0; j < 32; j += 2) {
        const int t = t0 + j;
        const float y0 = bet[t] * (__bfloat162float(Vs[t * D + row]) - gam[t] * __uint_as_float(r[j]));
        const float y1 =
            bet[t + 1] * (__bfloat162float(Vs[(t + 1) * D + row]) - gam[t + 1] * __uint_as_float(r[j + 1]));
        split_pair(y0, y1, hv[j / 2], lv[j / 2]);
      }
      tmem_st16(tl + kColYh + 16 * half, hv);
      tmem_st16(tl + kColYl + 16 * half, lv);
      tmem_ld32_nowait(tl + kColQS + t0, r);
      tmem_ld_wait();
#pragma unroll
      for (int j = 0; j < 32; ++j) r[j] = __float_as_uint(__uint_as_float(r[j]) * (p.scale * gam[t0 + j]));
      tmem_st32(tl + kColQS + t0, r);
      tmem_st_wait();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (sm.abort) break;

    // ---- M3: U^T = Y^T T^T; the V buffer is free again: the next chunk's V loads meanwhile
    if (mma_thread) {
      const uint32_t th = rec + kRecTh, tlo = rec + kRecTl;
#pragma unroll
      for (int ks = 0; ks < 4; ++ks)
        mma_ts(tmem + kColU, tmem + kColYh + 8 * ks, desc_sw128(th + 32 * ks), idesc_m128(64), ks > 0);
#pragma unroll
      for (int ks = 0; ks < 4; ++ks)
        mma_ts(tmem + kColU, tmem + kColYh + 8 * ks, desc_sw128(tlo + 32 * ks), idesc_m128(64), 1);
#pragma unroll
      for (int ks = 0; ks < 4; ++ks)
        mma_ts(tmem + kColU, tmem + kColYl + 8 * ks, desc_sw128(th + 32 * ks), idesc_m128(64), 1);
      mma_commit(bar_m3);
    }
    if (epi) {
      if (has_next) load_v(c + 1);
      wait_bar(bar_m3, ph);
      tc_fence_after();
      // U^T hi / lo into TMEM (over Y^T): warps 0-3 columns t 0..31, warps 4-7 t 32..63
      uint32_t r[32];
      tmem_ld32_nowait(tl + kColU + 32 * half, r);
      tmem_ld_wait();
      uint32_t hv[16], lv[16];
#pragma unroll
      for (int j = 0; j < 32; j += 2) split_pair(__uint_as_float(r[j]), __uint_as_float(r[j + 1]), hv[j / 2], lv[j / 2]);
      tmem_st16(tl + kColYh + 16 * half, hv);
      tmem_st16(tl + kColYl + 16 * half, lv);
      tmem_st_wait();
      if (has_next) {  // chunk c + 1's K / Q (all groups but the newest, its V) and record
        asm volatile("cp.async.wait_group 1;" ::: "memory");
        wait_rec(c + 1);
        fence_proxy_async();
      }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (sm.abort) break;

    // ---- M4: S^T += U^T (fK) (committed first: the state split starts while the rest runs);  O^T += U^T P^T
    if (mma_thread) {
      const uint32_t fh = sbase + kOffFKT + b * 2 * kFKTBytes, fl = fh + kFKTBytes;
      const uint32_t pph = rec + kRecPh, ppl = rec + kRecPl;
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {
        mma_ts(tmem + kColMaster, tmem + kColYh + 8 * ks, desc_sw128(fh + 32 * ks), idesc_m128(128), 1);
        mma_ts(tmem + kColMaster, tmem + kColYh + 8 * ks, desc_sw128(fl + 32 * ks), idesc_m128(128), 1);
        mma_ts(tmem + kColMaster, tmem + kColYl + 8 * ks, desc_sw128(fh + 32 * ks), idesc_m128(128), 1);
      }
      mma_commit(bar_m4);
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {
        mma_ts(tmem + kColQS, tmem + kColYh + 8 * ks, desc_sw128(pph + 32 * ks), idesc_m128(64), 1);
        mma_ts(tmem + kColQS, tmem + kColYh + 8 * ks, desc_sw128(ppl + 32 * ks), idesc_m128(64), 1);
        mma_ts(tmem + kColQS, tmem + kColYl + 8 * ks, desc_sw128(pph + 32 * ks), idesc_m128(64), 1);
      }
      mma_commit(bar_m4o);
    }
    // ---- S^T master -> hi / lo for M2 of the next chunk and master *= its gamma_C (warps 0-3 keys 0..63, warps
    // 4-7 keys 64..127); O^T into registers (M2 of the next chunk overwrites its columns)
    uint32_t o[32];
    if (epi) {
      if (has_next) build_fkt(c + 1);
      wait_bar(bar_m4, ph);
      tc_fence_after();
      const float gamC = has_next ? rec_vec(c + 1, kRecGam)[C - 1] : 1.f;
#pragma unroll
      for (int part = 0; part < 2; ++part) {
        const uint32_t col = 64 * half + 32 * part;
        uint32_t m[32];
        tmem_ld32_nowait(tl + kColMaster + col, m);
        tmem_ld_wait();
        uint32_t hv[16], lv[16];
#pragma unroll
        for (int j = 0; j < 32; j += 2) split_pair(__uint_as_float(m[j]), __uint_as_float(m[j + 1]), hv[j / 2], lv[j / 2]);
        tmem_st16(tl + kColSh + 32 * half + 16 * part, hv);
        tmem_st16(tl + kColSl + 32 * half + 16 * part, lv);
        if (has_next) {
#pragma unroll
          for (int j = 0; j < 32; ++j) m[j] = __float_as_uint(__uint_as_float(m[j]) * gamC);
          tmem_st32(tl + kColMaster + col, m);
        }
      }
      wait_bar(bar_m4o, ph);
      tc_fence_after();
      tmem_ld32_nowait(tl + kColQS + 32 * half, o);
      tmem_ld_wait();
      tmem_st_wait();
      if (has_next) cp_async_wait_all();  // chunk c + 1's V (read by its Y step)
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (has_next && !sm.abort) {
      issue_m2(c + 1);
      if (c + 2 < nchunks) load_kqrec(c + 2);  // chunk c's KQ and record buffers are free: M4 has completed
    }
    // ---- O^T -> bf16 rows [t][v] staged over chunk c's (fK)^T hi tile (M4 has completed; the tile is next written
    // for chunk c + 2, during M4 of chunk c + 1), then written out as 256-byte rows while M2 of the next chunk runs
    if (epi) {
      __nv_bfloat16* os = reinterpret_cast<__nv_bfloat16*>(base + kOffFKT + b * 2 * kFKTBytes);
#pragma unroll
      for (int j = 0; j < 32; ++j) os[(32 * half + j) * D + row] = __float2bfloat16_rn(__uint_as_float(o[j]));
    }
    __syncthreads();
    write_rows(c);
  }

  if (p.final_state && !sm.abort && epi) {
    float* dst = p.final_state + ((slot * p.H + h) * D + row) * (int64_t)D + 64 * half;
#pragma unroll
    for (int part = 0; part < 2; ++part) {
      uint32_t m[32];
      tmem_ld32_nowait(tl + kColMaster + 64 * half + 32 * part, m);
      tmem_ld_wait();
#pragma unroll
      for (int j = 0; j < 32; j += 4)
        *reinterpret_cast<float4*>(dst + 32 * part + j) = make_float4(
            __uint_as_float(m[j]), __uint_as_float(m[j + 1]), __uint_as_float(m[j + 2]), __uint_as_float(m[j + 3]));
    }
  }
  cp_async_wait_all();
  // after an abort, the last record copy issued may still be in flight: it must land before the CTA's shared
  // memory is released
  if (tid == 0 && sm.abort && last_issued >= 0)
    zb::mbar_wait_bounded(zb::smem_addr(&sm.bar_rec[last_issued & 1]), (uint32_t)((last_issued >> 1) & 1), nullptr,
                          0);
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace

namespace zb {

int64_t gdn_prefill_tc_workspace_bytes(int64_t total_tokens, int num_seqs, int H) {
  return ((total_tokens + C - 1) / C + num_seqs) * (int64_t)H * kRecBytes;
}

// d_k = d_v = 128 chunked prefill on tcgen05 (called by zb_gdn_chunk_prefill after its argument checks).
int gdn_prefill_tc_launch(const uint16_t* q, const uint16_t* k, const uint16_t* v, const float* g, const float* beta,
                          const int32_t* cu_seqlens, int num_seqs, int H, float scale, const float* init_state,
                          const int64_t* state_slots, float* final_state, uint16_t* out, int64_t total_tokens,
                          void* workspace, int64_t workspace_bytes, cudaStream_t stream) {
  if (init_state) ZB_REQUIRE_ALIGNED(init_state, 16, "gdn_chunk_prefill init_state");
  if (final_state) ZB_REQUIRE_ALIGNED(final_state, 16, "gdn_chunk_prefill final_state");
  const int64_t need = gdn_prefill_tc_workspace_bytes(total_tokens, num_seqs, H);
  ZB_REQUIRE(workspace != nullptr && workspace_bytes >= need,
             "gdn_chunk_prefill: workspace of %lld bytes needed (got %lld)", (long long)need,
             (long long)workspace_bytes);
  ZB_REQUIRE_ALIGNED(workspace, 16, "gdn_chunk_prefill workspace");
  const int64_t ids = (total_tokens + C - 1) / C + num_seqs;
  ZB_REQUIRE(ids <= 0x7fffffff, "gdn_chunk_prefill: too many chunks");
  unsigned* status = device_status_ptr();
  if (ids > 0) {
    PrepParams pp{reinterpret_cast<const __nv_bfloat16*>(q), reinterpret_cast<const __nv_bfloat16*>(k), g, beta,
                  cu_seqlens, num_seqs, H, scale, static_cast<unsigned char*>(workspace), status};
    ZB_CUDA(cudaFuncSetAttribute(gdn_prefill_prep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)kPrepSmem));
    ZB_CUDA(zb::launch(gdn_prefill_prep_kernel, dim3(dim3((unsigned)ids, (unsigned)H)), dim3(kPrepThreads), kPrepSmem, stream, 1, pp));
    if (int rc = check_launch("gdn_chunk_prefill (prep)")) return rc;
  }
  StateParams sp{reinterpret_cast<const __nv_bfloat16*>(q), reinterpret_cast<const __nv_bfloat16*>(k),
                 reinterpret_cast<const __nv_bfloat16*>(v), cu_seqlens, init_state, state_slots, final_state,
                 reinterpret_cast<__nv_bfloat16*>(out), static_cast<const unsigned char*>(workspace), H, scale, status};
  ZB_CUDA(cudaFuncSetAttribute(gdn_prefill_state_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               (int)kSmemBytes));
  ZB_CUDA(zb::launch(gdn_prefill_state_kernel, dim3(dim3((unsigned)num_seqs, (unsigned)H)), dim3(kThreads), kSmemBytes, stream, 1, sp));
  return check_launch("gdn_chunk_prefill (state)");
}

}  // namespace zb

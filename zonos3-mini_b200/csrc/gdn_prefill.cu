// Gated-DeltaNet chunked prefill (WY / UT form), chunk C = 64, varlen sequences, fp32 state.
//
// Reference: FLA chunk_gated_delta_rule_fwd as called by OriginalGDN._run_packed
// (servers/sgl/src/zonos3_sgl/models/gdn.py:418-434: use_gate_in_kernel, scale, initial_state, output_final_state,
// state_v_first, cu_seqlens, chunk_size=64), whose result must equal the per-token recurrence of
// model/src/zonos3/reference/lm.py:576-582. Derivation used here (state S = M^T, dk x dv, M the reference's V-first
// state): with u_t = beta_t (v_t - d_t S_{t-1}^T k_t) the recurrence is S_t = d_t S_{t-1} + k_t u_t^T. Inside a
// chunk starting from S_0, with G_t = sum_{s<=t} g_s and gamma_t = exp(G_t):
//   (I + A) U = diag(beta) (V - diag(gamma) K S_0),   A_ts = beta_t exp(G_t - G_s) k_t.k_s  (s < t)
//   O = diag(gamma) Q S_0 + P U,                      P_ts = scale exp(G_t - G_s) q_t.k_s   (s <= t)
//   S_C = gamma_C S_0 + K^T diag(exp(G_C - G_t)) U
// This file holds the d_k = d_v = 64 kernel and the entry point; d = 128 runs on tcgen05 (gdn_prefill_tc.cu).
// One CTA owns one (sequence, head) and walks its chunks in order with the fp32 state resident in shared memory.
// Per chunk: K K^T and Q K^T on tensor cores (mma.sync m16n8k16, bf16 inputs exact); T = (I + A)^{-1} by blocked
// 16x16 forward substitution in fp32; K S_0, Q S_0, T Y, P U and K^T U on tensor cores with every fp32 operand
// split into bf16 hi + lo (products hi*hi + hi*lo + lo*hi), which keeps the state path near fp32 accuracy.
// Padded rows of a ragged last chunk load as q = k = v = 0, g = 0, beta = 0 and change nothing.
#include "common.cuh"

namespace {

constexpr int C = 64;           // chunk length
constexpr int kThreads = 256;   // 8 warps

struct PrefillParams {
  const __nv_bfloat16* q;  // [N, H, D]
  const __nv_bfloat16* k;  // [N, H, D]
  const __nv_bfloat16* v;  // [N, H, D]
  const float* g;          // [N, H] log decay
  const float* beta;       // [N, H]
  const int32_t* cu_seqlens;  // [num_seqs + 1]
  const float* init_state;    // [num_seqs, H, D(v), D(k)] or null (zeros)
  const int64_t* state_slots; // optional: sequence i uses state row slots[i] of init/final
  float* final_state;         // [num_seqs, H, D(v), D(k)] or null
  __nv_bfloat16* out;         // [N, H, D]
  int H;
  float scale;
};

__device__ __forceinline__ void mma16816(float c[4], const uint32_t a[4], const uint32_t b[2]) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

__device__ __forceinline__ uint32_t pack2(__nv_bfloat16 lo, __nv_bfloat16 hi) {
  return (uint32_t)__bfloat16_as_ushort(lo) | ((uint32_t)__bfloat16_as_ushort(hi) << 16);
}

// x = hi + lo with hi = bf16(x), lo = bf16(x - hi); packs the pair (x0, x1) into a hi word and a lo word.
__device__ __forceinline__ void split2(float x0, float x1, uint32_t& hi, uint32_t& lo) {
  const __nv_bfloat16 h0 = __float2bfloat16_rn(x0), h1 = __float2bfloat16_rn(x1);
  hi = pack2(h0, h1);
  lo = pack2(__float2bfloat16_rn(x0 - __bfloat162float(h0)), __float2bfloat16_rn(x1 - __bfloat162float(h1)));
}

__device__ __forceinline__ void cp_async16(void* dst, const void* src, bool valid) {
  const uint32_t d = zb::smem_addr(dst);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(d), "l"(src), "r"(valid ? 16 : 0) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

template <int D>
struct Smem {
  static constexpr int LB = D + 8;   // bf16 row length (elements): conflict-free fragment loads
  static constexpr int LC = C + 4;   // fp32 row length of [C, C] arrays
  __nv_bfloat16 q[C * LB];
  __nv_bfloat16 kb[2][C * LB];       // K, double-buffered across chunks
  __nv_bfloat16 v[C * LB];
  static constexpr int LY = C + 8;   // bf16 row length of [value][t] arrays
  // state S (K-first, S[key][value]) kept transposed and split, S^T[value][key] = Sh + Sl (bf16 hi + lo): the
  // mma B fragments of K S0 and Q S0 load as 32-bit words, each element split once per chunk
  __nv_bfloat16 Sh[D * LB];
  __nv_bfloat16 Sl[D * LB];
  float T[C * LC];                   // A, then T = (I + A)^{-1}
  float P[C * LC];
  // Y = diag(beta)(V - diag(gamma) K S0), then U, transposed and split: Y^T[value][t] = Yh + Yl
  // (fp32 scratch of the inverse before that)
  __nv_bfloat16 Yh[D * LY];
  __nv_bfloat16 Yl[D * LY];
  float G[C];                        // cumulative log decay inside the chunk
  float gam[C];                      // exp(G)
  float bet[C];
  float graw[2][C];                  // g of the chunk (double-buffered with K)
  float braw[2][C];
};

template <int D>
__global__ void __launch_bounds__(kThreads, 1) gdn_chunk_prefill_kernel(PrefillParams p) {
  zb::pdl_enter();
  using SM = Smem<D>;
  constexpr int LB = SM::LB, LC = SM::LC, LY = SM::LY;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  SM& sm = *reinterpret_cast<SM*>(smem_raw);
  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  const int g8 = lane >> 2, tq = lane & 3;
  const int seq = blockIdx.x, h = blockIdx.y;
  const int64_t t_begin = p.cu_seqlens[seq], t_end = p.cu_seqlens[seq + 1];
  const int64_t len = t_end - t_begin;
  const int nchunks = (int)((len + C - 1) / C);
  const int64_t row_stride = (int64_t)p.H * D;  // elements between tokens of q / k / v / out
  const int64_t slot = p.state_slots ? p.state_slots[seq] : seq;

  // ---- initial state (transposed into S[key][value])
  for (int i = tid; i < D * D; i += kThreads) {
    const int vi = i / D, ki = i % D;
    float s = 0.f;
    if (p.init_state) s = p.init_state[((slot * p.H + h) * D + vi) * (int64_t)D + ki];
    const __nv_bfloat16 hi = __float2bfloat16_rn(s);
    sm.Sh[vi * LB + ki] = hi;
    sm.Sl[vi * LB + ki] = __float2bfloat16_rn(s - __bfloat162float(hi));
  }

  auto load_rows = [&](__nv_bfloat16* dst, const __nv_bfloat16* src, int c) {
    constexpr int kVec = D / 8;
    for (int i = tid; i < C * kVec; i += kThreads) {
      const int r = i / kVec, cc = (i % kVec) * 8;
      const int64_t tok = (int64_t)c * C + r;
      const bool ok = tok < len;
      cp_async16(dst + r * LB + cc, src + (t_begin + (ok ? tok : 0)) * row_stride + (int64_t)h * D + cc, ok);
    }
  };
  auto load_gb = [&](int buf, int c) {
    for (int r = tid; r < C; r += kThreads) {
      const int64_t tok = (int64_t)c * C + r;
      const bool ok = tok < len;
      sm.graw[buf][r] = ok ? p.g[(t_begin + tok) * p.H + h] : 0.f;
      sm.braw[buf][r] = ok ? p.beta[(t_begin + tok) * p.H + h] : 0.f;
    }
  };

  if (nchunks > 0) {
    load_rows(sm.q, p.q, 0);
    load_rows(sm.kb[0], p.k, 0);
    load_rows(sm.v, p.v, 0);
    load_gb(0, 0);
    cp_async_commit();
  }

  for (int c = 0; c < nchunks; ++c) {
    const int kbuf = c & 1;
    const __nv_bfloat16* K = sm.kb[kbuf];
    cp_async_wait_all();
    __syncthreads();
    // prefetch the next chunk's K, g, beta into the other buffers (Q and V follow after step 3)
    if (c + 1 < nchunks) {
      load_rows(sm.kb[kbuf ^ 1], p.k, c + 1);
      load_gb(kbuf ^ 1, c + 1);
      cp_async_commit();
    }
    // ---- step 0: cumulative log decay, gamma, beta
    if (warp == 0) {
      const float a0 = sm.graw[kbuf][2 * lane], a1 = sm.graw[kbuf][2 * lane + 1];
      float incl = a0 + a1;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const float o = __shfl_up_sync(0xffffffffu, incl, off);
        if (lane >= off) incl += o;
      }
      const float g0 = incl - a1, g1 = incl;
      sm.G[2 * lane] = g0;
      sm.G[2 * lane + 1] = g1;
      sm.gam[2 * lane] = expf(g0);
      sm.gam[2 * lane + 1] = expf(g1);
      sm.bet[2 * lane] = sm.braw[kbuf][2 * lane];
      sm.bet[2 * lane + 1] = sm.braw[kbuf][2 * lane + 1];
    }
    __syncthreads();

    // ---- step 1: A = strict-lower(beta_t e^{G_t - G_s} K K^T), P = lower(scale e^{G_t - G_s} Q K^T)
    {
      const int mt = warp & 3, nh = warp >> 2;
      float accK[4][4] = {}, accQ[4][4] = {};
#pragma unroll
      for (int k0 = 0; k0 < D; k0 += 16) {
        uint32_t aK[4], aQ[4];
        const int r0 = 16 * mt + g8;
        aK[0] = *reinterpret_cast<const uint32_t*>(K + r0 * LB + k0 + 2 * tq);
        aK[1] = *reinterpret_cast<const uint32_t*>(K + (r0 + 8) * LB + k0 + 2 * tq);
        aK[2] = *reinterpret_cast<const uint32_t*>(K + r0 * LB + k0 + 2 * tq + 8);
        aK[3] = *reinterpret_cast<const uint32_t*>(K + (r0 + 8) * LB + k0 + 2 * tq + 8);
        aQ[0] = *reinterpret_cast<const uint32_t*>(sm.q + r0 * LB + k0 + 2 * tq);
        aQ[1] = *reinterpret_cast<const uint32_t*>(sm.q + (r0 + 8) * LB + k0 + 2 * tq);
        aQ[2] = *reinterpret_cast<const uint32_t*>(sm.q + r0 * LB + k0 + 2 * tq + 8);
        aQ[3] = *reinterpret_cast<const uint32_t*>(sm.q + (r0 + 8) * LB + k0 + 2 * tq + 8);
#pragma unroll
        for (int n = 0; n < 4; ++n) {
          const int s0 = 32 * nh + 8 * n + g8;  // B[kk][n] = K[s][k0 + kk]
          uint32_t b[2];
          b[0] = *reinterpret_cast<const uint32_t*>(K + s0 * LB + k0 + 2 * tq);
          b[1] = *reinterpret_cast<const uint32_t*>(K + s0 * LB + k0 + 2 * tq + 8);
          mma16816(accK[n], aK, b);
          mma16816(accQ[n], aQ, b);
        }
      }
#pragma unroll
      for (int n = 0; n < 4; ++n) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int t = 16 * mt + g8 + (e >= 2 ? 8 : 0);
          const int s = 32 * nh + 8 * n + 2 * tq + (e & 1);
          const float dec = s <= t ? expf(sm.G[t] - sm.G[s]) : 0.f;
          sm.T[t * LC + s] = s < t ? sm.bet[t] * dec * accK[n][e] : 0.f;
          sm.P[t * LC + s] = p.scale * dec * accQ[n][e];
        }
      }
    }
    __syncthreads();

    // ---- step 2: T = (I + A)^{-1}, blocked 16 x 16
    {
      // (a) diagonal blocks by forward substitution: thread (block b, column j)
      float x[16];
      const int b = tid / 16, j = tid % 16;
      if (tid < 64) {
#pragma unroll
        for (int r = 0; r < 16; ++r) {
          float acc = (r == j) ? 1.f : 0.f;
#pragma unroll
          for (int s = 0; s < r; ++s) acc -= sm.T[(16 * b + r) * LC + 16 * b + s] * x[s];
          x[r] = acc;
        }
      }
      __syncthreads();
      if (tid < 64) {
#pragma unroll
        for (int r = 0; r < 16; ++r) sm.T[(16 * b + r) * LC + 16 * b + j] = x[r];
      }
      __syncthreads();
      // (b) off-diagonal blocks: X_ij = -X_ii * sum_{k=j}^{i-1} A_ik X_kj, by distance i - j = 1, 2, 3.
      // Results park in Z (free here): block (i, j) at Z + blk(i, j) * 256, row-major 16 x 16; tmp after them.
      float* X = reinterpret_cast<float*>(sm.Yh);  // Y / U are not live during the inverse
      auto blk = [](int i, int jj) { return (i * (i - 1)) / 2 + jj; };  // (1,0)=0 (2,0)=1 (2,1)=2 (3,0)=3 ...
      float* tmp = X + 6 * 256;
      auto Xat = [&](int i, int jj, int r, int cc) -> float {
        return i == jj ? sm.T[(16 * i + r) * LC + 16 * jj + cc] : X[blk(i, jj) * 256 + r * 16 + cc];
      };
      for (int dist = 1; dist <= 3; ++dist) {
        const int nblk = 4 - dist;  // blocks (j + dist, j) for j = 0 .. nblk - 1
        for (int e = tid; e < nblk * 256; e += kThreads) {
          const int jj = e / 256, r = (e % 256) / 16, cc = e % 16;
          const int i = jj + dist;
          float acc = 0.f;
          for (int kk = jj; kk < i; ++kk)
#pragma unroll
            for (int m = 0; m < 16; ++m) acc += sm.T[(16 * i + r) * LC + 16 * kk + m] * Xat(kk, jj, m, cc);
          tmp[jj * 256 + r * 16 + cc] = acc;
        }
        __syncthreads();
        for (int e = tid; e < nblk * 256; e += kThreads) {
          const int jj = e / 256, r = (e % 256) / 16, cc = e % 16;
          const int i = jj + dist;
          float acc = 0.f;
#pragma unroll
          for (int m = 0; m < 16; ++m) acc -= sm.T[(16 * i + r) * LC + 16 * i + m] * tmp[jj * 256 + m * 16 + cc];
          X[blk(i, jj) * 256 + r * 16 + cc] = acc;
        }
        __syncthreads();
      }
      // A's off-diagonal blocks are no longer needed: replace them by T's
      for (int e = tid; e < 6 * 256; e += kThreads) {
        const int bi = e / 256, r = (e % 256) / 16, cc = e % 16;
        int i = 1, jj = bi;
        while (jj >= i) { jj -= i; ++i; }
        sm.T[(16 * i + r) * LC + 16 * jj + cc] = X[bi * 256 + r * 16 + cc];
      }
      __syncthreads();
    }

    // ---- step 3: Y = diag(beta)(V - diag(gamma) K S0) -> Z;  Oacc = diag(gamma) Q S0 (registers)
    constexpr int NW = D / 16;                // n8-tiles of a warp tile
    const int mt = warp & 3, nh = warp >> 2;  // warp tile: rows 16mt.., columns nh*D/2 .. (NW n8-tiles)
    const int cbase = nh * (D / 2);
    float oacc[NW][4] = {};
    {
      float accK[NW][4] = {};
#pragma unroll 2
      for (int k0 = 0; k0 < D; k0 += 16) {
        uint32_t aK[4], aQ[4];
        const int r0 = 16 * mt + g8;
        aK[0] = *reinterpret_cast<const uint32_t*>(K + r0 * LB + k0 + 2 * tq);
        aK[1] = *reinterpret_cast<const uint32_t*>(K + (r0 + 8) * LB + k0 + 2 * tq);
        aK[2] = *reinterpret_cast<const uint32_t*>(K + r0 * LB + k0 + 2 * tq + 8);
        aK[3] = *reinterpret_cast<const uint32_t*>(K + (r0 + 8) * LB + k0 + 2 * tq + 8);
        aQ[0] = *reinterpret_cast<const uint32_t*>(sm.q + r0 * LB + k0 + 2 * tq);
        aQ[1] = *reinterpret_cast<const uint32_t*>(sm.q + (r0 + 8) * LB + k0 + 2 * tq);
        aQ[2] = *reinterpret_cast<const uint32_t*>(sm.q + r0 * LB + k0 + 2 * tq + 8);
        aQ[3] = *reinterpret_cast<const uint32_t*>(sm.q + (r0 + 8) * LB + k0 + 2 * tq + 8);
#pragma unroll
        for (int n = 0; n < NW; ++n) {
          const int col = cbase + 8 * n + g8;  // B[kk][n] = S[k0 + kk][col] = S^T[col][k0 + kk]
          const __nv_bfloat16* sh = sm.Sh + col * LB + k0 + 2 * tq;
          const __nv_bfloat16* sl = sm.Sl + col * LB + k0 + 2 * tq;
          uint32_t bh[2], bl[2];
          bh[0] = *reinterpret_cast<const uint32_t*>(sh);
          bh[1] = *reinterpret_cast<const uint32_t*>(sh + 8);
          bl[0] = *reinterpret_cast<const uint32_t*>(sl);
          bl[1] = *reinterpret_cast<const uint32_t*>(sl + 8);
          mma16816(accK[n], aK, bh);
          mma16816(accK[n], aK, bl);
          mma16816(oacc[n], aQ, bh);
          mma16816(oacc[n], aQ, bl);
        }
      }
#pragma unroll
      for (int n = 0; n < NW; ++n) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int t = 16 * mt + g8 + (e >= 2 ? 8 : 0);
          const int col = cbase + 8 * n + 2 * tq + (e & 1);
          const float vv = __bfloat162float(sm.v[t * LB + col]);
          const float y = sm.bet[t] * (vv - sm.gam[t] * accK[n][e]);
          const __nv_bfloat16 hi = __float2bfloat16_rn(y);
          sm.Yh[col * LY + t] = hi;
          sm.Yl[col * LY + t] = __float2bfloat16_rn(y - __bfloat162float(hi));
          oacc[n][e] *= sm.gam[t] * p.scale;
        }
      }
    }
    __syncthreads();
    // Q and V of this chunk are consumed: prefetch the next chunk's
    if (c + 1 < nchunks) {
      load_rows(sm.q, p.q, c + 1);
      load_rows(sm.v, p.v, c + 1);
      cp_async_commit();
    }

    // ---- step 4: U = T Y (T lower triangular: k-blocks above the row block are zero)
    {
      float accU[NW][4] = {};
      for (int k0 = 0; k0 < 16 * (mt + 1); k0 += 16) {
        uint32_t ah[4], al[4];
        const int r0 = 16 * mt + g8;
        split2(sm.T[r0 * LC + k0 + 2 * tq], sm.T[r0 * LC + k0 + 2 * tq + 1], ah[0], al[0]);
        split2(sm.T[(r0 + 8) * LC + k0 + 2 * tq], sm.T[(r0 + 8) * LC + k0 + 2 * tq + 1], ah[1], al[1]);
        split2(sm.T[r0 * LC + k0 + 2 * tq + 8], sm.T[r0 * LC + k0 + 2 * tq + 9], ah[2], al[2]);
        split2(sm.T[(r0 + 8) * LC + k0 + 2 * tq + 8], sm.T[(r0 + 8) * LC + k0 + 2 * tq + 9], ah[3], al[3]);
#pragma unroll
        for (int n = 0; n < NW; ++n) {
          const int col = cbase + 8 * n + g8;  // B[kk][n] = Y[k0 + kk][col] = Y^T[col][k0 + kk]
          const __nv_bfloat16* yh = sm.Yh + col * LY + k0 + 2 * tq;
          const __nv_bfloat16* yl = sm.Yl + col * LY + k0 + 2 * tq;
          uint32_t bh[2], bl[2];
          bh[0] = *reinterpret_cast<const uint32_t*>(yh);
          bh[1] = *reinterpret_cast<const uint32_t*>(yh + 8);
          bl[0] = *reinterpret_cast<const uint32_t*>(yl);
          bl[1] = *reinterpret_cast<const uint32_t*>(yl + 8);
          mma16816(accU[n], ah, bh);
          mma16816(accU[n], ah, bl);
          mma16816(accU[n], al, bh);
        }
      }
      __syncthreads();  // every warp has read Y
#pragma unroll
      for (int n = 0; n < NW; ++n) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int t = 16 * mt + g8 + (e >= 2 ? 8 : 0);
          const int col = cbase + 8 * n + 2 * tq + (e & 1);
          const __nv_bfloat16 hi = __float2bfloat16_rn(accU[n][e]);
          sm.Yh[col * LY + t] = hi;
          sm.Yl[col * LY + t] = __float2bfloat16_rn(accU[n][e] - __bfloat162float(hi));
        }
      }
    }
    __syncthreads();

    // ---- step 5: O = Oacc + P U (P lower triangular), bf16 out
    {
      for (int k0 = 0; k0 < 16 * (mt + 1); k0 += 16) {
        uint32_t ah[4], al[4];
        const int r0 = 16 * mt + g8;
        split2(sm.P[r0 * LC + k0 + 2 * tq], sm.P[r0 * LC + k0 + 2 * tq + 1], ah[0], al[0]);
        split2(sm.P[(r0 + 8) * LC + k0 + 2 * tq], sm.P[(r0 + 8) * LC + k0 + 2 * tq + 1], ah[1], al[1]);
        split2(sm.P[r0 * LC + k0 + 2 * tq + 8], sm.P[r0 * LC + k0 + 2 * tq + 9], ah[2], al[2]);
        split2(sm.P[(r0 + 8) * LC + k0 + 2 * tq + 8], sm.P[(r0 + 8) * LC + k0 + 2 * tq + 9], ah[3], al[3]);
#pragma unroll
        for (int n = 0; n < NW; ++n) {
          const int col = cbase + 8 * n + g8;  // B[kk][n] = U[k0 + kk][col] = U^T[col][k0 + kk]
          const __nv_bfloat16* uh = sm.Yh + col * LY + k0 + 2 * tq;
          const __nv_bfloat16* ul = sm.Yl + col * LY + k0 + 2 * tq;
          uint32_t bh[2], bl[2];
          bh[0] = *reinterpret_cast<const uint32_t*>(uh);
          bh[1] = *reinterpret_cast<const uint32_t*>(uh + 8);
          bl[0] = *reinterpret_cast<const uint32_t*>(ul);
          bl[1] = *reinterpret_cast<const uint32_t*>(ul + 8);
          mma16816(oacc[n], ah, bh);
          mma16816(oacc[n], ah, bl);
          mma16816(oacc[n], al, bh);
        }
      }
#pragma unroll
      for (int n = 0; n < NW; ++n) {
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          const int t = 16 * mt + g8 + 8 * half;
          const int64_t tok = (int64_t)c * C + t;
          if (tok < len) {
            const int col = cbase + 8 * n + 2 * tq;
            *reinterpret_cast<__nv_bfloat162*>(p.out + (t_begin + tok) * row_stride + (int64_t)h * D + col) =
                __floats2bfloat162_rn(oacc[n][2 * half], oacc[n][2 * half + 1]);
          }
        }
      }
    }

    // ---- step 6: S = gamma_C S + K^T diag(exp(G_C - G_t)) U; warp w owns state rows (keys) 16w .. 16w+15
    {
      const float gC = sm.G[C - 1];
      const float gamC = sm.gam[C - 1];
      constexpr int NT = D / 8;
      const int m0 = 16 * warp;
      const bool owner = m0 < D;  // D = 64 leaves warps 4..7 without state rows
      float acc[NT][4];
      if (owner) {
#pragma unroll
        for (int n = 0; n < NT; ++n) {
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int row = m0 + g8 + (e >= 2 ? 8 : 0), col = 8 * n + 2 * tq + (e & 1);
            acc[n][e] = gamC * (__bfloat162float(sm.Sh[col * LB + row]) + __bfloat162float(sm.Sl[col * LB + row]));
          }
        }
#pragma unroll
        for (int k0 = 0; k0 < C; k0 += 16) {
          // A[m][kk] = exp(G_C - G_t) K[t = k0 + kk][m0 + m] (diag(f) K, transposed), split into bf16 hi + lo
          const float f0 = expf(gC - sm.G[k0 + 2 * tq]), f1 = expf(gC - sm.G[k0 + 2 * tq + 1]);
          const float f8 = expf(gC - sm.G[k0 + 2 * tq + 8]), f9 = expf(gC - sm.G[k0 + 2 * tq + 9]);
          auto kv = [&](int t, int m) { return __bfloat162float(K[t * LB + m0 + m]); };
          uint32_t ah[4], al[4];
          split2(f0 * kv(k0 + 2 * tq, g8), f1 * kv(k0 + 2 * tq + 1, g8), ah[0], al[0]);
          split2(f0 * kv(k0 + 2 * tq, g8 + 8), f1 * kv(k0 + 2 * tq + 1, g8 + 8), ah[1], al[1]);
          split2(f8 * kv(k0 + 2 * tq + 8, g8), f9 * kv(k0 + 2 * tq + 9, g8), ah[2], al[2]);
          split2(f8 * kv(k0 + 2 * tq + 8, g8 + 8), f9 * kv(k0 + 2 * tq + 9, g8 + 8), ah[3], al[3]);
#pragma unroll
          for (int n = 0; n < NT; ++n) {
            const int col = 8 * n + g8;  // B[kk][n] = U[k0 + kk][col] = U^T[col][k0 + kk]
            const __nv_bfloat16* uh = sm.Yh + col * LY + k0 + 2 * tq;
            const __nv_bfloat16* ul = sm.Yl + col * LY + k0 + 2 * tq;
            uint32_t bh[2], bl[2];
            bh[0] = *reinterpret_cast<const uint32_t*>(uh);
            bh[1] = *reinterpret_cast<const uint32_t*>(uh + 8);
            bl[0] = *reinterpret_cast<const uint32_t*>(ul);
            bl[1] = *reinterpret_cast<const uint32_t*>(ul + 8);
            mma16816(acc[n], ah, bh);
            mma16816(acc[n], ah, bl);
            mma16816(acc[n], al, bh);
          }
        }
      }
      __syncthreads();  // all reads of S0 (steps 3 and 6) are done before it is overwritten
      if (owner) {
#pragma unroll
        for (int n = 0; n < NT; ++n) {
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int row = m0 + g8 + (e >= 2 ? 8 : 0), col = 8 * n + 2 * tq + (e & 1);
            const __nv_bfloat16 hi = __float2bfloat16_rn(acc[n][e]);
            sm.Sh[col * LB + row] = hi;
            sm.Sl[col * LB + row] = __float2bfloat16_rn(acc[n][e] - __bfloat162float(hi));
          }
        }
      }
    }
    __syncthreads();
  }

  if (p.final_state) {
    for (int i = tid; i < D * D; i += kThreads) {
      const int vi = i / D, ki = i % D;
      p.final_state[((slot * p.H + h) * D + vi) * (int64_t)D + ki] =
          __bfloat162float(sm.Sh[vi * LB + ki]) + __bfloat162float(sm.Sl[vi * LB + ki]);
    }
  }
}

}  // namespace

namespace zb {
int64_t gdn_prefill_tc_workspace_bytes(int64_t total_tokens, int num_seqs, int H);
int gdn_prefill_tc_launch(const uint16_t* q, const uint16_t* k, const uint16_t* v, const float* g, const float* beta,
                          const int32_t* cu_seqlens, int num_seqs, int H, float scale, const float* init_state,
                          const int64_t* state_slots, float* final_state, uint16_t* out, int64_t total_tokens,
                          void* workspace, int64_t workspace_bytes, cudaStream_t stream);
}

ZB_API int64_t zb_gdn_chunk_prefill_workspace_bytes(int64_t total_tokens, int num_seqs, int H, int dk) {
  if (total_tokens < 0 || num_seqs < 0 || H <= 0 || dk != 128) return 0;
  return zb::gdn_prefill_tc_workspace_bytes(total_tokens, num_seqs, H);
}

ZB_API int zb_gdn_chunk_prefill(const uint16_t* q, const uint16_t* k, const uint16_t* v, const float* g,
                                const float* beta, const int32_t* cu_seqlens, int num_seqs, int H, int dk, int dv,
                                float scale, const float* init_state, const int64_t* state_slots, float* final_state,
                                uint16_t* out, int64_t total_tokens, void* workspace, int64_t workspace_bytes,
                                cudaStream_t stream) {
  ZB_REQUIRE(num_seqs >= 0 && H > 0 && total_tokens >= 0, "gdn_chunk_prefill: bad sizes num_seqs=%d H=%d N=%lld",
             num_seqs, H, (long long)total_tokens);
  if (dk != dv || (dk != 64 && dk != 128))
    return zb::fail(zb::kUnsupported, "gdn_chunk_prefill: dk=%d dv=%d (equal, 64 or 128)", dk, dv);
  if (num_seqs == 0) return zb::kOk;
  ZB_REQUIRE(q && k && v && g && beta && cu_seqlens && out, "gdn_chunk_prefill: null pointer");
  for (const void* ptr : {(const void*)q, (const void*)k, (const void*)v, (const void*)out})
    ZB_REQUIRE_ALIGNED(ptr, 16, "gdn_chunk_prefill q/k/v/out");
  ZB_REQUIRE(H <= 65535, "gdn_chunk_prefill: H=%d (grid y limit)", H);
  if (dk == 128)
    return zb::gdn_prefill_tc_launch(q, k, v, g, beta, cu_seqlens, num_seqs, H, scale, init_state, state_slots,
                                     final_state, out, total_tokens, workspace, workspace_bytes, stream);
  PrefillParams p{reinterpret_cast<const __nv_bfloat16*>(q), reinterpret_cast<const __nv_bfloat16*>(k),
                  reinterpret_cast<const __nv_bfloat16*>(v), g, beta, cu_seqlens, init_state, state_slots,
                  final_state, reinterpret_cast<__nv_bfloat16*>(out), H, scale};
  const size_t smem = sizeof(Smem<64>);
  ZB_CUDA(cudaFuncSetAttribute(gdn_chunk_prefill_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               (int)smem));
  ZB_CUDA(zb::launch(gdn_chunk_prefill_kernel<64>, dim3(dim3((unsigned)num_seqs, (unsigned)H)), dim3(kThreads), smem, stream, 1, p));
  return zb::check_launch("gdn_chunk_prefill");
}

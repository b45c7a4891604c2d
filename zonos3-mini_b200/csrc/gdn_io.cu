// GDN prologue and epilogue around the recurrence.
//
// Prologue (replaces FLA causal_conv1d_fwd + l2norm_fwd x2 + the in-kernel gate and fused_beta_sigmoid_fwd of
// OriginalGDN._run_packed, servers/sgl/src/zonos3_sgl/models/gdn.py:403-434; math of
// model/src/zonos3/reference/lm.py:561-573): from the in_proj output rows [qkv (3*inner) | z (inner) | a (H) | b (H)]
//   conv = SiLU(depthwise causal conv, kernel W, over the qkv channels, continuing each sequence's history)
//   q, k = conv_q, conv_k * rsqrt(sum^2 + 1e-6) per head;  v = conv_v
//   g = -exp(A_log) * softplus(a + dt_bias)  (log decay);  beta = sigmoid(b)
// One CTA per (token, q / k / v part); a warp covers one head slice (D / 32 channels per lane), so the per-head L2
// norm is a warp reduction. History rows before a sequence's first token come from conv_state [slot, channels, W-1]
// (the layout of LMCache.conv_state); a second small kernel then writes each sequence's new history (its last W-1
// inputs), after every token has read the old one. Decode (one token per sequence, zb_gdn_prologue_decode): the CTA
// that reads a sequence's history rows of its channels is their only reader, so it writes the shifted history
// (the last W-2 entries and the token's input) itself and the second kernel is not launched; for D = 64 / 128 it runs
// gdn_prologue_decode8_kernel, 8 channels (16-byte vectors) per thread, so the step's 256 x 3 CTAs are one wave.
//
// Epilogue (replaces FLA layer_norm_gated_fwd, gdn.py:435-445; lm.py:585-587): gated = RMSNorm(o; out_weight,
// 1e-5) * SiLU(z) per head, computed in fp32 and rounded once to bf16; one warp per (token, head).
#include "common.cuh"

namespace {

constexpr int kW = 4;  // conv kernel width of the release GDN

struct PrologueParams {
  const __nv_bfloat16* mixed;  // [N, 4*inner + 2H]
  int64_t mixed_stride;
  const __nv_bfloat16* conv_w;  // [3*inner, W]
  const float* A_log;           // [H]
  const float* dt_bias;         // [H]
  const int32_t* cu_seqlens;    // [n + 1] (decode: n = N, cu = 0..N)
  const int32_t* seq_of_token;  // [N] sequence index of every token
  const int64_t* slots;         // [n] conv-state row of each sequence
  __nv_bfloat16* conv_state;    // [rows, 3*inner, W-1]
  int64_t rows;                 // conv_state rows; a slot outside [0, rows) is a padding sequence
  const uint8_t* fresh;         // [n] 1 = history starts at zero (or null: always use conv_state)
  __nv_bfloat16* q;             // [N, H, D]
  __nv_bfloat16* k;
  __nv_bfloat16* v;
  float* g;                     // [N, H]
  float* beta;
  int N, H, D;
};

__device__ __forceinline__ float silu(float x) { return x / (1.0f + expf(-x)); }
__device__ __forceinline__ float softplus(float x) { return x > 20.f ? x : log1pf(expf(x)); }

// PL consecutive bf16 values (PL = 1, 2 or 4; 2- / 4- / 8-byte aligned) as floats
template <int PL>
__device__ __forceinline__ void load_bf(const __nv_bfloat16* src, float (&out)[PL]) {
  if constexpr (PL == 4) {
    const uint2 u = *reinterpret_cast<const uint2*>(src);
    out[0] = __uint_as_float(u.x << 16);
    out[1] = __uint_as_float(u.x & 0xffff0000u);
    out[2] = __uint_as_float(u.y << 16);
    out[3] = __uint_as_float(u.y & 0xffff0000u);
  } else if constexpr (PL == 2) {
    const uint32_t u = *reinterpret_cast<const uint32_t*>(src);
    out[0] = __uint_as_float(u << 16);
    out[1] = __uint_as_float(u & 0xffff0000u);
  } else {
#pragma unroll
    for (int j = 0; j < PL; ++j) out[j] = __bfloat162float(src[j]);
  }
}

// One CTA per (token, part): part 0 = q, 1 = k, 2 = v; warp h covers head h's D channels, lane owns PL = D / 32
// consecutive channels. Every input of a lane (its PL x W weights, the history rows and the rows of this sequence)
// is loaded before any arithmetic. kDecode: token i is sequence i (no cu_seqlens / seq_of_token / fresh), and the
// lane replaces its channels' history rows.
template <int PL, bool kDecode>
__global__ void __launch_bounds__(1024) gdn_prologue_kernel(PrologueParams p) {
  zb::pdl_enter();
  const int64_t tok = blockIdx.x;
  const int part = blockIdx.y;
  const int h = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int inner = p.H * p.D;
  const int seq = kDecode ? (int)tok : p.seq_of_token[tok];
  const int64_t start = kDecode ? tok : p.cu_seqlens[seq];
  const int64_t pos = tok - start;  // position inside the sequence
  const int64_t slot = p.slots[seq];
  // a padding sequence (graph padding rows) reads a zero history and never writes one
  const bool padding = slot < 0 || slot >= p.rows;
  const bool fresh = (!kDecode && p.fresh ? p.fresh[seq] != 0 : false) || padding;
  const __nv_bfloat16* row = p.mixed + tok * p.mixed_stride;
  const int ch0 = part * inner + h * p.D + lane * PL;

  float wt[PL * kW];  // conv weights [channel][tap]
  {
    float tmp[4];
#pragma unroll
    for (int j = 0; j < PL * kW; j += 4) {
      load_bf<4>(p.conv_w + (int64_t)ch0 * kW + j, tmp);
#pragma unroll
      for (int u = 0; u < 4; ++u) wt[j + u] = tmp[u];
    }
  }
  float hist[PL * (kW - 1)];  // history [channel][entry], zero for a fresh sequence
  if (!fresh && pos < kW - 1) {
    const __nv_bfloat16* hp = p.conv_state + (slot * 3 * inner + ch0) * (kW - 1);
    if constexpr (PL == 4) {  // 12 entries, 8-byte aligned: three 8-byte loads
      float tmp[4];
#pragma unroll
      for (int j = 0; j < 12; j += 4) {
        load_bf<4>(hp + j, tmp);
#pragma unroll
        for (int u = 0; u < 4; ++u) hist[j + u] = tmp[u];
      }
    } else {
#pragma unroll
      for (int j = 0; j < PL * (kW - 1); ++j) hist[j] = __bfloat162float(hp[j]);
    }
  } else {
#pragma unroll
    for (int j = 0; j < PL * (kW - 1); ++j) hist[j] = 0.f;
  }
  float xin[kW][PL];  // tap w = the input (W-1-w) steps before this token
#pragma unroll
  for (int w = 0; w < kW; ++w) {
    const int64_t back = kW - 1 - w;
    if (back <= pos) {
      load_bf<PL>(row - back * p.mixed_stride + ch0, xin[w]);
    } else {  // from the history: entry (W-1) - (back - pos)
      const int64_t hidx = (kW - 1) - (back - pos);
#pragma unroll
      for (int j = 0; j < PL; ++j) xin[w][j] = hist[j * (kW - 1) + hidx];
    }
  }
  if (kDecode && !padding) {  // new history of the lane's channels: old entries 1 .. W-2, then this token's input
    float nh[PL * (kW - 1)];
#pragma unroll
    for (int j = 0; j < PL; ++j) {
#pragma unroll
      for (int e = 0; e < kW - 2; ++e) nh[j * (kW - 1) + e] = hist[j * (kW - 1) + e + 1];
      nh[j * (kW - 1) + kW - 2] = xin[kW - 1][j];
    }
    __nv_bfloat16* hp = p.conv_state + (slot * 3 * inner + ch0) * (kW - 1);
    if constexpr (PL == 4) {  // 12 entries, 8-byte aligned: three 8-byte stores
#pragma unroll
      for (int j = 0; j < 12; j += 4) {
        const __nv_bfloat162 a = __floats2bfloat162_rn(nh[j], nh[j + 1]);
        const __nv_bfloat162 b = __floats2bfloat162_rn(nh[j + 2], nh[j + 3]);
        *reinterpret_cast<uint2*>(hp + j) =
            make_uint2(*reinterpret_cast<const uint32_t*>(&a), *reinterpret_cast<const uint32_t*>(&b));
      }
    } else {
#pragma unroll
      for (int j = 0; j < PL * (kW - 1); ++j) hp[j] = __float2bfloat16_rn(nh[j]);
    }
  }
  float acc[PL];
#pragma unroll
  for (int j = 0; j < PL; ++j) {
    float a = 0.f;
#pragma unroll
    for (int w = 0; w < kW; ++w) a = fmaf(wt[j * kW + w], xin[w][j], a);
    acc[j] = zb::bf16_round(silu(a));  // the conv output is an activation of the model dtype
  }
  float scale = 1.f;
  if (part < 2) {
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < PL; ++j) ss = fmaf(acc[j], acc[j], ss);
    scale = rsqrtf(zb::warp_sum(ss) + 1e-6f);
  }
  __nv_bfloat16* dst = (part == 0 ? p.q : part == 1 ? p.k : p.v) + (tok * p.H + h) * p.D + lane * PL;
  if constexpr (PL == 4) {
    const __nv_bfloat162 o0 = __floats2bfloat162_rn(acc[0] * scale, acc[1] * scale);
    const __nv_bfloat162 o1 = __floats2bfloat162_rn(acc[2] * scale, acc[3] * scale);
    *reinterpret_cast<uint2*>(dst) =
        make_uint2(*reinterpret_cast<const uint32_t*>(&o0), *reinterpret_cast<const uint32_t*>(&o1));
  } else {
#pragma unroll
    for (int j = 0; j < PL; ++j) dst[j] = __float2bfloat16_rn(acc[j] * scale);
  }
  if (part == 0 && threadIdx.x < p.H) {
    const int hh = threadIdx.x;
    const float a = __bfloat162float(row[4 * inner + hh]);
    const float b = __bfloat162float(row[4 * inner + p.H + hh]);
    p.g[tok * p.H + hh] = -expf(p.A_log[hh]) * softplus(a + p.dt_bias[hh]);
    p.beta[tok * p.H + hh] = 1.f / (1.f + expf(-b));
  }
}

// The decode prologue with 8 channels per thread: every input of a thread is one to four 16-byte loads (taps,
// history, the token's in_proj row) issued together, and a (token, part) CTA of inner / 8 threads fits the whole
// 256-stream step in one wave. A head's D channels are D / 8 consecutive lanes, so its L2 norm is a shuffle
// reduction over that lane group. Same arithmetic per channel as gdn_prologue_kernel (taps oldest first).
template <int D>
__global__ void __launch_bounds__(1024) gdn_prologue_decode8_kernel(PrologueParams p) {
  zb::pdl_enter();
  constexpr int kLanesPerHead = D / 8;
  const int64_t tok = blockIdx.x;
  const int part = blockIdx.y;
  const int inner = p.H * D;
  const int c0 = threadIdx.x * 8;     // channel inside the part
  const int ch0 = part * inner + c0;  // conv channel
  const int64_t slot = p.slots[tok];
  const bool padding = slot < 0 || slot >= p.rows;  // graph padding row: zero history, never written
  uint4 wq[4], hq[3];
  const uint4* wp = reinterpret_cast<const uint4*>(p.conv_w + (int64_t)ch0 * kW);
#pragma unroll
  for (int u = 0; u < 4; ++u) wq[u] = __ldg(wp + u);
  uint4* hp = reinterpret_cast<uint4*>(p.conv_state + ((padding ? 0 : slot) * 3 * inner + ch0) * (kW - 1));
  if (!padding) {
#pragma unroll
    for (int u = 0; u < 3; ++u) hq[u] = hp[u];
  } else {
#pragma unroll
    for (int u = 0; u < 3; ++u) hq[u] = make_uint4(0u, 0u, 0u, 0u);
  }
  const uint4 xq = *reinterpret_cast<const uint4*>(p.mixed + tok * p.mixed_stride + ch0);
  const __nv_bfloat16* wt = reinterpret_cast<const __nv_bfloat16*>(wq);  // [8 channels][W]
  const __nv_bfloat16* hist = reinterpret_cast<const __nv_bfloat16*>(hq);  // [8 channels][W-1]
  const __nv_bfloat16* xin = reinterpret_cast<const __nv_bfloat16*>(&xq);
  float acc[8];
  float ss = 0.f;
  uint4 nq[3];
  __nv_bfloat16* nh = reinterpret_cast<__nv_bfloat16*>(nq);
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    float a = 0.f;
#pragma unroll
    for (int w = 0; w < kW - 1; ++w)
      a = fmaf(__bfloat162float(wt[j * kW + w]), __bfloat162float(hist[j * (kW - 1) + w]), a);
    a = fmaf(__bfloat162float(wt[j * kW + kW - 1]), __bfloat162float(xin[j]), a);
    acc[j] = zb::bf16_round(silu(a));  // the conv output is an activation of the model dtype
    ss = fmaf(acc[j], acc[j], ss);
#pragma unroll
    for (int e = 0; e < kW - 2; ++e) nh[j * (kW - 1) + e] = hist[j * (kW - 1) + e + 1];
    nh[j * (kW - 1) + kW - 2] = xin[j];
  }
  if (!padding) {
#pragma unroll
    for (int u = 0; u < 3; ++u) hp[u] = nq[u];
  }
  float scale = 1.f;
  if (part < 2) {
#pragma unroll
    for (int off = kLanesPerHead / 2; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
    scale = rsqrtf(ss + 1e-6f);
  }
  float o[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) o[j] = acc[j] * scale;
  __nv_bfloat16* dst = (part == 0 ? p.q : part == 1 ? p.k : p.v) + tok * inner + c0;
  *reinterpret_cast<uint4*>(dst) = zb::pack_bf16x8(o);
  if (part == 0 && threadIdx.x < p.H) {
    const int hh = threadIdx.x;
    const __nv_bfloat16* row = p.mixed + tok * p.mixed_stride;
    const float av = __bfloat162float(row[4 * inner + hh]);
    const float bv = __bfloat162float(row[4 * inner + p.H + hh]);
    p.g[tok * p.H + hh] = -expf(p.A_log[hh]) * softplus(av + p.dt_bias[hh]);
    p.beta[tok * p.H + hh] = 1.f / (1.f + expf(-bv));
  }
}

// New history of every sequence: its last W-1 conv inputs (shifted in after the old history when it is shorter).
// Grid (sequence, channel block): a thread owns 8 consecutive channels (24 history entries, 48 contiguous bytes).
__global__ void __launch_bounds__(256) gdn_conv_history_kernel(PrologueParams p) {
  zb::pdl_enter();
  const int seq = blockIdx.x;
  const int64_t start = p.cu_seqlens[seq], len = p.cu_seqlens[seq + 1] - start;
  const int64_t slot = p.slots[seq];
  if (slot < 0 || slot >= p.rows) return;
  const bool fresh = p.fresh ? p.fresh[seq] != 0 : false;
  const int channels = 3 * p.H * p.D;
  const int ch = (blockIdx.y * blockDim.x + threadIdx.x) * 8;
  if (ch >= channels) return;
  uint4* hist = reinterpret_cast<uint4*>(p.conv_state + (slot * channels + ch) * (kW - 1));
  uint4 ov[3] = {make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0)};
  if (!fresh && len < kW - 1) {
#pragma unroll
    for (int i = 0; i < 3; ++i) ov[i] = hist[i];
  }
  const __nv_bfloat16* old = reinterpret_cast<const __nv_bfloat16*>(ov);  // [8 channels][W-1 entries]
  uint2 rows[kW - 1][2];  // input rows (W-1-j) steps before the end, 8 channels each (two 8-byte loads)
#pragma unroll
  for (int j = 0; j < kW - 1; ++j) {
    const int64_t back = kW - 1 - j;  // 1 .. W-1
    if (back <= len) {
      const uint2* src = reinterpret_cast<const uint2*>(p.mixed + (start + len - back) * p.mixed_stride + ch);
      rows[j][0] = src[0];
      rows[j][1] = src[1];
    }
  }
  uint4 nv[3];
  __nv_bfloat16* nb = reinterpret_cast<__nv_bfloat16*>(nv);
#pragma unroll
  for (int c = 0; c < 8; ++c) {
#pragma unroll
    for (int j = 0; j < kW - 1; ++j) {
      const int64_t back = kW - 1 - j;
      __nv_bfloat16 x;
      if (back <= len) {
        const __nv_bfloat16* r = reinterpret_cast<const __nv_bfloat16*>(rows[j]);
        x = r[c];
      } else {
        x = old[c * (kW - 1) + j + len];
      }
      nb[c * (kW - 1) + j] = x;
    }
  }
#pragma unroll
  for (int i = 0; i < 3; ++i) hist[i] = nv[i];
}

struct EpilogueParams {
  const __nv_bfloat16* o;  // [N, H, D]
  const __nv_bfloat16* z;  // [N, ...] with row stride z_stride, H*D channels
  int64_t z_stride;
  const __nv_bfloat16* weight;  // [D]
  float eps;
  __nv_bfloat16* out;  // [N, H*D]
  int N, H, D;
};

// A warp per (token, head), PL = D / 32 consecutive channels per lane; o, z and the weight are all loaded (PL-wide
// vectors) before the reduction.
template <int PL>
__global__ void __launch_bounds__(256) gdn_gated_norm_kernel(EpilogueParams p) {
  zb::pdl_enter();
  const int64_t unit = (int64_t)blockIdx.x * 8 + threadIdx.x / 32;  // (token, head)
  const int lane = threadIdx.x % 32;
  if (unit >= (int64_t)p.N * p.H) return;
  const int64_t tok = unit / p.H;
  const int h = (int)(unit % p.H);
  const int c = lane * PL;
  float x[PL], zz[PL], w[PL];
  load_bf<PL>(p.o + unit * p.D + c, x);
  load_bf<PL>(p.z + tok * p.z_stride + h * p.D + c, zz);
  load_bf<PL>(p.weight + c, w);
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < PL; ++j) ss = fmaf(x[j], x[j], ss);
  const float r = rsqrtf(zb::warp_sum(ss) / (float)p.D + p.eps);
  __nv_bfloat16* dst = p.out + tok * (int64_t)p.H * p.D + h * p.D + c;
  if constexpr (PL == 4) {
    const __nv_bfloat162 o0 = __floats2bfloat162_rn(x[0] * r * w[0] * silu(zz[0]), x[1] * r * w[1] * silu(zz[1]));
    const __nv_bfloat162 o1 = __floats2bfloat162_rn(x[2] * r * w[2] * silu(zz[2]), x[3] * r * w[3] * silu(zz[3]));
    *reinterpret_cast<uint2*>(dst) =
        make_uint2(*reinterpret_cast<const uint32_t*>(&o0), *reinterpret_cast<const uint32_t*>(&o1));
  } else {
#pragma unroll
    for (int j = 0; j < PL; ++j) dst[j] = __float2bfloat16_rn(x[j] * r * w[j] * silu(zz[j]));
  }
}

}  // namespace

ZB_API int zb_gdn_prologue(const uint16_t* mixed, int64_t mixed_stride, const uint16_t* conv_weight, const float* A_log,
                           const float* dt_bias, const int32_t* cu_seqlens, const int32_t* seq_of_token,
                           const int64_t* slots, const uint8_t* fresh, uint16_t* conv_state, int64_t conv_rows,
                           int num_seqs, int N,
                           int H, int D, uint16_t* q, uint16_t* k, uint16_t* v, float* g, float* beta,
                           cudaStream_t stream) {
  ZB_REQUIRE(N >= 0 && num_seqs >= 0 && H > 0, "gdn_prologue: bad sizes N=%d n=%d H=%d", N, num_seqs, H);
  if (D % 32 != 0 || D > 128) return zb::fail(zb::kUnsupported, "gdn_prologue: head dim %d (32..128, /32)", D);
  if (N == 0) return zb::kOk;
  ZB_REQUIRE(mixed && conv_weight && A_log && dt_bias && cu_seqlens && seq_of_token && slots && conv_state && q && k &&
                 v && g && beta,
             "gdn_prologue: null pointer");
  ZB_REQUIRE(mixed_stride >= 4LL * H * D + 2 * H, "gdn_prologue: mixed row stride %lld too small",
             (long long)mixed_stride);
  ZB_REQUIRE(H <= 32, "gdn_prologue: H=%d (at most 32)", H);
  ZB_REQUIRE(mixed_stride % 4 == 0, "gdn_prologue: mixed row stride %lld must be a multiple of 4",
             (long long)mixed_stride);
  ZB_REQUIRE_ALIGNED(mixed, 16, "gdn_prologue mixed");
  ZB_REQUIRE_ALIGNED(conv_weight, 16, "gdn_prologue conv_weight");
  ZB_REQUIRE_ALIGNED(conv_state, 16, "gdn_prologue conv_state");
  PrologueParams p{reinterpret_cast<const __nv_bfloat16*>(mixed), mixed_stride,
                   reinterpret_cast<const __nv_bfloat16*>(conv_weight), A_log, dt_bias, cu_seqlens, seq_of_token,
                   slots, reinterpret_cast<__nv_bfloat16*>(conv_state), conv_rows, fresh,
                   reinterpret_cast<__nv_bfloat16*>(q), reinterpret_cast<__nv_bfloat16*>(k),
                   reinterpret_cast<__nv_bfloat16*>(v), g, beta, N, H, D};
  const dim3 grid((unsigned)N, 3);
  const unsigned threads = 32u * (unsigned)H;
  switch (D / 32) {
    case 1: ZB_CUDA(zb::launch(gdn_prologue_kernel<1, false>, dim3(grid), dim3(threads), 0, stream, 1, p)); break;
    case 2: ZB_CUDA(zb::launch(gdn_prologue_kernel<2, false>, dim3(grid), dim3(threads), 0, stream, 1, p)); break;
    case 4: ZB_CUDA(zb::launch(gdn_prologue_kernel<4, false>, dim3(grid), dim3(threads), 0, stream, 1, p)); break;
    default: return zb::fail(zb::kUnsupported, "gdn_prologue: head dim %d (32, 64 or 128)", D);
  }
  if (int rc = zb::check_launch("gdn_prologue")) return rc;
  const int channels = 3 * H * D;
  if (num_seqs > 0)
    ZB_CUDA(zb::launch(gdn_conv_history_kernel, dim3(dim3((unsigned)num_seqs, (unsigned)((channels / 8 + 255) / 256))), dim3(256), 0, stream, 1, p));
  return zb::check_launch("gdn_prologue(history)");
}

ZB_API int zb_gdn_prologue_decode(const uint16_t* mixed, int64_t mixed_stride, const uint16_t* conv_weight,
                                  const float* A_log, const float* dt_bias, const int64_t* slots, uint16_t* conv_state,
                                  int64_t conv_rows, int N, int H, int D, uint16_t* q, uint16_t* k, uint16_t* v,
                                  float* g, float* beta, cudaStream_t stream) {
  ZB_REQUIRE(N >= 0 && H > 0, "gdn_prologue_decode: bad sizes N=%d H=%d", N, H);
  if (D % 32 != 0 || D > 128) return zb::fail(zb::kUnsupported, "gdn_prologue_decode: head dim %d (32..128, /32)", D);
  if (N == 0) return zb::kOk;
  ZB_REQUIRE(mixed && conv_weight && A_log && dt_bias && slots && conv_state && q && k && v && g && beta,
             "gdn_prologue_decode: null pointer");
  ZB_REQUIRE(mixed_stride >= 4LL * H * D + 2 * H, "gdn_prologue_decode: mixed row stride %lld too small",
             (long long)mixed_stride);
  ZB_REQUIRE(H <= 32, "gdn_prologue_decode: H=%d (at most 32)", H);
  ZB_REQUIRE(mixed_stride % 4 == 0, "gdn_prologue_decode: mixed row stride %lld must be a multiple of 4",
             (long long)mixed_stride);
  ZB_REQUIRE_ALIGNED(mixed, 16, "gdn_prologue_decode mixed");
  ZB_REQUIRE_ALIGNED(conv_weight, 16, "gdn_prologue_decode conv_weight");
  ZB_REQUIRE_ALIGNED(conv_state, 16, "gdn_prologue_decode conv_state");
  PrologueParams p{reinterpret_cast<const __nv_bfloat16*>(mixed), mixed_stride,
                   reinterpret_cast<const __nv_bfloat16*>(conv_weight), A_log, dt_bias, nullptr, nullptr, slots,
                   reinterpret_cast<__nv_bfloat16*>(conv_state), conv_rows, nullptr,
                   reinterpret_cast<__nv_bfloat16*>(q), reinterpret_cast<__nv_bfloat16*>(k),
                   reinterpret_cast<__nv_bfloat16*>(v), g, beta, N, H, D};
  const dim3 grid((unsigned)N, 3);
  const int inner = H * D;
  if ((D == 64 || D == 128) && inner % 256 == 0 && inner <= 8192 && mixed_stride % 8 == 0) {
    // 8 channels per thread, one wave (mixed rows 16-byte aligned: the row stride a multiple of 8)
    const unsigned threads8 = (unsigned)(inner / 8);
    if (D == 64)
      ZB_CUDA(zb::launch(gdn_prologue_decode8_kernel<64>, grid, dim3(threads8), 0, stream, 1, p));
    else
      ZB_CUDA(zb::launch(gdn_prologue_decode8_kernel<128>, grid, dim3(threads8), 0, stream, 1, p));
    return zb::check_launch("gdn_prologue_decode");
  }
  const unsigned threads = 32u * (unsigned)H;
  switch (D / 32) {
    case 1: ZB_CUDA(zb::launch(gdn_prologue_kernel<1, true>, dim3(grid), dim3(threads), 0, stream, 1, p)); break;
    case 2: ZB_CUDA(zb::launch(gdn_prologue_kernel<2, true>, dim3(grid), dim3(threads), 0, stream, 1, p)); break;
    case 4: ZB_CUDA(zb::launch(gdn_prologue_kernel<4, true>, dim3(grid), dim3(threads), 0, stream, 1, p)); break;
    default: return zb::fail(zb::kUnsupported, "gdn_prologue_decode: head dim %d (32, 64 or 128)", D);
  }
  return zb::check_launch("gdn_prologue_decode");
}

ZB_API int zb_gdn_gated_norm(const uint16_t* o, const uint16_t* z, int64_t z_stride, const uint16_t* weight, float eps,
                             int N, int H, int D, uint16_t* out, cudaStream_t stream) {
  ZB_REQUIRE(N >= 0 && H > 0, "gdn_gated_norm: bad sizes N=%d H=%d", N, H);
  if (D % 32 != 0 || D > 128) return zb::fail(zb::kUnsupported, "gdn_gated_norm: head dim %d (32..128, /32)", D);
  if (N == 0) return zb::kOk;
  ZB_REQUIRE(o && z && weight && out, "gdn_gated_norm: null pointer");
  ZB_REQUIRE(z_stride >= (int64_t)H * D, "gdn_gated_norm: z_stride");
  EpilogueParams p{reinterpret_cast<const __nv_bfloat16*>(o), reinterpret_cast<const __nv_bfloat16*>(z), z_stride,
                   reinterpret_cast<const __nv_bfloat16*>(weight), eps, reinterpret_cast<__nv_bfloat16*>(out), N, H,
                   D};
  const int pl = D / 32;  // channels per lane, loaded as one vector of pl bf16
  ZB_REQUIRE(z_stride % pl == 0, "gdn_gated_norm: z_stride %lld must be a multiple of %d", (long long)z_stride, pl);
  for (const void* ptr : {(const void*)o, (const void*)z, (const void*)weight, (const void*)out}) {
    ZB_REQUIRE_ALIGNED(ptr, 2 * pl, "gdn_gated_norm tensors");
  }
  const int64_t units = (int64_t)N * H;
  const dim3 grid((unsigned)((units + 7) / 8));
  switch (pl) {
    case 1: ZB_CUDA(zb::launch(gdn_gated_norm_kernel<1>, grid, dim3(256), 0, stream, 1, p)); break;
    case 2: ZB_CUDA(zb::launch(gdn_gated_norm_kernel<2>, grid, dim3(256), 0, stream, 1, p)); break;
    case 4: ZB_CUDA(zb::launch(gdn_gated_norm_kernel<4>, grid, dim3(256), 0, stream, 1, p)); break;
    default: return zb::fail(zb::kUnsupported, "gdn_gated_norm: head dim %d (32, 64 or 128)", D);
  }
  return zb::check_launch("gdn_gated_norm");
}

// GDN prologue and epilogue around the recurrence.
//
// Prologue (replaces FLA causal_conv1d_fwd + l2norm_fwd x2 + the in-kernel gate and fused_beta_sigmoid_fwd of
// OriginalGDN._run_packed, servers/sgl/src/zonos3_sgl/models/gdn.py:403-434; math of
// model/src/zonos3/reference/lm.py:561-573): from the in_proj output rows [qkv (3*inner) | z (inner) | a (H) | b (H)]
//   conv = SiLU(depthwise causal conv, kernel W, over the qkv channels, continuing each sequence's history)
//   q, k = conv_q, conv_k * rsqrt(sum^2 + 1e-6) per head;  v = conv_v
//   g = -exp(A_log) * softplus(a + dt_bias)  (log decay);  beta = sigmoid(b)
// One CTA per token; a warp covers one 128-wide head slice (4 channels per lane), so the per-head L2 norm is a warp
// reduction. History rows before a sequence's first token come from conv_state [slot, channels, W-1] (the layout of
// LMCache.conv_state); a second small kernel then writes each sequence's new history (its last W-1 inputs), after
// every token has read the old one.
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

__global__ void __launch_bounds__(256) gdn_prologue_kernel(PrologueParams p) {
  const int64_t tok = blockIdx.x;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int inner = p.H * p.D;
  const int seq = p.seq_of_token[tok];
  const int64_t start = p.cu_seqlens[seq];
  const int64_t pos = tok - start;  // position inside the sequence
  const int64_t slot = p.slots[seq];
  // a padding sequence (graph padding rows) reads a zero history and never writes one
  const bool fresh = (p.fresh ? p.fresh[seq] != 0 : false) || slot < 0 || slot >= p.rows;
  const __nv_bfloat16* row = p.mixed + tok * p.mixed_stride;
  // 3H head slices of D channels: slice s covers channels [s*D, (s+1)*D); lane owns D/32 consecutive channels
  const int per_lane = p.D / 32;
  for (int slice = warp; slice < 3 * p.H; slice += 8) {
    float acc[4];
    const int c0 = slice * p.D + lane * per_lane;
    for (int j = 0; j < per_lane; ++j) {
      const int ch = c0 + j;
      float a = 0.f;
#pragma unroll
      for (int w = 0; w < kW; ++w) {
        const int64_t back = kW - 1 - w;  // weight[w] multiplies the input `back` steps before this token
        float x;
        if (back <= pos) {
          x = __bfloat162float(row[-back * p.mixed_stride + ch]);
        } else {  // from the history: history index (W-1) - (back - pos)
          const int64_t hidx = (kW - 1) - (back - pos);
          x = fresh ? 0.f : __bfloat162float(p.conv_state[(slot * 3 * inner + ch) * (kW - 1) + hidx]);
        }
        a = fmaf(__bfloat162float(p.conv_w[ch * kW + w]), x, a);
      }
      acc[j] = zb::bf16_round(silu(a));  // the conv output is an activation of the model dtype
    }
    const int part = slice / p.H, head = slice % p.H;  // 0 = q, 1 = k, 2 = v
    float scale = 1.f;
    if (part < 2) {
      float ss = 0.f;
      for (int j = 0; j < per_lane; ++j) ss = fmaf(acc[j], acc[j], ss);
      scale = rsqrtf(zb::warp_sum(ss) + 1e-6f);
    }
    __nv_bfloat16* dst = (part == 0 ? p.q : part == 1 ? p.k : p.v) + (tok * p.H + head) * p.D + lane * per_lane;
    for (int j = 0; j < per_lane; ++j) dst[j] = __float2bfloat16_rn(acc[j] * scale);
  }
  if (threadIdx.x < p.H) {
    const int h = threadIdx.x;
    const float a = __bfloat162float(row[4 * inner + h]);
    const float b = __bfloat162float(row[4 * inner + p.H + h]);
    p.g[tok * p.H + h] = -expf(p.A_log[h]) * softplus(a + p.dt_bias[h]);
    p.beta[tok * p.H + h] = 1.f / (1.f + expf(-b));
  }
}

// New history of every sequence: its last W-1 conv inputs (shifted in after the old history when it is shorter).
__global__ void __launch_bounds__(256) gdn_conv_history_kernel(PrologueParams p) {
  const int seq = blockIdx.x;
  const int64_t start = p.cu_seqlens[seq], len = p.cu_seqlens[seq + 1] - start;
  const int64_t slot = p.slots[seq];
  if (slot < 0 || slot >= p.rows) return;
  const bool fresh = p.fresh ? p.fresh[seq] != 0 : false;
  const int channels = 3 * p.H * p.D;
  for (int ch = threadIdx.x; ch < channels; ch += blockDim.x) {
    __nv_bfloat16* hist = p.conv_state + (slot * channels + ch) * (kW - 1);
    float old[kW - 1];
#pragma unroll
    for (int j = 0; j < kW - 1; ++j) old[j] = fresh ? 0.f : __bfloat162float(hist[j]);
#pragma unroll
    for (int j = 0; j < kW - 1; ++j) {
      // new history entry j = input (W-1-j) steps before the end of the sequence
      const int64_t back = kW - 1 - j;  // 1 .. W-1
      float x;
      if (back <= len) x = __bfloat162float(p.mixed[(start + len - back) * p.mixed_stride + ch]);
      else x = old[j + len];
      hist[j] = __float2bfloat16_rn(x);
    }
  }
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

__global__ void __launch_bounds__(256) gdn_gated_norm_kernel(EpilogueParams p) {
  const int64_t unit = (int64_t)blockIdx.x * 8 + threadIdx.x / 32;  // (token, head)
  const int lane = threadIdx.x % 32;
  if (unit >= (int64_t)p.N * p.H) return;
  const int64_t tok = unit / p.H;
  const int h = (int)(unit % p.H);
  const int per_lane = p.D / 32;
  float x[4], ss = 0.f;
  for (int j = 0; j < per_lane; ++j) {
    x[j] = __bfloat162float(p.o[unit * p.D + lane * per_lane + j]);
    ss = fmaf(x[j], x[j], ss);
  }
  const float r = rsqrtf(zb::warp_sum(ss) / (float)p.D + p.eps);
  for (int j = 0; j < per_lane; ++j) {
    const int c = lane * per_lane + j;
    const float zz = __bfloat162float(p.z[tok * p.z_stride + h * p.D + c]);
    const float w = __bfloat162float(p.weight[c]);
    p.out[tok * (int64_t)p.H * p.D + h * p.D + c] = __float2bfloat16_rn(x[j] * r * w * silu(zz));
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
  PrologueParams p{reinterpret_cast<const __nv_bfloat16*>(mixed), mixed_stride,
                   reinterpret_cast<const __nv_bfloat16*>(conv_weight), A_log, dt_bias, cu_seqlens, seq_of_token,
                   slots, reinterpret_cast<__nv_bfloat16*>(conv_state), conv_rows, fresh,
                   reinterpret_cast<__nv_bfloat16*>(q), reinterpret_cast<__nv_bfloat16*>(k),
                   reinterpret_cast<__nv_bfloat16*>(v), g, beta, N, H, D};
  gdn_prologue_kernel<<<(unsigned)N, 256, 0, stream>>>(p);
  if (int rc = zb::check_launch("gdn_prologue")) return rc;
  if (num_seqs > 0) gdn_conv_history_kernel<<<(unsigned)num_seqs, 256, 0, stream>>>(p);
  return zb::check_launch("gdn_prologue(history)");
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
  const int64_t units = (int64_t)N * H;
  gdn_gated_norm_kernel<<<(unsigned)((units + 7) / 8), 256, 0, stream>>>(p);
  return zb::check_launch("gdn_gated_norm");
}

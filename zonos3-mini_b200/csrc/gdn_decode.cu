// Gated-DeltaNet recurrent decode step: one new token per stream updates each head's fp32 state in place.
//
// Math (the per-token loop of model/src/zonos3/reference/lm.py:576-582, state V-first [H, dv, dk]):
//   S <- S * exp(g)                      decay
//   pred  = S k                          per value row i: sum_j S[i,j] k[j]
//   delta = beta (v - pred)
//   S <- S + delta k^T
//   o = S (q * scale)
// Every value row i of a head is independent once k, q, g, beta are known, so the kernel maps one row of
// DK fp32 (512 B at dk=128) to a group of DK/16 lanes. Each lane holds 16 state floats (four 16-byte
// vectors), and one pass of three fused lane-group reductions gives S_i.k, S_i.q and k.q. The update is then
//   S'_i = d S_i + delta_i k,   o_i = scale (d S_i.q + delta_i k.q),   delta_i = beta (v_i - d S_i.k)
// which is the reference recurrence with the decay folded into the dot products. The state streams through
// once (read 16 B vectors with the evict-first hint, written back the same way); nothing else is re-read.
#include "common.cuh"

namespace {

constexpr int kThreads = 256;

struct DecodeParams {
  const __nv_bfloat16* q;
  const __nv_bfloat16* k;
  const __nv_bfloat16* v;
  int64_t q_stride_b, k_stride_b, v_stride_b;  // elements between consecutive streams
  const float* g;
  const float* beta;
  int64_t gb_stride_b;
  float* state;
  const int64_t* slots;
  int64_t num_slots;
  __nv_bfloat16* out;
  int64_t out_stride_b;
  int B, H, dv;
  float scale;
};

template <int DK>
__global__ void __launch_bounds__(kThreads) gdn_decode_kernel(DecodeParams p) {
  zb::pdl_enter();
  constexpr int LPR = DK / 16;                // lanes per value row
  constexpr int ROWS_PER_CTA = kThreads / LPR;
  const int lane = threadIdx.x % LPR;
  const int64_t row = (int64_t)blockIdx.x * ROWS_PER_CTA + threadIdx.x / LPR;
  const int64_t total_rows = (int64_t)p.B * p.H * p.dv;
  // Rows past the end still take part in the lane-group shuffles with a zero contribution.
  const bool active = row < total_rows;
  const int64_t r = active ? row : 0;
  const int i = (int)(r % p.dv);
  const int64_t bh = r / p.dv;
  const int h = (int)(bh % p.H);
  const int b = (int)(bh / p.H);
  int64_t slot = p.slots ? p.slots[b] : b;
  const bool valid = active && slot >= 0 && slot < p.num_slots;
  if (!valid) slot = 0;

  float* srow = p.state + ((slot * p.H + h) * (int64_t)p.dv + i) * DK;
  const __nv_bfloat16* kp = p.k + b * p.k_stride_b + (int64_t)h * DK;
  const __nv_bfloat16* qp = p.q + b * p.q_stride_b + (int64_t)h * DK;

  float s[16], kk[16], qq[16];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int col = 4 * (lane + LPR * j);
    float4 v4 = valid ? zb::ld_stream_f4(srow + col) : make_float4(0.f, 0.f, 0.f, 0.f);
    s[4 * j + 0] = v4.x; s[4 * j + 1] = v4.y; s[4 * j + 2] = v4.z; s[4 * j + 3] = v4.w;
    zb::ld_bf16x4(kp + col, kk + 4 * j);
    zb::ld_bf16x4(qp + col, qq + 4 * j);
  }
  float sk = 0.f, sq = 0.f, kq = 0.f;
#pragma unroll
  for (int c = 0; c < 16; ++c) {
    sk = fmaf(s[c], kk[c], sk);
    sq = fmaf(s[c], qq[c], sq);
    kq = fmaf(kk[c], qq[c], kq);
  }
#pragma unroll
  for (int off = LPR / 2; off > 0; off >>= 1) {
    sk += __shfl_xor_sync(0xffffffffu, sk, off);
    sq += __shfl_xor_sync(0xffffffffu, sq, off);
    kq += __shfl_xor_sync(0xffffffffu, kq, off);
  }
  const float d = expf(p.g[b * p.gb_stride_b + h]);
  const float bt = p.beta[b * p.gb_stride_b + h];
  const float vi = __bfloat162float(p.v[b * p.v_stride_b + (int64_t)h * p.dv + i]);
  const float delta = bt * (vi - d * sk);
  if (valid) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int col = 4 * (lane + LPR * j);
      float4 o4;
      o4.x = fmaf(d, s[4 * j + 0], delta * kk[4 * j + 0]);
      o4.y = fmaf(d, s[4 * j + 1], delta * kk[4 * j + 1]);
      o4.z = fmaf(d, s[4 * j + 2], delta * kk[4 * j + 2]);
      o4.w = fmaf(d, s[4 * j + 3], delta * kk[4 * j + 3]);
      zb::st_stream_f4(srow + col, o4);
    }
  }
  if (active && lane == 0) {
    const float o = valid ? p.scale * fmaf(d, sq, delta * kq) : 0.f;
    p.out[b * p.out_stride_b + (int64_t)h * p.dv + i] = __float2bfloat16_rn(o);
  }
}

}  // namespace

ZB_API int zb_gdn_decode_step(const uint16_t* q, const uint16_t* k, const uint16_t* v, int64_t q_stride_b,
                                  int64_t k_stride_b, int64_t v_stride_b, const float* g, const float* beta,
                                  int64_t gb_stride_b, float* state, const int64_t* slots, int64_t num_slots,
                                  uint16_t* out, int64_t out_stride_b, int B, int H, int dk, int dv, float scale,
                                  cudaStream_t stream) {
  ZB_REQUIRE(B >= 0 && H > 0 && dv > 0, "gdn_decode_step: bad sizes B=%d H=%d dv=%d", B, H, dv);
  if (dk != 64 && dk != 128) return zb::fail(zb::kUnsupported, "gdn_decode_step: dk=%d (64 or 128)", dk);
  if (B == 0) return zb::kOk;
  ZB_REQUIRE(q && k && v && g && beta && state && out, "gdn_decode_step: null pointer");
  ZB_REQUIRE(num_slots >= (slots ? 1 : B), "gdn_decode_step: num_slots=%lld too small", (long long)num_slots);
  ZB_REQUIRE_ALIGNED(state, 16, "state");
  ZB_REQUIRE_ALIGNED(q, 8, "q");
  ZB_REQUIRE_ALIGNED(k, 8, "k");
  ZB_REQUIRE(q_stride_b % 4 == 0 && k_stride_b % 4 == 0, "gdn_decode_step: q/k batch strides must be multiples of 4");
  ZB_REQUIRE(q_stride_b >= (int64_t)H * dk && k_stride_b >= (int64_t)H * dk && v_stride_b >= (int64_t)H * dv &&
                 out_stride_b >= (int64_t)H * dv && gb_stride_b >= H,
             "gdn_decode_step: batch strides smaller than a row");
  DecodeParams p{reinterpret_cast<const __nv_bfloat16*>(q),
                 reinterpret_cast<const __nv_bfloat16*>(k),
                 reinterpret_cast<const __nv_bfloat16*>(v),
                 q_stride_b, k_stride_b, v_stride_b, g, beta, gb_stride_b, state, slots, num_slots,
                 reinterpret_cast<__nv_bfloat16*>(out), out_stride_b, B, H, dv, scale};
  const int64_t rows = (int64_t)B * H * dv;
  if (dk == 128) {
    const int64_t grid = (rows + (kThreads / 8) - 1) / (kThreads / 8);
    ZB_CUDA(zb::launch(gdn_decode_kernel<128>, dim3((unsigned)grid), dim3(kThreads), 0, stream, 1, p));
  } else {
    const int64_t grid = (rows + (kThreads / 4) - 1) / (kThreads / 4);
    ZB_CUDA(zb::launch(gdn_decode_kernel<64>, dim3((unsigned)grid), dim3(kThreads), 0, stream, 1, p));
  }
  return zb::check_launch("gdn_decode_step");
}

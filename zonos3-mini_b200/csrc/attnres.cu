// Full AttnRes route: one softmax mix over every bank source so far, optionally fused with the RMSNorm that
// follows it and with the append of the current source to the bank.
//
// Reference: full_attnres_route (model/src/zonos3/reference/lm.py:384-389; servers/sgl/src/zonos3_sgl/models/
// zonos3.py:99-113) and the fused Triton route _block_attnres_fwd_kernel (servers/sgl/src/zonos3_sgl/models/
// training_attnres_kernels.py:1268-1348), whose rounding points this kernel keeps: key = bf16(v * inv_rms),
// product = bf16(key * q), logit = fp32 sum, fp32 softmax, weight = bf16, term = bf16(v * weight), fp32 sum of
// terms, bf16 output. The Triton kernel runs one warp per token over the bank twice; here the logit pass is spread
// over one warp per (source, token) row and the mix pass re-reads the rows the logit pass streamed just before,
// so they come from L2 and HBM delivers each source row once.
#include "common.cuh"

namespace {

constexpr int kMaxSources = 256;
constexpr int kThreads = 256;  // 8 warps per token

struct RouteParams {
  const __nv_bfloat16* bank;  // [>= S, T, D]
  int64_t bank_stride;        // elements between two sources of the bank
  int S;                      // bank sources routed over
  const __nv_bfloat16* source;  // optional current source [T, D] (routed as source S)
  __nv_bfloat16* append;        // optional: where to write `source` (the next bank row)
  const __nv_bfloat16* query;   // [D]
  float eps;
  const __nv_bfloat16* norm_weight;  // optional RMSNorm weight applied to the mix
  float norm_eps;
  __nv_bfloat16* out;      // [T, D]: normalised mix if norm_weight, else the mix
  __nv_bfloat16* mix_out;  // optional [T, D]: the un-normalised mix (when norm_weight is given)
  int T, D;
  unsigned* status;
};

// Two kernels per route.
//  attnres_logits_kernel: one warp per (source, token) row — every row of every token is an independent unit of
//  work, so the whole bank streams from HBM with full parallelism. A lane holds VPL 16-byte vectors of the row
//  (D = 256 * VPL, all loads in flight at once); the row's sum of squares and then its logit are warp-shuffle
//  reductions with the reference rounding points. Logits of token t are parked in the first 4*ns bytes of its own
//  output row (ns <= D/2), so the route needs no scratch memory.
//  attnres_mix_kernel: one CTA per token: softmax over its logits (fp32, bf16 weights), then thread i sums the
//  weighted terms of 16-byte column vectors i, i + 256, ... over all sources, 16 sources' loads in flight. Those
//  rows were streamed by the logits kernel just before and are served by L2, so HBM delivers each row once.
constexpr int kLogitWarps = 4;
constexpr int kLogitRows = 2;  // rows per warp, all loads in flight together

template <int VPL>
__global__ void __launch_bounds__(32 * kLogitWarps) attnres_logits_kernel(RouteParams p) {
  const int lane = threadIdx.x % 32;
  const int ns = p.S + (p.source ? 1 : 0);
  const int64_t total = (int64_t)ns * p.T;
  const int64_t row0 = ((int64_t)blockIdx.x * kLogitWarps + threadIdx.x / 32) * kLogitRows;  // rows s * T + t
  const int D = p.D;
  // every load of the warp is issued before any is used: its rows, then its query columns
  uint4 v4[kLogitRows][VPL];
#pragma unroll
  for (int r = 0; r < kLogitRows; ++r) {
    const int64_t row = row0 + r < total ? row0 + r : total - 1;
    const int s = (int)(row / p.T);
    const int64_t t = row % p.T;
    const __nv_bfloat16* src = (s < p.S ? p.bank + (int64_t)s * p.bank_stride : p.source) + t * D;
#pragma unroll
    for (int u = 0; u < VPL; ++u) v4[r][u] = __ldcs(reinterpret_cast<const uint4*>(src + u * 256 + lane * 8));
  }
  uint4 q4[VPL];
#pragma unroll
  for (int u = 0; u < VPL; ++u) q4[u] = *reinterpret_cast<const uint4*>(p.query + u * 256 + lane * 8);
#pragma unroll
  for (int r = 0; r < kLogitRows; ++r) {
    float ss = 0.f;
#pragma unroll
    for (int u = 0; u < VPL; ++u) {
      float v[8];
      zb::ld_bf16x8(reinterpret_cast<const __nv_bfloat16*>(&v4[r][u]), v);
#pragma unroll
      for (int j = 0; j < 8; ++j) ss = fmaf(v[j], v[j], ss);
    }
    const float rr = rsqrtf(zb::warp_sum(ss) / (float)D + p.eps);
    float lg = 0.f;
#pragma unroll
    for (int u = 0; u < VPL; ++u) {
      float v[8], qv[8];
      zb::ld_bf16x8(reinterpret_cast<const __nv_bfloat16*>(&v4[r][u]), v);
      zb::ld_bf16x8(reinterpret_cast<const __nv_bfloat16*>(&q4[u]), qv);
#pragma unroll
      for (int j = 0; j < 8; ++j) lg += zb::bf16_round(zb::bf16_round(v[j] * rr) * qv[j]);
    }
    lg = zb::warp_sum(lg);
    const int64_t row = row0 + r;
    if (lane == 0 && row < total) reinterpret_cast<float*>(p.out + (row % p.T) * D)[row / p.T] = lg;
  }
}

constexpr int kMixBatch = 16;  // source rows in flight per thread in the mix

template <int VPL>
__global__ void __launch_bounds__(kThreads) attnres_mix_kernel(RouteParams p) {
  constexpr int kWarps = kThreads / 32;
  constexpr int kVecs = (32 * VPL + kThreads - 1) / kThreads;  // 16-byte column vectors per thread
  const int64_t t = blockIdx.x;
  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  const int ns = p.S + (p.source ? 1 : 0);
  const int D = p.D;
  __shared__ float weight[kMaxSources];
  __shared__ float red[kWarps];
  const float* logits = reinterpret_cast<const float*>(p.out + t * D);
  for (int s = tid; s < ns; s += kThreads) weight[s] = logits[s];
  __syncthreads();
  if (warp == 0) {  // softmax over the sources (fp32), weights rounded to bf16
    float m = -INFINITY;
    for (int s = lane; s < ns; s += 32) m = fmaxf(m, weight[s]);
    m = zb::warp_max(m);
    float den = 0.f;
    for (int s = lane; s < ns; s += 32) den += expf(weight[s] - m);
    den = zb::warp_sum(den);
    __syncwarp();
    for (int s = lane; s < ns; s += 32) weight[s] = zb::bf16_round(expf(weight[s] - m) / den);
  }
  __syncthreads();  // every thread has read the logits before any output is written over them

  auto row_ptr = [&](int s) -> const __nv_bfloat16* {
    return (s < p.S ? p.bank + (int64_t)s * p.bank_stride : p.source) + t * D;
  };
  const int nvec = D / 8;
  float mix[kVecs][8];
#pragma unroll
  for (int c = 0; c < kVecs; ++c) {
#pragma unroll
    for (int j = 0; j < 8; ++j) mix[c][j] = 0.f;
    const int vec = tid + c * kThreads;
    if (vec >= nvec) continue;
    for (int s0 = 0; s0 < ns; s0 += kMixBatch) {
      uint4 raw[kMixBatch];
#pragma unroll
      for (int i = 0; i < kMixBatch; ++i)
        if (s0 + i < ns) raw[i] = __ldcg(reinterpret_cast<const uint4*>(row_ptr(s0 + i) + vec * 8));
#pragma unroll
      for (int i = 0; i < kMixBatch; ++i) {
        if (s0 + i < ns) {
          float v[8];
          zb::ld_bf16x8(reinterpret_cast<const __nv_bfloat16*>(&raw[i]), v);
          const float w = weight[s0 + i];
#pragma unroll
          for (int j = 0; j < 8; ++j) mix[c][j] += zb::bf16_round(v[j] * w);
        }
      }
      if (p.append && s0 + kMixBatch >= ns) {  // the current source is the last one routed: append it
#pragma unroll
        for (int i = 0; i < kMixBatch; ++i)
          if (s0 + i == ns - 1) *reinterpret_cast<uint4*>(p.append + t * D + vec * 8) = raw[i];
      }
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) mix[c][j] = zb::bf16_round(mix[c][j]);
  }
  if (p.norm_weight) {
    float ss = 0.f;
#pragma unroll
    for (int c = 0; c < kVecs; ++c)
      if (tid + c * kThreads < nvec)
#pragma unroll
        for (int j = 0; j < 8; ++j) ss = fmaf(mix[c][j], mix[c][j], ss);
    ss = zb::warp_sum(ss);
    if (lane == 0) red[warp] = ss;
    __syncthreads();
    float total = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) total += red[w];
    const float rn = rsqrtf(total / (float)D + p.norm_eps);
#pragma unroll
    for (int c = 0; c < kVecs; ++c) {
      const int vec = tid + c * kThreads;
      if (vec >= nvec) continue;
      float nw[8], y[8];
      zb::ld_bf16x8(p.norm_weight + vec * 8, nw);
#pragma unroll
      for (int j = 0; j < 8; ++j) y[j] = mix[c][j] * rn * nw[j];
      if (p.mix_out) *reinterpret_cast<uint4*>(p.mix_out + t * D + vec * 8) = zb::pack_bf16x8(mix[c]);
      *reinterpret_cast<uint4*>(p.out + t * D + vec * 8) = zb::pack_bf16x8(y);
    }
  } else {
#pragma unroll
    for (int c = 0; c < kVecs; ++c) {
      const int vec = tid + c * kThreads;
      if (vec >= nvec) continue;
      *reinterpret_cast<uint4*>(p.out + t * D + vec * 8) = zb::pack_bf16x8(mix[c]);
    }
  }
}

template <int VPL>
int launch(const RouteParams& p, cudaStream_t stream) {
  const int ns = p.S + (p.source ? 1 : 0);
  const int64_t rows = (int64_t)ns * p.T;
  const int64_t per_cta = (int64_t)kLogitWarps * kLogitRows;
  attnres_logits_kernel<VPL><<<(unsigned)((rows + per_cta - 1) / per_cta), 32 * kLogitWarps, 0, stream>>>(p);
  if (int rc = zb::check_launch("attnres_route(logits)")) return rc;
  attnres_mix_kernel<VPL><<<(unsigned)p.T, kThreads, 0, stream>>>(p);
  return zb::check_launch("attnres_route(mix)");
}

}  // namespace

ZB_API int zb_attnres_route(const uint16_t* bank, int64_t bank_stride, int S, const uint16_t* source,
                            uint16_t* append, const uint16_t* query, float eps, const uint16_t* norm_weight,
                            float norm_eps, uint16_t* out, uint16_t* mix_out, int T, int D, cudaStream_t stream) {
  const int ns = S + (source ? 1 : 0);
  ZB_REQUIRE(S >= 0 && T >= 0 && D > 0, "attnres_route: bad sizes S=%d T=%d D=%d", S, T, D);
  ZB_REQUIRE(ns >= 1, "attnres_route: no source to route over");
  if (ns > kMaxSources) return zb::fail(zb::kUnsupported, "attnres_route: %d sources (max %d)", ns, kMaxSources);
  if (D % 256 != 0 || D > 8 * 512)
    return zb::fail(zb::kUnsupported, "attnres_route: D=%d (a multiple of 256, at most 4096)", D);
  if (ns > D / 2)
    return zb::fail(zb::kUnsupported, "attnres_route: %d sources need D >= %d (the logits park in the output row)",
                    ns, 2 * ns);
  if (T == 0) return zb::kOk;
  ZB_REQUIRE(query && out, "attnres_route: null query/out");
  ZB_REQUIRE(out != source && out != append && (mix_out == nullptr || (mix_out != out && mix_out != source)),
             "attnres_route: out / mix_out must not alias the sources");
  ZB_REQUIRE(S == 0 || bank, "attnres_route: null bank with S=%d", S);
  ZB_REQUIRE(!append || source, "attnres_route: append needs a source");
  ZB_REQUIRE(!mix_out || norm_weight, "attnres_route: mix_out is only written with norm_weight");
  ZB_REQUIRE(S == 0 || bank_stride >= (int64_t)T * D, "attnres_route: bank_stride smaller than T*D");
  ZB_REQUIRE(bank_stride % 8 == 0, "attnres_route: bank_stride must be a multiple of 8 elements");
  for (const void* ptr : {(const void*)bank, (const void*)source, (const void*)append, (const void*)query,
                          (const void*)norm_weight, (const void*)out, (const void*)mix_out}) {
    ZB_REQUIRE_ALIGNED(ptr, 16, "attnres_route tensors");
  }
  RouteParams p{reinterpret_cast<const __nv_bfloat16*>(bank), bank_stride, S,
                reinterpret_cast<const __nv_bfloat16*>(source), reinterpret_cast<__nv_bfloat16*>(append),
                reinterpret_cast<const __nv_bfloat16*>(query), eps,
                reinterpret_cast<const __nv_bfloat16*>(norm_weight), norm_eps,
                reinterpret_cast<__nv_bfloat16*>(out), reinterpret_cast<__nv_bfloat16*>(mix_out), T, D,
                zb::device_status_ptr()};
  switch (D / 256) {
    case 1: return launch<1>(p, stream);
    case 2: return launch<2>(p, stream);
    case 3: return launch<3>(p, stream);
    case 4: return launch<4>(p, stream);
    case 6: return launch<6>(p, stream);
    case 8: return launch<8>(p, stream);
    case 12: return launch<12>(p, stream);
    case 16: return launch<16>(p, stream);
    default: return zb::fail(zb::kUnsupported, "attnres_route: D=%d (256, 512, 768, 1024, 1536, 2048, 3072 or 4096)", D);
  }
}

// Full AttnRes route: one softmax mix over every bank source so far, optionally fused with the RMSNorm that
// follows it and with the append of the current source to the bank.
//
// Reference: full_attnres_route (model/src/zonos3/reference/lm.py:384-389; servers/sgl/src/zonos3_sgl/models/
// zonos3.py:99-113) and the fused Triton route _block_attnres_fwd_kernel (servers/sgl/src/zonos3_sgl/models/
// training_attnres_kernels.py:1268-1348), whose rounding points this kernel keeps: key = bf16(v * inv_rms),
// product = bf16(key * q), logit = fp32 sum, fp32 softmax, weight = bf16, term = bf16(v * weight), fp32 sum of
// terms, bf16 output. The Triton kernel reads every bank row twice (logit pass, mix pass); here a token's
// sources are staged in shared memory by one TMA bulk copy per source and read from HBM exactly once.
//
// Parallel layout: a token is one thread-block cluster of CL CTAs; CTA r of the cluster owns columns
// [r*256W, (r+1)*256W) of every source (W warps, 8 bf16 = 16 bytes per thread). The per-source sums that need
// the full row (sum of squares, logit, and the optional norm of the mix) are reduced inside each CTA with warp
// shuffles, then across the cluster through distributed shared memory.
#include <cooperative_groups.h>

#include "common.cuh"

namespace cg = cooperative_groups;

namespace {

constexpr int kMaxSources = 256;

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

template <int W>
__global__ void __launch_bounds__(32 * W) attnres_route_kernel(RouteParams p) {
  constexpr int kThreads = 32 * W;
  constexpr int kCols = 256 * W;  // columns of one CTA
  cg::cluster_group cluster = cg::this_cluster();
  const int CL = (int)cluster.num_blocks();
  const int rank = (int)cluster.block_rank();
  const int64_t t = blockIdx.x / CL;
  const int c0 = rank * kCols;
  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  const int ns = p.S + (p.source ? 1 : 0);

  extern __shared__ __align__(128) unsigned char smem_raw[];
  __nv_bfloat16* tiles = reinterpret_cast<__nv_bfloat16*>(smem_raw);  // [ns][kCols]
  float* red = reinterpret_cast<float*>(smem_raw + (size_t)ns * kCols * 2);  // [ns][W]
  float* part_ss = red + ns * W;                                           // [ns] this CTA's sum of squares
  float* part_lg = part_ss + ns;                                           // [ns] this CTA's logit part
  float* inv_rms = part_lg + ns;                                           // [ns]
  float* weight = inv_rms + ns;                                            // [ns] logits, then bf16 weights
  float* part_n = weight + ns;                                             // [1] norm partial of the mix
  const size_t bar_off = ((size_t)ns * kCols * 2 + (size_t)(ns * W + 4 * ns + 2) * 4 + 7) & ~(size_t)7;
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem_raw + bar_off);
  const uint32_t bar_addr = zb::smem_addr(bar);

  if (tid == 0) {
    zb::mbar_init(bar_addr, 1);
    zb::fence_mbar_init();
  }
  __syncthreads();
  if (tid == 0) {
    const uint32_t slice_bytes = kCols * 2;
    zb::mbar_arrive_expect_tx(bar_addr, slice_bytes * ns);
    for (int s = 0; s < ns; ++s) {
      const __nv_bfloat16* src = (s < p.S ? p.bank + (int64_t)s * p.bank_stride : p.source) + t * p.D + c0;
      zb::bulk_g2s(zb::smem_addr(tiles + (size_t)s * kCols), src, slice_bytes, bar_addr);
    }
  }
  float q[8];
  zb::ld_bf16x8(p.query + c0 + tid * 8, q);
  zb::mbar_wait_bounded(bar_addr, 0, p.status, zb::kStatusAttnresLoadTimeout);

  // sweep 1: sum of squares of every source row (this CTA's columns)
  for (int s = 0; s < ns; ++s) {
    float v[8];
    zb::ld_bf16x8(tiles + (size_t)s * kCols + tid * 8, v);
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) ss = fmaf(v[j], v[j], ss);
    ss = zb::warp_sum(ss);
    if (lane == 0) red[s * W + warp] = ss;
  }
  __syncthreads();
  for (int s = tid; s < ns; s += kThreads) {
    float acc = 0.f;
#pragma unroll
    for (int w = 0; w < W; ++w) acc += red[s * W + w];
    part_ss[s] = acc;
  }
  cluster.sync();
  const float inv_d = 1.0f / (float)p.D;
  for (int s = tid; s < ns; s += kThreads) {
    float total = 0.f;
    for (int r = 0; r < CL; ++r) total += cluster.map_shared_rank(part_ss, r)[s];
    inv_rms[s] = rsqrtf(total * inv_d + p.eps);
  }
  __syncthreads();

  // sweep 2: logits = sum bf16(bf16(v * inv_rms) * q)
  for (int s = 0; s < ns; ++s) {
    float v[8];
    zb::ld_bf16x8(tiles + (size_t)s * kCols + tid * 8, v);
    const float r = inv_rms[s];
    float lg = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) lg += zb::bf16_round(zb::bf16_round(v[j] * r) * q[j]);
    lg = zb::warp_sum(lg);
    if (lane == 0) red[s * W + warp] = lg;
  }
  __syncthreads();
  for (int s = tid; s < ns; s += kThreads) {
    float acc = 0.f;
#pragma unroll
    for (int w = 0; w < W; ++w) acc += red[s * W + w];
    part_lg[s] = acc;
  }
  cluster.sync();
  for (int s = tid; s < ns; s += kThreads) {
    float total = 0.f;
    for (int r = 0; r < CL; ++r) total += cluster.map_shared_rank(part_lg, r)[s];
    weight[s] = total;
  }
  __syncthreads();

  // softmax over the sources (fp32), weights rounded to bf16
  if (warp == 0) {
    float m = -INFINITY;
    for (int s = lane; s < ns; s += 32) m = fmaxf(m, weight[s]);
    m = zb::warp_max(m);
    float den = 0.f;
    for (int s = lane; s < ns; s += 32) den += expf(weight[s] - m);
    den = zb::warp_sum(den);
    __syncwarp();
    for (int s = lane; s < ns; s += 32) weight[s] = zb::bf16_round(expf(weight[s] - m) / den);
  }
  __syncthreads();

  // sweep 3: mix = sum bf16(v * w) in fp32
  float mix[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  for (int s = 0; s < ns; ++s) {
    float v[8];
    zb::ld_bf16x8(tiles + (size_t)s * kCols + tid * 8, v);
    const float w = weight[s];
#pragma unroll
    for (int j = 0; j < 8; ++j) mix[j] += zb::bf16_round(v[j] * w);
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) mix[j] = zb::bf16_round(mix[j]);
  const int64_t off = t * p.D + c0 + tid * 8;
  if (p.norm_weight) {
    if (p.mix_out) *reinterpret_cast<uint4*>(p.mix_out + off) = zb::pack_bf16x8(mix);
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) ss = fmaf(mix[j], mix[j], ss);
    ss = zb::warp_sum(ss);
    if (lane == 0) red[warp] = ss;
    __syncthreads();
    if (tid == 0) {
      float acc = 0.f;
      for (int w = 0; w < W; ++w) acc += red[w];
      part_n[0] = acc;
    }
    cluster.sync();
    float total = 0.f;
    for (int r = 0; r < CL; ++r) total += cluster.map_shared_rank(part_n, r)[0];
    const float rn = rsqrtf(total * inv_d + p.norm_eps);
    float nw[8], y[8];
    zb::ld_bf16x8(p.norm_weight + c0 + tid * 8, nw);
#pragma unroll
    for (int j = 0; j < 8; ++j) y[j] = mix[j] * rn * nw[j];
    *reinterpret_cast<uint4*>(p.out + off) = zb::pack_bf16x8(y);
  } else {
    *reinterpret_cast<uint4*>(p.out + off) = zb::pack_bf16x8(mix);
  }
  if (p.append) {
    *reinterpret_cast<uint4*>(p.append + off) =
        *reinterpret_cast<const uint4*>(tiles + (size_t)(ns - 1) * kCols + tid * 8);
  }
  cluster.sync();  // keep this CTA's shared memory alive until every cluster peer has read it
}

template <int W>
int launch(const RouteParams& p, int CL, cudaStream_t stream) {
  const int ns = p.S + (p.source ? 1 : 0);
  const size_t smem = (size_t)ns * 256 * W * 2 + (size_t)(ns * W + ns * 4 + 2) * sizeof(float) + 16;
  auto kernel = attnres_route_kernel<W>;
  if (smem > 48 * 1024) {
    ZB_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(p.T * CL));
  cfg.blockDim = dim3(32 * W);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = CL;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  ZB_CUDA(cudaLaunchKernelEx(&cfg, kernel, p));
  return zb::check_launch("attnres_route");
}

}  // namespace

ZB_API int zb_attnres_route(const uint16_t* bank, int64_t bank_stride, int S, const uint16_t* source,
                            uint16_t* append, const uint16_t* query, float eps, const uint16_t* norm_weight,
                            float norm_eps, uint16_t* out, uint16_t* mix_out, int T, int D, cudaStream_t stream) {
  const int ns = S + (source ? 1 : 0);
  ZB_REQUIRE(S >= 0 && T >= 0 && D > 0, "attnres_route: bad sizes S=%d T=%d D=%d", S, T, D);
  ZB_REQUIRE(ns >= 1, "attnres_route: no source to route over");
  if (ns > kMaxSources) return zb::fail(zb::kUnsupported, "attnres_route: %d sources (max %d)", ns, kMaxSources);
  if (D % 256 != 0 || D > 8 * 8 * 256)
    return zb::fail(zb::kUnsupported, "attnres_route: D=%d (a multiple of 256, at most 16384)", D);
  if (T == 0) return zb::kOk;
  ZB_REQUIRE(query && out, "attnres_route: null query/out");
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
  // W warps per CTA and CL CTAs per cluster with 256*W*CL == D: the smallest W whose cluster fits in the
  // portable limit of 8, preferring clusters of at most 4 (several small CTAs per SM keep more loads in flight).
  const int units = D / 256;  // = W * CL
  int W = 0, CL = 0;
  for (int w : {1, 2, 4, 8}) {
    if (units % w == 0 && units / w <= 4) { W = w; CL = units / w; break; }
  }
  if (W == 0) {
    for (int w : {1, 2, 4, 8}) {
      if (units % w == 0 && units / w <= 8) { W = w; CL = units / w; break; }
    }
  }
  if (W == 0) return zb::fail(zb::kUnsupported, "attnres_route: D=%d has no cluster split", D);
  switch (W) {
    case 1: return launch<1>(p, CL, stream);
    case 2: return launch<2>(p, CL, stream);
    case 4: return launch<4>(p, CL, stream);
    case 8: return launch<8>(p, CL, stream);
    default: return zb::fail(zb::kUnsupported, "attnres_route: D=%d", D);
  }
}

// Multi-codebook input embedding with the embedding RMSNorm fused: the first two steps of a forward,
//   x = sum_c E_c[ids[:, c]]      (MultiEmbedding.forward, servers/sgl/src/zonos3_sgl/models/zonos3.py:225-255)
//   x = RMSNorm(x; weight, eps)   (emb_norm, zonos3.py:1066-1070 and :1218; weightless there)
// The reference sums the columns' rows one at a time in bf16 (result = result + emb, each add rounded to bf16), so
// this kernel keeps that order and those roundings; the norm computes in fp32 and rounds once.
//
// One CTA per token row, D / 8 threads (rounded up to whole warps), each owning 8 consecutive columns (16-byte loads of every table row). The
// (C + 1) table rows of a token are independent loads issued back to back; the sum of squares is a block reduction.
// An id outside its table is read as a zero row and sets kStatusEmbedIndex in the library status word (the reference
// raises there; a kernel cannot).
#include <algorithm>

#include "common.cuh"

namespace {

constexpr int kMaxTables = 16;

struct EmbedParams {
  const int32_t* ids;  // [N, ncols] (row stride ids_stride)
  int64_t ids_stride;
  int ncols;
  const __nv_bfloat16* table[kMaxTables];  // [rows_c, D] each, contiguous rows
  int rows[kMaxTables];
  const __nv_bfloat16* norm_weight;  // [D] or null (weightless norm)
  float eps;
  int normalize;  // 0: write the plain sum
  int N, D;
  __nv_bfloat16* out;  // [N, D] (row stride out_stride)
  int64_t out_stride;
  unsigned* status;
};

__global__ void __launch_bounds__(512) embed_norm_kernel(EmbedParams p) {
  zb::pdl_enter();
  const int64_t tok = blockIdx.x;
  const int c0 = threadIdx.x * 8;
  const bool live = c0 < p.D;  // the block is a whole number of warps; lanes past the row only join reductions
  __shared__ float partial[32];
  __shared__ float total;
  float acc[8];
  bool bad = false;
  {
    uint4 raw[kMaxTables];
#pragma unroll
    for (int c = 0; c < kMaxTables; ++c) {
      raw[c] = make_uint4(0, 0, 0, 0);
      if (c < p.ncols && live) {
        const int id = p.ids[tok * p.ids_stride + c];
        const bool ok = id >= 0 && id < p.rows[c];
        bad |= !ok;
        if (ok) raw[c] = *reinterpret_cast<const uint4*>(p.table[c] + (int64_t)id * p.D + c0);
      }
    }
#pragma unroll
    for (int c = 0; c < kMaxTables; ++c) {
      if (c < p.ncols) {
        const uint32_t w[4] = {raw[c].x, raw[c].y, raw[c].z, raw[c].w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[i]));
          if (c == 0) {
            acc[2 * i] = f.x;
            acc[2 * i + 1] = f.y;
          } else {  // bf16 + bf16, rounded to bf16: torch's elementwise add of two bf16 tensors
            acc[2 * i] = zb::bf16_round(acc[2 * i] + f.x);
            acc[2 * i + 1] = zb::bf16_round(acc[2 * i + 1] + f.y);
          }
        }
      }
    }
  }
  if (bad && p.status) atomicOr(p.status, zb::kStatusEmbedIndex);
  __nv_bfloat16* dst = p.out + tok * p.out_stride + c0;
  if (!p.normalize) {
    if (live) *reinterpret_cast<uint4*>(dst) = zb::pack_bf16x8(acc);
    return;
  }
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < 8; ++j) ss = fmaf(acc[j], acc[j], ss);
  ss = zb::warp_sum(ss);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32, warps = blockDim.x / 32;
  if (lane == 0) partial[warp] = ss;
  __syncthreads();
  if (warp == 0) {
    float v = lane < warps ? partial[lane] : 0.f;
    v = zb::warp_sum(v);
    if (lane == 0) total = v;
  }
  __syncthreads();
  const float r = rsqrtf(total / (float)p.D + p.eps);
  if (!live) return;
  float y[8];
  if (p.norm_weight) {
    float w[8];
    zb::ld_bf16x8(p.norm_weight + c0, w);
#pragma unroll
    for (int j = 0; j < 8; ++j) y[j] = acc[j] * r * w[j];
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j) y[j] = acc[j] * r;
  }
  *reinterpret_cast<uint4*>(dst) = zb::pack_bf16x8(y);
}

}  // namespace

ZB_API int zb_embed_norm(const int32_t* ids, int64_t ids_stride, int ncols, const uint16_t* const* tables,
                         const int32_t* table_rows, const uint16_t* norm_weight, float eps, int normalize, int N, int D,
                         uint16_t* out, int64_t out_stride, cudaStream_t stream) {
  ZB_REQUIRE(N >= 0 && D > 0, "embed_norm: bad sizes N=%d D=%d", N, D);
  ZB_REQUIRE(ncols >= 1 && ncols <= kMaxTables, "embed_norm: %d id columns (1..%d)", ncols, kMaxTables);
  if (D % 8 != 0 || D > 4096) return zb::fail(zb::kUnsupported, "embed_norm: hidden %d (a multiple of 8, <= 4096)", D);
  if (N == 0) return zb::kOk;
  ZB_REQUIRE(ids && tables && table_rows && out, "embed_norm: null pointer");
  ZB_REQUIRE(ids_stride >= ncols, "embed_norm: ids row stride %lld < %d columns", (long long)ids_stride, ncols);
  ZB_REQUIRE(out_stride >= D && out_stride % 8 == 0, "embed_norm: out row stride %lld", (long long)out_stride);
  ZB_REQUIRE_ALIGNED(out, 16, "embed_norm out");
  if (norm_weight) ZB_REQUIRE_ALIGNED(norm_weight, 16, "embed_norm norm_weight");
  EmbedParams p{};
  p.ids = ids;
  p.ids_stride = ids_stride;
  p.ncols = ncols;
  for (int c = 0; c < ncols; ++c) {
    ZB_REQUIRE(tables[c] != nullptr && table_rows[c] > 0, "embed_norm: table %d missing or empty", c);
    ZB_REQUIRE_ALIGNED(tables[c], 16, "embed_norm tables");
    p.table[c] = reinterpret_cast<const __nv_bfloat16*>(tables[c]);
    p.rows[c] = table_rows[c];
  }
  p.norm_weight = reinterpret_cast<const __nv_bfloat16*>(norm_weight);
  p.eps = eps;
  p.normalize = normalize != 0;
  p.N = N;
  p.D = D;
  p.out = reinterpret_cast<__nv_bfloat16*>(out);
  p.out_stride = out_stride;
  p.status = zb::device_status_ptr();
  const unsigned threads = (unsigned)((D / 8 + 31) / 32 * 32);
  ZB_CUDA(zb::launch(embed_norm_kernel, dim3((unsigned)N), dim3(threads), 0, stream, 1, p));
  return zb::check_launch("embed_norm");
}

// ------------------------------------------------------------------------------------ decode-step bookkeeping

namespace {

struct AdvanceParams {
  const int32_t* codes;  // [B, codes_cols] sampled codes (then the text column)
  int codes_cols;
  int32_t* ids;  // [B, ids_cols]: the next step's input ids
  int ids_cols;
  int32_t* history;  // [B, C, W] repetition window, or null
  int C, W;
  int64_t* ring;     // [1] next window column
  int64_t* counter;  // [1] the sampler's draw counter
  int32_t* positions;
  int32_t* seqlens;
  int32_t* out_loc;
  const int32_t* page_table;  // [B, max_len]
  int64_t table_stride;
  int max_len;
  int B;
};

// One block: every stream's next ids, its codes in the repetition window at the ring column, its position and
// cache length + 1, its next KV slot from the page table; then the ring column and the draw counter advance.
__global__ void __launch_bounds__(1024) decode_advance_kernel(AdvanceParams p) {
  zb::pdl_enter();
  const int64_t col = p.W > 0 ? *p.ring : 0;
  for (int b = threadIdx.x; b < p.B; b += blockDim.x) {
    const int32_t* cb = p.codes + (int64_t)b * p.codes_cols;
    for (int j = 0; j < p.ids_cols; ++j) p.ids[(int64_t)b * p.ids_cols + j] = cb[j];
    if (p.history)
      for (int c = 0; c < p.C; ++c) p.history[((int64_t)b * p.C + c) * p.W + col] = cb[c];
    p.positions[b] += 1;
    const int len = min(p.seqlens[b] + 1, p.max_len);
    p.seqlens[b] = len;
    p.out_loc[b] = p.page_table[(int64_t)b * p.table_stride + len - 1];
  }
  __syncthreads();  // every thread has read the ring column
  if (threadIdx.x == 0) {
    if (p.W > 0) *p.ring = (col + 1) % p.W;
    *p.counter += 1;
  }
}

}  // namespace

ZB_API int zb_decode_advance(const int32_t* codes, int codes_cols, int32_t* ids, int ids_cols, int32_t* history,
                             int C, int W, int64_t* ring, int64_t* counter, int32_t* positions, int32_t* seqlens,
                             int32_t* out_loc, const int32_t* page_table, int64_t table_stride, int max_len, int B,
                             cudaStream_t stream) {
  ZB_REQUIRE(B >= 0 && codes_cols > 0 && ids_cols > 0 && ids_cols <= codes_cols && C >= 0 && C <= codes_cols &&
                 W >= 0 && max_len > 0 && table_stride >= max_len,
             "decode_advance: bad sizes B=%d codes_cols=%d ids_cols=%d C=%d W=%d max_len=%d", B, codes_cols, ids_cols,
             C, W, max_len);
  if (B == 0) return zb::kOk;
  ZB_REQUIRE(codes && ids && counter && positions && seqlens && out_loc && page_table && (!history || (W > 0 && ring)),
             "decode_advance: null pointer");
  AdvanceParams p{codes, codes_cols, ids, ids_cols, history, C, W, ring, counter, positions, seqlens, out_loc,
                  page_table, table_stride, max_len, B};
  ZB_CUDA(zb::launch(decode_advance_kernel, dim3(1), dim3((unsigned)std::min(B, 1024)), 0, stream, 1, p));
  return zb::check_launch("decode_advance");
}

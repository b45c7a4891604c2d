/* zonos3_b200.h — C ABI of libzonos3_b200.so, the B200 (sm_100a) kernels of the ZONOS3-Mini LM-backbone hot path.
 *
 * Conventions shared by every entry point:
 *  - All tensor pointers are DEVICE pointers owned by the caller; the library allocates nothing unless an entry
 *    point says so. bf16 tensors are passed as uint16_t* (raw bf16 bits), fp32 as float*.
 *  - Every call is asynchronous on `stream` and never synchronises the host, so it can be captured in a CUDA graph.
 *  - Every call returns an int status: 0 ok, 1 invalid argument (rejected before any launch), 2 CUDA error,
 *    3 unsupported size, 4 a bounded device-side wait expired. zb_last_error() gives the message of the last
 *    failure on the calling host thread. No C++ exception crosses this boundary.
 *  - Strides are in elements. "[B, H, d]" means B rows of H*d contiguous elements with a caller-given row stride.
 */
#ifndef ZONOS3_B200_H_
#define ZONOS3_B200_H_

#include <cuda_runtime_api.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Message of the last failed call on this host thread ("" if none). */
const char* zb_last_error(void);
void zb_clear_error(void);
int zb_version(void);

/* Kernel launches this library has issued in this process (every device; a launch during stream capture counts
 * once, when it is captured, not on each replay). For launch accounting of captured steps. No reference
 * counterpart. */
uint64_t zb_launch_count(void);

/* Reads the current device's status word (bits set by kernels whose bounded device-side waits expired:
 * 1 = AttnRes source load, 2 = grouped GEMM pipeline, 4 = chunked prefill pipeline, 8 = AttnRes exchange,
 * 16 = decode attention pipeline; 32 = an embedding id outside its table); clear != 0 resets it.
 * Synchronous (a device-to-host copy); for diagnostics and tests, not for the hot path. No reference counterpart:
 * the reference's kernels have no device-side waits. */
int zb_device_status(unsigned* flags, int clear);

/* ------------------------------------------------------------------------------------------- gated DeltaNet */

/* One recurrent gated-delta-rule step per stream, state updated in place.
 * Replaces the per-token recurrence of model/src/zonos3/reference/lm.py:576-582 and the decode use of
 * FLA chunk_gated_delta_rule_fwd in servers/sgl/src/zonos3_sgl/models/gdn.py:418-434 (via _forward_decode_static,
 * gdn.py:329-355).
 *   q, k   [B, H, dk] bf16, L2-normalised per head; row strides q_stride_b, k_stride_b (multiples of 4)
 *   v      [B, H, dv] bf16, row stride v_stride_b
 *   g      [B, H] fp32 log-decay (decay = exp(g)); beta [B, H] fp32; both with row stride gb_stride_b
 *   state  [num_slots, H, dv, dk] fp32 (V-first), 16-byte aligned; stream b uses slot slots[b] (slots == NULL:
 *          slot b); a negative or out-of-range slot marks a padding row: its output is 0 and no state changes
 *   out    [B, H, dv] bf16 = S_new (q * scale), row stride out_stride_b
 *   dk in {64, 128}. */
int zb_gdn_decode_step(const uint16_t* q, const uint16_t* k, const uint16_t* v, int64_t q_stride_b,
                       int64_t k_stride_b, int64_t v_stride_b, const float* g, const float* beta,
                       int64_t gb_stride_b, float* state, const int64_t* slots, int64_t num_slots, uint16_t* out,
                       int64_t out_stride_b, int B, int H, int dk, int dv, float scale, cudaStream_t stream);

/* Chunked (C = 64) gated delta rule over packed variable-length sequences: the prefill / continuation pass.
 * Replaces FLA chunk_gated_delta_rule_fwd as called by OriginalGDN._run_packed
 * (servers/sgl/src/zonos3_sgl/models/gdn.py:418-434; use_gate_in_kernel, state_v_first, cu_seqlens, chunk 64);
 * result equal to the per-token recurrence of model/src/zonos3/reference/lm.py:576-582.
 *   q, k [N, H, dk], v [N, H, dv] bf16 contiguous (16-byte aligned); g (log decay), beta [N, H] fp32
 *   cu_seqlens [num_seqs + 1] int32 (device): sequence i is tokens [cu[i], cu[i+1]); total_tokens = N
 *   init_state / final_state [rows, H, dv, dk] fp32 V-first or NULL (zero start / not written); sequence i uses
 *   row state_slots[i] (int64) or row i when state_slots is NULL; out [N, H, dv] bf16 = S_t (q_t * scale)
 *   dk == dv in {64, 128}. dk = 128 runs on tcgen05 in two kernels (a parallel chunk preparation, then one CTA per
 *   (sequence, head) with the fp32 state in tensor memory) and needs a 16-byte aligned device workspace of
 *   zb_gdn_chunk_prefill_workspace_bytes(N, num_seqs, H, dk) bytes; dk = 64 needs none (NULL, 0). */
int zb_gdn_chunk_prefill(const uint16_t* q, const uint16_t* k, const uint16_t* v, const float* g, const float* beta,
                         const int32_t* cu_seqlens, int num_seqs, int H, int dk, int dv, float scale,
                         const float* init_state, const int64_t* state_slots, float* final_state, uint16_t* out,
                         int64_t total_tokens, void* workspace, int64_t workspace_bytes, cudaStream_t stream);

/* Workspace bytes zb_gdn_chunk_prefill needs for N = total_tokens tokens in num_seqs sequences (0 when dk != 128):
 * 33,792 bytes per (chunk record, head), (ceil(N / 64) + num_seqs) records. The torch-side equivalent is the
 * intermediate tensors FLA's chunk_gated_delta_rule_fwd allocates per call. */
int64_t zb_gdn_chunk_prefill_workspace_bytes(int64_t total_tokens, int num_seqs, int H, int dk);

/* GDN prologue: from the in_proj output rows mixed [N, 4*H*D + 2*H] (qkv | z | a | b, row stride mixed_stride):
 * depthwise causal conv (kernel 4, conv_weight [3*H*D, 1, 4] bf16) + SiLU over the qkv channels continuing each
 * sequence's history, per-head L2 norm (eps 1e-6) of q and k, g = -exp(A_log) * softplus(a + dt_bias), beta =
 * sigmoid(b). Sequences: cu_seqlens [num_seqs + 1] int32, seq_of_token [N] int32, slots [num_seqs] int64 (row of
 * conv_state [conv_rows, 3*H*D, 3] bf16, read as history and replaced by the sequence's last 3 inputs; a slot
 * outside [0, conv_rows) is a padding sequence: zero history, nothing written), fresh [num_seqs] uint8 or NULL
 * (1 = zero history). Outputs q, k, v [N, H, D] bf16, g, beta [N, H] fp32.
 * Replaces FLA causal_conv1d_fwd / l2norm_fwd / fused_beta_sigmoid_fwd and the gate of
 * chunk_gated_delta_rule_fwd in OriginalGDN._run_packed (servers/sgl/src/zonos3_sgl/models/gdn.py:403-434);
 * math of model/src/zonos3/reference/lm.py:561-573. D a multiple of 32, at most 128. */
int zb_gdn_prologue(const uint16_t* mixed, int64_t mixed_stride, const uint16_t* conv_weight, const float* A_log,
                    const float* dt_bias, const int32_t* cu_seqlens, const int32_t* seq_of_token, const int64_t* slots,
                    const uint8_t* fresh, uint16_t* conv_state, int64_t conv_rows, int num_seqs, int N, int H, int D,
                    uint16_t* q,
                    uint16_t* k, uint16_t* v, float* g, float* beta, cudaStream_t stream);

/* The GDN prologue of a decode batch: row i of mixed is the one new token of request i, whose conv history is row
 * slots[i] of conv_state (a slot outside [0, conv_rows) is a padding row: zero history, nothing written); the same
 * kernel replaces each history by its last 2 entries and the token's input, so no second launch follows. Same
 * outputs as zb_gdn_prologue with cu_seqlens = 0..N, seq_of_token = 0..N-1, fresh = NULL. Replaces the conv / L2
 * norm / gate steps of one OriginalGDN._forward_decode_static call (servers/sgl/src/zonos3_sgl/models/gdn.py:329-355
 * through _run_packed, 395-434) for the new row; math of model/src/zonos3/reference/lm.py:561-573. */
int zb_gdn_prologue_decode(const uint16_t* mixed, int64_t mixed_stride, const uint16_t* conv_weight,
                           const float* A_log, const float* dt_bias, const int64_t* slots, uint16_t* conv_state,
                           int64_t conv_rows, int N, int H, int D, uint16_t* q, uint16_t* k, uint16_t* v, float* g,
                           float* beta, cudaStream_t stream);

/* GDN epilogue: out[N, H*D] = bf16(RMSNorm(o; weight [D], eps) * SiLU(z)) per (token, head), o [N, H, D] bf16,
 * z [N, H*D] bf16 with row stride z_stride. Replaces FLA layer_norm_gated_fwd (swish gate, RMS) in
 * OriginalGDN._run_packed (servers/sgl/src/zonos3_sgl/models/gdn.py:435-445); lm.py:585-587. */
int zb_gdn_gated_norm(const uint16_t* o, const uint16_t* z, int64_t z_stride, const uint16_t* weight, float eps, int N,
                      int H, int D, uint16_t* out, cudaStream_t stream);

/* ------------------------------------------------------------------------------- dense projections (tcgen05) */

/* Device workspace bytes of a projection GEMM of T tokens, N output columns and reduction length K with column tile
 * block_n (64, 128, 256; 0 = chosen from the shape) and `splits` K slices (0 = chosen): the split-K ticket counters
 * (first, 256-byte padded) and fp32 partial tiles; 0 when the plan has one slice. */
int64_t zb_proj_gemm_workspace_bytes(int T, int N, int K, int block_n, int splits);

/* out[T, N] = bf16(x[T, K] . weight[N, K]^T), fp32 accumulation on tcgen05 CTA pairs. Replaces the F.linear
 * calls of the decode step: OriginalGDN's wo (servers/sgl/src/zonos3_sgl/models/gdn.py:447), the attention layer's
 * fused projection and wo (servers/sgl/src/zonos3_sgl/models/zonos3.py:326-390) and the multi-codebook head
 * (zonos3.py:1341-1360). K a multiple of 128, N of 8; x / out row strides multiples of 8 elements. With more than one
 * K slice, `workspace` (256-byte aligned, zb_proj_gemm_workspace_bytes) must start with its ticket bytes zeroed
 * before the first launch; every launch leaves them zero. Launches sharing a workspace run in stream order. */
int zb_proj_gemm(const uint16_t* x, int64_t x_stride, int T, int K, const uint16_t* weight, int N, uint16_t* out,
                 int64_t out_stride, int block_n, int splits, void* workspace, int64_t workspace_bytes,
                 cudaStream_t stream);

/* The DeltaNet in_proj GEMM fused with its decode prologue: mixed = x . in_proj^T (in_proj [4*H*D + 2H, K]) is
 * never stored; the GEMM's epilogue runs zb_gdn_prologue_decode's math on it (causal conv continuing conv_state row
 * slots[t], which it shifts in place; SiLU; per-head L2 norm of q and k; g = -exp(A_log) * softplus(a + dt_bias),
 * beta = sigmoid(b)) and stores z [T, H*D] for zb_gdn_gated_norm (z_stride = H*D). Same rounding points as the
 * unfused in_proj + prologue. Replaces OriginalGDN's in_proj and prologue for a decode batch
 * (servers/sgl/src/zonos3_sgl/models/gdn.py:399-434 through _forward_decode_static, :329-355). D = 64 or 128,
 * H*D a multiple of 128, H <= 64; workspace as for zb_proj_gemm with N = 4*H*D + 2H and block_n = 128. */
int zb_gdn_in_proj_decode(const uint16_t* x, int64_t x_stride, int T, int K, const uint16_t* in_proj,
                          const uint16_t* conv_weight, const float* A_log, const float* dt_bias, const int64_t* slots,
                          uint16_t* conv_state, int64_t conv_rows, int H, int D, uint16_t* q, uint16_t* k, uint16_t* v,
                          uint16_t* z, float* g, float* beta, int splits, void* workspace, int64_t workspace_bytes,
                          cudaStream_t stream);

/* ------------------------------------------------------------------------------------------- Full AttnRes */

/* Full AttnRes route of every token over bank sources [0, S) plus, if `source` is non-NULL, `source` as the last
 * source; reads every source row from HBM once (one TMA bulk copy per source slice into shared memory).
 * Replaces full_attnres_route (model/src/zonos3/reference/lm.py:384-389; servers/sgl/src/zonos3_sgl/models/
 * zonos3.py:99-113) and _FusedFullAttnRes.forward / _block_attnres_fwd_kernel
 * (servers/sgl/src/zonos3_sgl/models/training_attnres_kernels.py:2727-2779, :1268-1348), with the bank append of
 * FusedBlockAttnResContext.route_metadata (training_attnres_kernels.py:1491-1513) and the RMSNorm that follows each
 * route (servers/sgl/src/zonos3_sgl/models/training_attnres.py:67-70) fused in.
 *   bank        [>= S, T, D] bf16, bank_stride elements between sources (multiple of 8), rows [T, D] contiguous
 *   source      [T, D] bf16 or NULL; append: [T, D] bf16 destination for `source` or NULL
 *   query       [D] bf16; eps: the key RMSNorm epsilon
 *   norm_weight [D] bf16 or NULL: out = RMSNorm(mix; norm_weight, norm_eps) and mix_out (optional) = mix;
 *               NULL: out = mix (mix_out must be NULL)
 *   rms_cache   fp32 [T, rms_stride] or NULL (16-byte aligned; rms_stride a multiple of 4, at least the routed
 *               sources rounded up to 4): the key inverse RMS of source s for token t at t * rms_stride + s.
 *               Sources [0, cached) are read from it; every later source's value
 *               is computed and written back, so a bank that grows by one row per route reads each row's sum of
 *               squares once (the cached_norm mode of training_attnres_kernels.py:1268-1348).
 *   D a multiple of 256 (at most 8192), S + (source != NULL) in [1, 256]; all pointers 16-byte aligned. */
int zb_attnres_route(const uint16_t* bank, int64_t bank_stride, int S, const uint16_t* source, uint16_t* append,
                     const uint16_t* query, float eps, const uint16_t* norm_weight, float norm_eps, uint16_t* out,
                     uint16_t* mix_out, float* rms_cache, int64_t rms_stride, int cached, int T, int D,
                     cudaStream_t stream);

/* The same route for a forward whose route queries are registered up front (queries [num_routes, D]), with the
 * logits carried from each route to the next in a table (fp32 [num_routes][T][table_stride]): route `route` takes
 * the logits of bank rows [0, S) from table[route][t][s] and computes only its current source's (`source`); while
 * its mix streams the bank rows it computes the next route's logits of those rows (keys from their inverse RMS in
 * inv_rms [T][inv_stride]) and, when the current source becomes bank row S (append != NULL, or source_in_bank != 0
 * for a source that already is bank row S), of the current source, storing them in table[route + 1]; that source's
 * inverse RMS goes to inv_rms[t][S]. A (source, route) logit depends on nothing else, so the table holds what the
 * reference's route recomputes (same rounding points as zb_attnres_route; the mix sums the terms in source order).
 * Same reference interface as zb_attnres_route (FusedBlockAttnResContext.route over a forward's fixed route order,
 * servers/sgl/src/zonos3_sgl/models/training_attnres.py:59-78).
 *   D a multiple of 256 (at most 4096), S + 1 <= 256, table_stride and inv_stride >= S + (source becomes row S);
 *   bank, source, append, queries, norm_weight, out, mix_out 16-byte aligned. */
int zb_attnres_route_tabled(const uint16_t* bank, int64_t bank_stride, int S, const uint16_t* source,
                            uint16_t* append, int source_in_bank, const uint16_t* queries, int num_routes, int route,
                            float eps, const uint16_t* norm_weight, float norm_eps, uint16_t* out, uint16_t* mix_out,
                            float* table, int64_t table_stride, float* inv_rms, int64_t inv_stride, int T, int D,
                            cudaStream_t stream);

/* ----------------------------------------------------------------------------------------------------- MoE */

/* Fused router: logits = bf16(rmsnorm_eda(x) @ w_router^T), the top-k experts by (float(logit) - bias descending,
 * expert index ascending), and their gate weights: weight_mode 0 = softmax over the k selected logits (the
 * training-router weights), 1 = the selected entries of the softmax over all experts; renormalize != 0 divides by
 * (sum + 1e-8). Replaces Router.forward / _select_balanced_topk (servers/sgl/src/zonos3_sgl/models/zonos3.py:746-828),
 * the router lines of Zonos3LM._feed_forward (model/src/zonos3/reference/lm.py:610-617) and the renormalisation of
 * FusedMoE.forward (servers/sgl/src/zonos3_sgl/layers/moe/fused_moe/layer.py:159-161).
 *   x [T, D] bf16 (row stride x_stride); norm_weight [D] bf16; w_router [E, D] bf16; bias [E] fp32 or NULL
 *   logits_out [T, E] bf16 or NULL; ids [T, k] int32; weights [T, k] fp32.  E <= 128, k <= min(E, 32),
 *   D a multiple of 64. */
int zb_moe_router(const uint16_t* x, int64_t x_stride, const uint16_t* norm_weight, float eps,
                  const uint16_t* w_router, const float* bias, int T, int D, int E, int k, int weight_mode,
                  int renormalize, uint16_t* logits_out, int32_t* ids, float* weights, cudaStream_t stream);

/* The selection and weights of zb_moe_router from given logits [T, E] (fp32, or bf16 if logits_bf16 != 0). */
int zb_moe_select(const void* logits, int logits_bf16, const float* bias, int T, int E, int k, int weight_mode,
                  int renormalize, int32_t* ids, float* weights, cudaStream_t stream);

/* Stable counting sort of the T*k (token, slot) pairs p = t*k + slot by expert, each expert's segment padded to a
 * multiple of `block` rows: counts [E] (the per-expert token histogram), offsets [E+1] (padded segment starts,
 * offsets[E] = rows in use), sorted_pairs [capacity] (pair of each row, -1 for padding and unused rows),
 * position [T*k] (row of each pair). capacity >= roundup(T*k + E*(block-1), block); hist is scratch of
 * ceil(T*k / 256) * E int32 (one expert histogram per 256-pair slice). Replaces moe_align_block_size
 * (servers/sgl/src/zonos3_sgl/layers/moe/fused_moe/fused_moe_impl.py:28-86; sgl_kernel). */
int zb_moe_permute(const int32_t* ids, int T, int k, int E, int block, int64_t capacity, int32_t* hist,
                   int32_t* counts, int32_t* offsets, int32_t* sorted_pairs, int32_t* position, cudaStream_t stream);

/* zb_moe_permute and zb_moe_gather (below) in two launches instead of three: the scatter launch also copies
 * x_perm[position[i]] = x[i / k] for every routed pair (x [T, D] bf16, row stride x_stride; x_perm [capacity, D]
 * bf16, padding rows left as they are). Same outputs as the two calls. Replaces moe_align_block_size plus the row
 * gather of fused_moe_kernel (fused_moe_impl.py:28-86; kernel/triton/fused_moe.py:145). */
int zb_moe_permute_gather(const int32_t* ids, int T, int k, int E, int block, int64_t capacity, int32_t* hist,
                          int32_t* counts, int32_t* offsets, int32_t* sorted_pairs, int32_t* position,
                          const uint16_t* x, int64_t x_stride, int D, uint16_t* x_perm, cudaStream_t stream);

/* out[r] = x[sorted_pairs[r] / k] for r < rows where sorted_pairs[r] >= 0: the A operand of the grouped GEMM, the
 * row gather fused_moe_kernel does through `offs_token // top_k` (servers/sgl/src/zonos3_sgl/kernel/triton/
 * fused_moe.py:145). Padding rows (sorted_pairs[r] < 0) are left as they are: the reference masks them to zero,
 * here the GEMMs compute them row-independently and drop their results, so no output depends on them. */
int zb_moe_gather(const uint16_t* x, int64_t x_stride, const int32_t* sorted_pairs, int k, int64_t rows, int D,
                  uint16_t* out, cudaStream_t stream);

/* GEMM1 of the routed experts on tcgen05 tensor cores, SwiGLU fused in the epilogue:
 * h[r, :] = bf16(silu(bf16(x_perm[r] . gate_up[e, 0:I]^T)) * bf16(x_perm[r] . gate_up[e, I:2I]^T)) for rows r of
 * expert e's segment [offsets[e], offsets[e+1]). Replaces the first fused_moe_kernel call plus silu_and_mul of
 * fused_experts_impl (servers/sgl/src/zonos3_sgl/layers/moe/fused_moe/fused_moe_impl.py:218-234).
 *   x_perm [capacity, D] bf16; gate_up [E, 2I, D] bf16 (gate rows first, zonos3.py:488-490); h [capacity, I] bf16
 *   counts [E] (zb_moe_permute's) or NULL: with counts, decode-sized batches load only each segment's routed rows
 *   (h rows past them hold garbage, like every padding row's).
 *   D a multiple of 64, I a multiple of 128, capacity a multiple of 128. */
int zb_moe_gemm_swiglu(const uint16_t* x_perm, int64_t capacity, const uint16_t* gate_up, int E, int D, int I,
                       const int32_t* offsets, const int32_t* counts, uint16_t* h, cudaStream_t stream);

/* GEMM2 of the routed experts on tcgen05 tensor cores with the routing weight fused:
 * y[p, :] = bf16((h[r] . down[e]^T) * weights[p]) for every row r with pair p = sorted_pairs[r] >= 0.
 * Replaces the second fused_moe_kernel call (MUL_ROUTED_WEIGHT) of fused_experts_impl (fused_moe_impl.py:236-259).
 *   h [capacity, I] bf16; down [E, D, I] bf16; weights [T*k] fp32; y [T*k, D] bf16; counts as for
 *   zb_moe_gemm_swiglu.  I % 64 == 0, D % 128 == 0. */
int zb_moe_gemm_down(const uint16_t* h, int64_t capacity, const uint16_t* down, int E, int D, int I,
                     const int32_t* offsets, const int32_t* counts, const int32_t* sorted_pairs, const float* weights,
                     uint16_t* y, cudaStream_t stream);

/* Both expert GEMMs (zb_moe_gemm_swiglu, then zb_moe_gemm_down on its h) in one call. At decode sizes (the
 * single-CTA shape) they run as one persistent launch: a down tile of expert e starts as soon as every SwiGLU tile of
 * e has stored its h rows, so the SwiGLU GEMM's last partial wave overlaps the down GEMM. flags [E + 1] uint32 are
 * those per-expert counters: zero before the first call, left zero by every call (a bounded wait that expired, status
 * bit 2, may leave them non-zero: re-zero them then). Larger batches make the two pair-shape launches. The grid never
 * exceeds the CTAs the GPU holds at once, which the counters rely on. Replaces both fused_moe_kernel calls of
 * fused_experts_impl (fused_moe_impl.py:218-259). D % 128 == 0, I % 128 == 0. */
int zb_moe_gemms(const uint16_t* x_perm, int64_t capacity, const uint16_t* gate_up, const uint16_t* down, int E,
                 int D, int I, const int32_t* offsets, const int32_t* counts, const int32_t* sorted_pairs,
                 const float* weights, uint16_t* h, uint16_t* y, uint32_t* flags, cudaStream_t stream);

/* out[t, :] = bf16(sum over slots s of float(y[t*k + s, :])): the un-permute combine (the add / moe_sum_reduce of
 * fused_experts_impl, fused_moe_impl.py:267-288). out has row stride out_stride. */
int zb_moe_combine(const uint16_t* y, int T, int k, int D, uint16_t* out, int64_t out_stride, cudaStream_t stream);

/* zb_moe_gemm_down followed by zb_moe_combine, without the caller's [T*k, D] intermediate buffer. No counterpart in
 * the reference: it is for callers that cannot call cudaMalloc (a serving runtime that reserves its device memory
 * at start-up and forbids allocation afterwards, or a C / Go / Java binding with no device allocator of its own).
 * The intermediate rows live in a static device array of 4,194,304 bf16 elements (8 MiB) that every GPU loading the
 * library holds until exit, so T*k*D must be at most 4,194,304 (status 3 otherwise, nothing queued). Calls share
 * the array: each clears the rows it uses first, and calls that overlap on the GPU race. Pair ids in sorted_pairs
 * at or beyond T*k are dropped (sorted_pairs should come from zb_moe_permute with the same T and k). The first call
 * on a device looks up the array's address with that device current; make it before any stream capture. The
 * address is kept per device ordinal for the life of the process (one context per device). Allocates nothing.
 * Arguments as zb_moe_gemm_down (h .. weights; counts NULL loads every row of each tile, the permutation's counts
 * load only the routed rows) and zb_moe_combine (T, k, out, out_stride). */
int zb_moe_down_combine_noalloc(const uint16_t* h, int64_t capacity, const uint16_t* down, int E, int D, int I,
                                const int32_t* offsets, const int32_t* counts, const int32_t* sorted_pairs,
                                const float* weights, int T, int k, uint16_t* out, int64_t out_stride,
                                cudaStream_t stream);

/* ------------------------------------------------------------------------------ GQA decode attention (KV cache) */

/* Copies row i of k and v ([N, Hkv*hd] bf16, row strides k_stride / v_stride) to slot slots[i] of k_cache and
 * v_cache (slot s at s * slot_stride elements; a slot outside [0, num_slots) stores nothing). Replaces MHAKVCache.store_kv /
 * store_cache (servers/sgl/src/zonos3_sgl/kvcache/mha_pool.py:58-67,
 * servers/sgl/src/zonos3_sgl/kernel/csrc/jit/store.cu:28-50). Hkv*hd and the strides multiples of 8; caches, k and v
 * 16-byte aligned. */
int zb_kv_store(uint16_t* k_cache, uint16_t* v_cache, int64_t slot_stride, int64_t num_slots, const int32_t* slots,
                const uint16_t* k, int64_t k_stride, const uint16_t* v, int64_t v_stride, int N, int Hkv, int hd,
                cudaStream_t stream);

/* Decode attention of one query row per request over its cached keys: out[b, h] = softmax(q[b, h] . K^T *
 * softmax_scale) V over the seq_lens[b] positions of request b, whose slots are page_table[b, 0 .. seq_lens[b]);
 * query head h reads KV head h / (Hq / Hkv). Replaces flash_attn_with_kvcache as the FA backend calls it for a decode
 * batch (servers/sgl/src/zonos3_sgl/attention/fa.py:64-81, :171-212; one token per page).
 *   q [B, Hq, hd] bf16 (request stride q_stride); k_cache / v_cache slot s, head g at s * slot_stride + g * hd,
 *   s in [0, num_slots) (a table entry outside that range masks its key position, nothing is read for it);
 *   page_table [B, table_stride] int32 whose first max_seq_len columns are read; seq_lens [B] int32, clamped to
 *   max_seq_len (0, or every key masked: zero output); out [B, Hq, hd] bf16 (out_stride). gate (NULL: none)
 *   [B, Hq] bf16 gate logits, request stride gate_stride: out = bf16(bf16(o) * bf16(sigmoid(gate))), the layer's
 *   output gate (servers/sgl/src/zonos3_sgl/models/zonos3.py:326, :383-385) at torch's rounding points.
 *   The key range of a request is cut into `splits` pieces of split_len positions (a multiple of 32; splits *
 *   split_len must cover the longest seq_len, keys past it are not read); with splits > 1 the partials go to a
 *   workspace of B * Hq * splits * (hd + 2) floats (4-byte each) and a second kernel merges them. The reference
 *   runs this model's decode unsplit (fa.py:41-50), which splits = 1 matches. hd in {32, 64, 128}, Hq / Hkv in
 *   {1, 2, 4, 8}. */
int zb_gqa_decode(const uint16_t* q, int64_t q_stride, const uint16_t* k_cache, const uint16_t* v_cache,
                  int64_t slot_stride, int64_t num_slots, const int32_t* page_table, int64_t table_stride,
                  const int32_t* seq_lens, int max_seq_len, int B, int Hq, int Hkv, int hd, float softmax_scale,
                  int splits, int split_len, float* workspace, int64_t workspace_bytes, uint16_t* out,
                  int64_t out_stride, const uint16_t* gate, int64_t gate_stride, cudaStream_t stream);

/* The attention layer's decode prologue: from the fused projection rows proj [N, Hq*hd | Hkv*hd | Hkv*hd | ...]
 * (q | k | v, row stride proj_stride), q = bf16(RMSNorm(q, eps)) * bf16(|temp|) (rounded), k = bf16(RMSNorm(k, eps)),
 * both rotated by interleaved RoPE at positions[t] (inverse frequency 1 / rope_theta^(2i / hd)); q to q_out
 * [N, Hq, hd], k and v to slot out_loc[t] of the caches (slot stride slot_stride; a slot outside [0, num_slots)
 * stores nothing). Replaces the q/k norm, temperature, rotary and store_kv steps of Attention.forward
 * (servers/sgl/src/zonos3_sgl/models/zonos3.py:340-375). hd = 128; tensors 8-byte aligned, strides multiples of 4. */
int zb_gqa_prologue_decode(const uint16_t* proj, int64_t proj_stride, const uint16_t* temp, const int32_t* positions,
                           float rope_theta, float eps, uint16_t* q_out, uint16_t* k_cache, uint16_t* v_cache,
                           int64_t slot_stride, int64_t num_slots, const int32_t* out_loc, int N, int Hq, int Hkv,
                           int hd, cudaStream_t stream);

/* ---------------------------------------------------------------------------------------------- TTS sampler */

/* Next audio codes from per-codebook logits [B, C, V] (row (b, c) of V at b * batch_stride + c * row_stride elements,
 * so a padded [B, >= C * V] head output can be read in place; bf16 when
 * logits_fp32 == 0, else fp32), one row per (request, codebook): softcap > 0 first applies the head's soft cap
 * softcap * tanh(x / softcap) (MultiOutputHead + softcap, servers/sgl/src/zonos3_sgl/models/zonos3.py:1341-1360,
 * rounded to bf16 after each op for bf16 logits, as torch evaluates it), then invalid ids masked (audio_pad_id; ids >=
 * codebook_size other than stop_ids[b]; ids past codebook_sizes[c] (NULL: codebook_size); the stop id while
 * stop_blocked[b, c] (NULL: never)), stop_bias[b] added to the stop id (NULL: none), repetition penalty
 * rep_penalties[b] over rep_ids[b, c, 0..W) (NULL / W = 0: none), then greedy argmax when `greedy` (every
 * temperature <= 0) or temperature[b], top_k (0 or >= V: off), softmax, top_p (in (0, 1)), min_p (> 0) and one
 * multinomial draw from Philox4x32-10 keyed by `seed` at counter (row, offset + *offset_dev; offset_dev NULL: + 0; a
 * device counter lets a captured decode step draw fresh numbers on each replay). top_k / top_p / min_p are the batch's
 * min / max / max, as the reference reduces them on the host. out [B, C + 1] int32: the codes, then text_vocab.
 * probs_out (NULL: not written) [B * C, V] fp32 receives each row's final distribution. V <= 16384.
 * Replaces sample_tts (model/src/zonos3/tts/sampler.py:159-372; ids drawn from a different random stream than
 * torch.multinomial, equal in distribution). */
int zb_sample_tts(const void* logits, int logits_fp32, float softcap, int64_t row_stride, int64_t batch_stride, int B,
                  int C, int V,
                  const float* temperatures, int greedy, int top_k, float top_p, float min_p, int codebook_size,
                  int audio_pad_id, const int32_t* stop_ids, const int32_t* codebook_sizes, const uint8_t* stop_blocked,
                  const float* stop_bias, const int32_t* rep_ids, int W, const float* rep_penalties, uint64_t seed,
                  uint64_t offset, const uint64_t* offset_dev, int text_vocab, int32_t* out, float* probs_out,
                  cudaStream_t stream);

/* -------------------------------------------------------------------------------------------- input embedding */

/* Input rows of the layer stack: x[t] = RMSNorm(sum over columns c of tables[c][ids[t, c]]; norm_weight, eps)
 * (normalize != 0; else the plain sum). The columns' rows are added one at a time in bf16, each add rounded to bf16,
 * as MultiEmbedding.forward sums them; the norm computes in fp32 and rounds once (norm_weight NULL = weightless, the
 * release's emb_norm). Replaces MultiEmbedding.forward + emb_norm in Zonos3ForCausalLM.embed
 * (servers/sgl/src/zonos3_sgl/models/zonos3.py:225-255, :1066-1070, :1163-1222).
 *   ids        [N, ncols] int32 (device), row stride ids_stride; ncols in 1..16 (codebooks + the text column)
 *   tables     HOST array of ncols device pointers, table c [table_rows[c], D] bf16 contiguous, 16-byte aligned
 *   table_rows HOST array of ncols row counts; an id outside [0, table_rows[c]) reads a zero row and sets status bit
 *              32 (zb_device_status)
 *   out        [N, D] bf16, row stride out_stride (a multiple of 8); D a multiple of 8, at most 4096. */
int zb_embed_norm(const int32_t* ids, int64_t ids_stride, int ncols, const uint16_t* const* tables,
                  const int32_t* table_rows, const uint16_t* norm_weight, float eps, int normalize, int N, int D,
                  uint16_t* out, int64_t out_stride, cudaStream_t stream);

/* The bookkeeping between two captured decode steps, in one single-block launch: ids[b, :ids_cols] = codes[b, ...]
 * (the sampled codes, then the text column, become the next input row), history[b, c, *ring] = codes[b, c] for the
 * first C codebooks (history NULL: none; W columns, *ring the next one), positions[b] += 1, seqlens[b] =
 * min(seqlens[b] + 1, max_len), out_loc[b] = page_table[b, seqlens[b] - 1]; then *ring = (*ring + 1) % W and
 * *counter += 1 (the sampler's draw counter). The engine does this on the host between steps (the scheduler builds
 * the next batch's ids and attention metadata); here it stays on the device so that replays alone decode. No
 * reference counterpart as a kernel. */
int zb_decode_advance(const int32_t* codes, int codes_cols, int32_t* ids, int ids_cols, int32_t* history, int C, int W,
                      int64_t* ring, int64_t* counter, int32_t* positions, int32_t* seqlens, int32_t* out_loc,
                      const int32_t* page_table, int64_t table_stride, int max_len, int B, cudaStream_t stream);

/* ------------------------------------------------------------------------- codec DSP tail (iSTFT head, resampler) */

/* Twiddle table out[e] = (cos, sin)(2 pi e / n), e in [0, n), interleaved float64 (16-byte aligned); 2 <= n <= 8192.
 * The head stream builds one per branch once (no reference counterpart: torch.fft.irfft plans its own). */
int zb_istft_twiddles(int n, double* out, cudaStream_t stream);

/* One push of the two-branch centred iSTFT head + FIR mixer for `streams` lock-step streams, or its flush
 * (IstftHeadStream.push / .flush, model/src/zonos3/codec/stream_host.py:39-101 and the torch twin
 * stream_device.py:58-124; float64 arithmetic, float32 output).
 *   y0, y1        [streams, cols, n_b + 2] float32 (y_is_f64 == 0) or float64, each stream's frames contiguous rows
 *                 and streams y_b_stride elements apart: per frame the log-magnitude of n_b/2 + 1 bins (clamped at
 *                 max_log_mag before exp), then the phase
 *   window_b      [n_b] float64; twiddle_b the zb_istft_twiddles table of n_b; mixer [2, taps] float64, taps odd
 *   carry_b       [2, streams, n_b - hop] float64: overlap-add sums carried between pushes; half carry_parity holds
 *                 the current carry and the push writes the next one into the other half (the caller flips the parity
 *                 after each push); zero before the first push
 *   ring_b        [streams, ring_size] float64 mixer-input history (power-of-two size, zero before the first push)
 *   frames_before head frames pushed before this call; mix_from / mix_to the mixer outputs to emit (the caller's
 *                 stream position and the reference's emission bound); flush: cols == 0, mix_to = frames * hop
 *   scratch       float64, streams * cols * (n0 + n1) elements always suffice: the synthesised frames, or for a push
 *                 of 32 frames or more with an even hop (n_b <= 17 hop) the overlap-add spans of its 16-frame groups,
 *                 which the frame kernels add up themselves (then less is enough: 2 * streams * (cols / 16) *
 *                 (31 hop + max(n) - hop) elements); out [streams, mix_to - mix_from] float32.
 * n_b even, a multiple of hop with n_b / hop >= 2, n_b <= 8192. */
int zb_istft_head_push(const void* y0, int64_t y0_stride, const void* y1, int64_t y1_stride, int y_is_f64,
                       int streams, int cols, int n0, int n1, int hop,
                       const double* window0, const double* window1, const double* twiddle0, const double* twiddle1,
                       double max_log_mag, const double* mixer, int taps, double* carry0, double* carry1,
                       int carry_parity, double* ring0, double* ring1, int ring_size, int64_t frames_before,
                       int64_t mix_from, int64_t mix_to, int flush, double* scratch, int64_t scratch_elems, float* out,
                       cudaStream_t stream);

/* One push (count > 0) or flush (count == 0) of the polyphase sinc resampler for `streams` lock-step streams
 * (ResamplerStream.push / .flush, model/src/zonos3/codec/stream_host.py:136-171, stream_device.py:169-197):
 * x [streams, count] (row stride x_stride; float32, or float64 when x_is_f64) is appended to the input ring
 * [streams, ring_size] float64 (power-of-two size) at n_in_before, then blocks [block_from, block_to) are emitted:
 * out[s, (b - block_from) * new + i] = sum_k kernel[i][k] * x[b * orig + k - width], inputs outside [0, n_in) zero,
 * the first out_count per stream (out [streams, out_count] float32). kernel_t is the kernel transposed, [2 * width +
 * orig, new] float64. workspace (16-byte aligned float64, or NULL) lets a call with few (stream, block) pairs split
 * the taps over more CTAs: up to 8 * streams * (block_to - block_from) * new elements are used; the slices are summed
 * in a fixed order, so the output does not depend on the split. */
int zb_resample_push(const void* x, int x_is_f64, int64_t x_stride, int streams, int count, double* ring,
                     int ring_size, int64_t n_in_before, const double* kernel_t, int orig, int new_freq, int width,
                     int64_t block_from, int64_t block_to, int64_t out_count, float* out, double* workspace,
                     int64_t workspace_elems, cudaStream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* ZONOS3_B200_H_ */

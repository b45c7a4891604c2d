"""Thin torch-facing wrappers over the C-ABI entry points.

Each wrapper validates shapes, dtypes and devices (raising ``ValueError`` the way the reference's layers do), then
passes raw device pointers, strides and the current CUDA stream to ``libzonos3_b200.so``. Outputs are written into
caller-provided tensors when given, so a wrapper allocates nothing inside a CUDA-graph capture.
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _require(cond: bool, msg: str) -> None:
    if not cond:
        raise ValueError(msg)


def _check_cuda(name: str, t: torch.Tensor, dtype: torch.dtype, device: torch.device | None = None) -> None:
    _require(isinstance(t, torch.Tensor), f"{name} must be a tensor")
    _require(t.is_cuda, f"{name} must be a CUDA tensor (the B200 kernels have no CPU path)")
    _require(t.dtype == dtype, f"{name} must be {dtype}, got {t.dtype}")
    if device is not None:
        _require(t.device == device, f"{name} is on {t.device}, expected {device}")


def _rows(name: str, t: torch.Tensor, inner: tuple[int, ...]) -> int:
    """Batch stride (elements) of a [B, *inner] tensor whose inner block is contiguous."""
    _require(tuple(t.shape[1:]) == inner, f"{name} must have shape [B, {', '.join(map(str, inner))}], got {tuple(t.shape)}")
    expected = 1
    for dim in range(t.dim() - 1, 0, -1):
        _require(t.stride(dim) == expected, f"{name} must be contiguous within a row")
        expected *= t.shape[dim]
    return t.stride(0) if t.shape[0] > 1 else expected


# --------------------------------------------------------------------------------------------- gated DeltaNet


def gdn_decode_step(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    g: torch.Tensor,
    beta: torch.Tensor,
    state: torch.Tensor,
    out: torch.Tensor | None = None,
    *,
    scale: float | None = None,
    slots: torch.Tensor | None = None,
) -> torch.Tensor:
    """One recurrent gated-delta-rule step per stream (model/src/zonos3/reference/lm.py:576-582).

    q, k: [B, H, dk] bf16 (L2-normalised); v: [B, H, dv] bf16; g: [B, H] fp32 log-decay (decay = exp(g));
    beta: [B, H] fp32; state: [slots, H, dv, dk] fp32, V-first like FLA's ``state_v_first`` and the reference
    ``LMCache.gdn_state``, updated in place; slots: optional [B] int64 state row per stream (negative = padding row,
    its output is zero and no state is touched). Returns out [B, H, dv] bf16 = S_new (q * scale).
    """
    dev = q.device
    _check_cuda("q", q, torch.bfloat16)
    B, H, dk = q.shape
    dv = v.shape[-1]
    for name, t, dt in (("k", k, torch.bfloat16), ("v", v, torch.bfloat16), ("g", g, torch.float32),
                        ("beta", beta, torch.float32), ("state", state, torch.float32)):
        _check_cuda(name, t, dt, dev)
    qs = _rows("q", q, (H, dk))
    ks = _rows("k", k, (H, dk))
    vs = _rows("v", v, (H, dv))
    gs = _rows("g", g, (H,))
    _require(beta.shape == g.shape and beta.stride() == g.stride(), "beta must match g's shape and strides")
    _require(state.dim() == 4 and tuple(state.shape[1:]) == (H, dv, dk) and state.is_contiguous(),
             f"state must be a contiguous [slots, {H}, {dv}, {dk}] tensor, got {tuple(state.shape)}")
    if slots is None:
        _require(state.shape[0] >= B, "state has fewer slots than streams")
        slot_ptr = None
    else:
        _check_cuda("slots", slots, torch.int64, dev)
        _require(slots.shape == (B,) and slots.is_contiguous(), "slots must be a contiguous [B] int64 tensor")
        slot_ptr = slots.data_ptr()
    if out is None:
        out = torch.empty((B, H, dv), device=dev, dtype=torch.bfloat16)
    _check_cuda("out", out, torch.bfloat16, dev)
    os_ = _rows("out", out, (H, dv))
    if scale is None:
        scale = dk ** -0.5
    _lib.call(
        "zb_gdn_decode_step",
        q.data_ptr(), k.data_ptr(), v.data_ptr(), qs, ks, vs,
        g.data_ptr(), beta.data_ptr(), gs, state.data_ptr(), slot_ptr, state.shape[0],
        out.data_ptr(), os_, B, H, dk, dv, float(scale), _stream(dev),
    )
    return out


# --------------------------------------------------------------------------------------------- Full AttnRes


def attnres_route(
    bank: torch.Tensor | None,
    num_sources: int,
    query: torch.Tensor,
    eps: float,
    *,
    source: torch.Tensor | None = None,
    append_to: torch.Tensor | None = None,
    norm_weight: torch.Tensor | None = None,
    norm_eps: float = 1e-5,
    out: torch.Tensor | None = None,
    mix_out: torch.Tensor | None = None,
    rms_cache: torch.Tensor | None = None,
    cached: int = 0,
) -> torch.Tensor:
    """Full AttnRes route over ``bank[:num_sources]`` (+ ``source`` as the last source) for every token.

    bank [>= num_sources, T, D] bf16 (rows contiguous [T, D]); source [T, D] bf16; query [D] bf16. The mix follows
    full_attnres_route (model/src/zonos3/reference/lm.py:384-389) with the fused Triton kernel's bf16 rounding
    points. ``norm_weight`` fuses the RMSNorm after the route (out = RMSNorm(mix) and, if given, mix_out = mix);
    ``append_to`` (a [T, D] bank row) receives ``source`` in the same pass. ``rms_cache`` (fp32 [>= T, >= sources
    rounded up to 4], token-major) holds each source's key inverse RMS: sources below ``cached`` are read, the
    others computed and stored.
    """
    _check_cuda("query", query, torch.bfloat16)
    dev = query.device
    (D,) = query.shape
    T = None
    bank_stride = 0
    if num_sources:
        _check_cuda("bank", bank, torch.bfloat16, dev)
        _require(bank.dim() == 3 and bank.shape[0] >= num_sources and bank.shape[2] == D,
                 f"bank must be [>= {num_sources}, T, {D}], got {tuple(bank.shape)}")
        _require(bank.stride(2) == 1 and bank.stride(1) == D, "bank rows must be contiguous [T, D]")
        T = bank.shape[1]
        bank_stride = bank.stride(0)
    if source is not None:
        _check_cuda("source", source, torch.bfloat16, dev)
        _require(source.dim() == 2 and source.shape[1] == D and source.is_contiguous(),
                 f"source must be a contiguous [T, {D}] tensor")
        _require(T is None or source.shape[0] == T, "source rows differ from the bank's")
        T = source.shape[0]
    _require(T is not None, "nothing to route: no bank sources and no source")
    if append_to is not None:
        _require(source is not None, "append_to needs a source")
        _check_cuda("append_to", append_to, torch.bfloat16, dev)
        _require(append_to.shape == (T, D) and append_to.is_contiguous(), "append_to must be a contiguous [T, D] row")
    if norm_weight is not None:
        _check_cuda("norm_weight", norm_weight, torch.bfloat16, dev)
        _require(norm_weight.shape == (D,), "norm_weight must be [D]")
    if out is None:
        out = torch.empty((T, D), device=dev, dtype=torch.bfloat16)
    for name, t in (("out", out), ("mix_out", mix_out)):
        if t is not None:
            _check_cuda(name, t, torch.bfloat16, dev)
            _require(t.shape == (T, D) and t.is_contiguous(), f"{name} must be a contiguous [T, D] tensor")
    _require(mix_out is None or norm_weight is not None, "mix_out is only produced with norm_weight")
    rms_stride = 0
    if rms_cache is not None:
        _check_cuda("rms_cache", rms_cache, torch.float32, dev)
        routed = num_sources + (source is not None)
        need = (routed + 3) // 4 * 4
        _require(rms_cache.dim() == 2 and rms_cache.shape[0] >= T and rms_cache.shape[1] >= need
                 and rms_cache.stride(1) == 1 and rms_cache.stride(0) % 4 == 0,
                 f"rms_cache must be [>= {T}, >= {need}] with unit column stride and a row stride multiple of 4")
        _require(0 <= cached <= num_sources, f"cached must be in [0, {num_sources}]")
        rms_stride = rms_cache.stride(0)
    else:
        cached = 0
    ptr = lambda t: None if t is None else t.data_ptr()  # noqa: E731
    _lib.call(
        "zb_attnres_route",
        ptr(bank) if num_sources else None, bank_stride, num_sources, ptr(source), ptr(append_to),
        query.data_ptr(), float(eps), ptr(norm_weight), float(norm_eps), out.data_ptr(), ptr(mix_out),
        ptr(rms_cache), rms_stride, int(cached), T, D, _stream(dev),
    )
    return out


def attnres_route_tabled(
    bank: torch.Tensor | None,
    num_sources: int,
    source: torch.Tensor,
    queries: torch.Tensor,
    route: int,
    table: torch.Tensor,
    inv_rms: torch.Tensor,
    eps: float,
    *,
    source_in_bank: bool = False,
    append_to: torch.Tensor | None = None,
    norm_weight: torch.Tensor | None = None,
    norm_eps: float = 1e-5,
    out: torch.Tensor | None = None,
    mix_out: torch.Tensor | None = None,
) -> torch.Tensor:
    """Route ``route`` of a forward whose route queries (``queries`` [R, D] bf16) are registered up front, over
    ``bank[:num_sources]`` + ``source`` (the current source).

    ``table`` (fp32 [R, T, >= sources]) carries the logits from route to route: this route reads its rows'
    logits from ``table[route]`` and, while it mixes, writes the next route's logits of the same rows and, when
    the source becomes bank row ``num_sources`` (``append_to`` given, or ``source_in_bank`` for a source that
    already is that row), of the source, to ``table[route + 1]``. ``inv_rms`` (fp32 [>= T, >= sources]) holds the
    bank rows' key inverse RMS; the source's is stored at column ``num_sources`` when it becomes that row. Same mix,
    rounding points, fused RMSNorm and append as :func:`attnres_route`.
    """
    _check_cuda("queries", queries, torch.bfloat16)
    dev = queries.device
    _require(queries.dim() == 2 and queries.is_contiguous(), "queries must be a contiguous [R, D] tensor")
    R, D = queries.shape
    _require(0 <= route < R, f"route {route} outside [0, {R})")
    _check_cuda("source", source, torch.bfloat16, dev)
    _require(source.dim() == 2 and source.shape[1] == D and source.is_contiguous(),
             f"source must be a contiguous [T, {D}] tensor")
    T = source.shape[0]
    bank_stride = 0
    if num_sources:
        _check_cuda("bank", bank, torch.bfloat16, dev)
        _require(bank.dim() == 3 and bank.shape[0] >= num_sources and bank.shape[1] == T and bank.shape[2] == D,
                 f"bank must be [>= {num_sources}, {T}, {D}], got {tuple(bank.shape)}")
        _require(bank.stride(2) == 1 and bank.stride(1) == D, "bank rows must be contiguous [T, D]")
        bank_stride = bank.stride(0)
    _require(not (source_in_bank and append_to is not None), "a source already in the bank is not appended")
    need = num_sources + (1 if source_in_bank or append_to is not None else 0)
    _check_cuda("table", table, torch.float32, dev)
    _require(table.dim() == 3 and table.shape[0] == R and table.shape[1] == T and table.shape[2] >= need
             and table.is_contiguous(), f"table must be a contiguous [{R}, {T}, >= {need}] tensor")
    _check_cuda("inv_rms", inv_rms, torch.float32, dev)
    _require(inv_rms.dim() == 2 and inv_rms.shape[0] >= T and inv_rms.shape[1] >= need and inv_rms.stride(1) == 1,
             f"inv_rms must be [>= {T}, >= {need}] with unit column stride")
    if append_to is not None:
        _check_cuda("append_to", append_to, torch.bfloat16, dev)
        _require(append_to.shape == (T, D) and append_to.is_contiguous(), "append_to must be a contiguous [T, D] row")
    if norm_weight is not None:
        _check_cuda("norm_weight", norm_weight, torch.bfloat16, dev)
        _require(norm_weight.shape == (D,), "norm_weight must be [D]")
    if out is None:
        out = torch.empty((T, D), device=dev, dtype=torch.bfloat16)
    for name, t in (("out", out), ("mix_out", mix_out)):
        if t is not None:
            _check_cuda(name, t, torch.bfloat16, dev)
            _require(t.shape == (T, D) and t.is_contiguous(), f"{name} must be a contiguous [T, D] tensor")
    _require(mix_out is None or norm_weight is not None, "mix_out is only produced with norm_weight")
    ptr = lambda t: None if t is None else t.data_ptr()  # noqa: E731
    _lib.call(
        "zb_attnres_route_tabled",
        ptr(bank) if num_sources else None, bank_stride, num_sources, source.data_ptr(), ptr(append_to),
        int(bool(source_in_bank)), queries.data_ptr(), R, int(route), float(eps), ptr(norm_weight), float(norm_eps),
        out.data_ptr(), ptr(mix_out), table.data_ptr(), table.shape[2], inv_rms.data_ptr(), inv_rms.stride(0), T, D,
        _stream(dev),
    )
    return out


def device_status(clear: bool = True) -> int:
    """Bits set by kernels whose bounded device-side waits expired on the current device (synchronous)."""
    import ctypes

    flags = ctypes.c_uint(0)
    _lib.call("zb_device_status", ctypes.byref(flags), int(clear))
    return flags.value


# --------------------------------------------------------------------------------------------- MoE

WEIGHT_MODES = {"selected_softmax": 0, "full_softmax": 1}
GEMM_BLOCK = 128  # rows of one grouped-GEMM tile; every expert segment is padded to a multiple of it


def moe_capacity(tokens: int, top_k: int, num_experts: int, block: int = GEMM_BLOCK) -> int:
    """Rows of the permuted, tile-padded pair layout: enough for any routing of ``tokens * top_k`` pairs."""
    pairs = tokens * top_k
    return -(-(pairs + num_experts * (block - 1)) // block) * block


def moe_router(x, norm_weight, eps, w_router, bias, top_k, *, weights="selected_softmax", renormalize=False,
               ids=None, topk_weights=None, logits=None):
    """Fused router: logits = router_linear(rmsnorm_eda(x)) (bf16), top-k by (logit - bias, index), gate weights.

    x [T, D] bf16; norm_weight [D] bf16; w_router [E, D] bf16; bias [E] fp32. Returns (ids [T, k] int32,
    weights [T, k] fp32); ``logits`` ([T, E] bf16) optionally receives the router logits.
    Follows servers/sgl/src/zonos3_sgl/models/zonos3.py:787-828 and model/src/zonos3/reference/lm.py:610-617.
    """
    _check_cuda("x", x, torch.bfloat16)
    dev = x.device
    T, D = x.shape
    _require(x.stride(1) == 1, "x rows must be contiguous")
    _check_cuda("w_router", w_router, torch.bfloat16, dev)
    E = w_router.shape[0]
    _require(w_router.shape == (E, D) and w_router.is_contiguous(), "w_router must be a contiguous [E, D] tensor")
    _check_cuda("norm_weight", norm_weight, torch.bfloat16, dev)
    _require(norm_weight.shape == (D,), "norm_weight must be [D]")
    if bias is not None:
        _check_cuda("bias", bias, torch.float32, dev)
        _require(bias.shape == (E,), "bias must be [E]")
    if ids is None:
        ids = torch.empty((T, top_k), device=dev, dtype=torch.int32)
    if topk_weights is None:
        topk_weights = torch.empty((T, top_k), device=dev, dtype=torch.float32)
    _check_cuda("ids", ids, torch.int32, dev)
    _check_cuda("topk_weights", topk_weights, torch.float32, dev)
    _require(ids.shape == (T, top_k) and ids.is_contiguous(), "ids must be a contiguous [T, k] int32 tensor")
    _require(topk_weights.shape == (T, top_k) and topk_weights.is_contiguous(), "topk_weights must be [T, k]")
    if logits is not None:
        _check_cuda("logits", logits, torch.bfloat16, dev)
        _require(logits.shape == (T, E) and logits.is_contiguous(), "logits must be a contiguous [T, E] tensor")
    _lib.call("zb_moe_router", x.data_ptr(), x.stride(0) if T > 1 else D, norm_weight.data_ptr(), float(eps),
              w_router.data_ptr(), None if bias is None else bias.data_ptr(), T, D, E, top_k,
              WEIGHT_MODES[weights], int(bool(renormalize)), None if logits is None else logits.data_ptr(),
              ids.data_ptr(), topk_weights.data_ptr(), _stream(dev))
    return ids, topk_weights


def moe_select(logits, bias, top_k, *, weights="selected_softmax", renormalize=False, ids=None, topk_weights=None):
    """Top-k selection and gate weights from given router logits [T, E] (fp32 or bf16); same contract as
    ``moe_router`` (used to check selection parity on identical logits)."""
    _require(logits.is_cuda and logits.dtype in (torch.float32, torch.bfloat16) and logits.is_contiguous(),
             "logits must be a contiguous CUDA fp32/bf16 [T, E] tensor")
    dev = logits.device
    T, E = logits.shape
    if bias is not None:
        _check_cuda("bias", bias, torch.float32, dev)
        _require(bias.shape == (E,), "bias must be [E]")
    if ids is None:
        ids = torch.empty((T, top_k), device=dev, dtype=torch.int32)
    if topk_weights is None:
        topk_weights = torch.empty((T, top_k), device=dev, dtype=torch.float32)
    _lib.call("zb_moe_select", logits.data_ptr(), int(logits.dtype == torch.bfloat16),
              None if bias is None else bias.data_ptr(), T, E, top_k, WEIGHT_MODES[weights], int(bool(renormalize)),
              ids.data_ptr(), topk_weights.data_ptr(), _stream(dev))
    return ids, topk_weights


PERMUTE_SLICE = 256  # pairs per CTA of the permutation kernels


def permute_hist_size(pairs: int, num_experts: int) -> int:
    """int32 elements of the permutation's scratch (one expert histogram per 256-pair slice)."""
    return max(1, -(-pairs // PERMUTE_SLICE)) * num_experts


def moe_permute(ids, num_experts, *, block=GEMM_BLOCK, capacity=None, out=None):
    """Stable sort of the (token, slot) pairs by expert, segments padded to ``block`` rows.

    Returns dict(counts [E], offsets [E+1], sorted_pairs [capacity] (-1 = padding), position [T*k], hist (scratch))
    as int32 device tensors; ``out`` may supply them (graph-safe reuse)."""
    _check_cuda("ids", ids, torch.int32)
    dev = ids.device
    T, k = ids.shape
    _require(ids.is_contiguous(), "ids must be contiguous")
    if capacity is None:
        capacity = moe_capacity(T, k, num_experts, block)
    if out is None:
        out = {
            "counts": torch.empty(num_experts, device=dev, dtype=torch.int32),
            "offsets": torch.empty(num_experts + 1, device=dev, dtype=torch.int32),
            "sorted_pairs": torch.empty(capacity, device=dev, dtype=torch.int32),
            "position": torch.empty(T * k, device=dev, dtype=torch.int32),
            "hist": torch.empty(permute_hist_size(T * k, num_experts), device=dev, dtype=torch.int32),
        }
    _require(out["hist"].numel() >= permute_hist_size(T * k, num_experts), "permutation scratch too small")
    _lib.call("zb_moe_permute", ids.data_ptr(), T, k, num_experts, block, capacity, out["hist"].data_ptr(),
              out["counts"].data_ptr(),
              out["offsets"].data_ptr(), out["sorted_pairs"].data_ptr(), out["position"].data_ptr(), _stream(dev))
    return out


def moe_permute_gather(ids, num_experts, x, x_perm, *, block=GEMM_BLOCK, capacity=None, out=None):
    """:func:`moe_permute` with :func:`moe_gather` folded into its scatter launch: also writes x_perm[position[i]] =
    x[i // k] for every routed pair (padding rows untouched). Returns the permutation dict."""
    _check_cuda("ids", ids, torch.int32)
    dev = ids.device
    T, k = ids.shape
    _require(ids.is_contiguous(), "ids must be contiguous")
    _check_cuda("x", x, torch.bfloat16, dev)
    _check_cuda("x_perm", x_perm, torch.bfloat16, dev)
    D = x.shape[1]
    _require(x.dim() == 2 and x.shape[0] == T and x.stride(1) == 1, "x must be [T, D] with contiguous rows")
    _require(x_perm.is_contiguous() and x_perm.shape[1] == D, "x_perm must be a contiguous [capacity, D] buffer")
    if capacity is None:
        capacity = moe_capacity(T, k, num_experts, block)
    _require(x_perm.shape[0] >= capacity, "x_perm has fewer rows than the capacity")
    if out is None:
        out = {
            "counts": torch.empty(num_experts, device=dev, dtype=torch.int32),
            "offsets": torch.empty(num_experts + 1, device=dev, dtype=torch.int32),
            "sorted_pairs": torch.empty(capacity, device=dev, dtype=torch.int32),
            "position": torch.empty(T * k, device=dev, dtype=torch.int32),
            "hist": torch.empty(permute_hist_size(T * k, num_experts), device=dev, dtype=torch.int32),
        }
    _require(out["hist"].numel() >= permute_hist_size(T * k, num_experts), "permutation scratch too small")
    _lib.call("zb_moe_permute_gather", ids.data_ptr(), T, k, num_experts, block, capacity, out["hist"].data_ptr(),
              out["counts"].data_ptr(), out["offsets"].data_ptr(), out["sorted_pairs"].data_ptr(),
              out["position"].data_ptr(), x.data_ptr(), x.stride(0) if T > 1 else D, D, x_perm.data_ptr(),
              _stream(dev))
    return out


def moe_gather(x, sorted_pairs, top_k, out):
    """out[r] = x[sorted_pairs[r] // k] for live rows; padding rows (sorted_pairs < 0) are left as they are."""
    dev = x.device
    _check_cuda("x", x, torch.bfloat16)
    _check_cuda("out", out, torch.bfloat16, dev)
    _require(out.shape == (sorted_pairs.shape[0], x.shape[1]) and out.is_contiguous(), "out must be [rows, D]")
    _lib.call("zb_moe_gather", x.data_ptr(), x.stride(0), sorted_pairs.data_ptr(), top_k, out.shape[0], x.shape[1],
              out.data_ptr(), _stream(dev))
    return out


def moe_gemm_swiglu(x_perm, gate_up, offsets, out, counts=None):
    """H = SwiGLU(x_perm @ gate_up[e].T) per expert segment (tcgen05 grouped GEMM, gate rows first). ``counts``
    (the permutation's routed rows per expert) lets decode-sized batches skip the padding rows' loads."""
    dev = x_perm.device
    E, two_i, D = gate_up.shape
    for name, t in (("x_perm", x_perm), ("gate_up", gate_up), ("out", out)):
        _check_cuda(name, t, torch.bfloat16, dev)
        _require(t.is_contiguous(), f"{name} must be contiguous")
    _require(x_perm.shape[1] == D and out.shape == (x_perm.shape[0], two_i // 2), "shape mismatch")
    _lib.call("zb_moe_gemm_swiglu", x_perm.data_ptr(), x_perm.shape[0], gate_up.data_ptr(), E, D, two_i // 2,
              offsets.data_ptr(), None if counts is None else counts.data_ptr(), out.data_ptr(), _stream(dev))
    return out


def moe_gemm_down(h, down, offsets, sorted_pairs, topk_weights, out, counts=None):
    """Y[pair] = (H[r] @ down[e].T) * weight[pair] for every non-padding row r (tcgen05 grouped GEMM); ``counts``
    as for :func:`moe_gemm_swiglu`."""
    dev = h.device
    E, D, I = down.shape
    for name, t in (("h", h), ("down", down), ("out", out)):
        _check_cuda(name, t, torch.bfloat16, dev)
        _require(t.is_contiguous(), f"{name} must be contiguous")
    _check_cuda("topk_weights", topk_weights, torch.float32, dev)
    _require(h.shape[1] == I and out.shape == (topk_weights.numel(), D), "shape mismatch")
    _lib.call("zb_moe_gemm_down", h.data_ptr(), h.shape[0], down.data_ptr(), E, D, I, offsets.data_ptr(),
              None if counts is None else counts.data_ptr(), sorted_pairs.data_ptr(), topk_weights.data_ptr(),
              out.data_ptr(), _stream(dev))
    return out


def moe_gemms(x_perm, gate_up, down, offsets, sorted_pairs, topk_weights, h, y, flags, counts=None):
    """Both grouped GEMMs of the experts: H = SwiGLU(x_perm @ gate_up[e].T), then Y[pair] = (H @ down[e].T) * w.
    Decode-sized batches run them as one persistent launch, a down tile of expert e starting as soon as every
    SwiGLU tile of e has stored its H rows; ``flags`` ([E + 1] int32, zero before the first call, left zero) are
    those per-expert counters. Larger batches run the two launches of :func:`moe_gemm_swiglu` /
    :func:`moe_gemm_down`."""
    dev = x_perm.device
    E, two_i, D = gate_up.shape
    I = two_i // 2
    for name, t in (("x_perm", x_perm), ("gate_up", gate_up), ("down", down), ("h", h), ("y", y)):
        _check_cuda(name, t, torch.bfloat16, dev)
        _require(t.is_contiguous(), f"{name} must be contiguous")
    _check_cuda("topk_weights", topk_weights, torch.float32, dev)
    _check_cuda("flags", flags, torch.int32, dev)
    _require(tuple(down.shape) == (E, D, I) and x_perm.shape[1] == D and h.shape == (x_perm.shape[0], I)
             and y.shape == (topk_weights.numel(), D) and flags.numel() >= E + 1, "shape mismatch")
    _lib.call("zb_moe_gemms", x_perm.data_ptr(), x_perm.shape[0], gate_up.data_ptr(), down.data_ptr(), E, D, I,
              offsets.data_ptr(), None if counts is None else counts.data_ptr(), sorted_pairs.data_ptr(),
              topk_weights.data_ptr(), h.data_ptr(), y.data_ptr(), flags.data_ptr(), _stream(dev))
    return y


def moe_combine(y, top_k, out):
    """out[t] = sum over slots of y[t * k + slot] (fp32 sum, bf16 result)."""
    dev = y.device
    _check_cuda("y", y, torch.bfloat16)
    _check_cuda("out", out, torch.bfloat16, dev)
    T, D = out.shape
    _require(y.shape == (T * top_k, D) and y.is_contiguous() and out.stride(1) == 1, "shape mismatch")
    _lib.call("zb_moe_combine", y.data_ptr(), T, top_k, D, out.data_ptr(), out.stride(0) if T > 1 else D,
              _stream(dev))
    return out


class MoEWorkspace:
    """Device buffers of one MoE call shape (tokens, top-k, experts, hidden, intermediate), allocated once and
    reused, so repeated calls and CUDA-graph captures allocate nothing."""

    def __init__(self, tokens, top_k, num_experts, hidden, intermediate, device):
        self.key = (tokens, top_k, num_experts, hidden, intermediate, torch.device(device))
        cap = moe_capacity(tokens, top_k, num_experts)
        self.capacity = cap
        i32 = dict(device=device, dtype=torch.int32)
        bf = dict(device=device, dtype=torch.bfloat16)
        self.ids = torch.empty(tokens, top_k, **i32)
        self.weights = torch.empty(tokens, top_k, device=device, dtype=torch.float32)
        self.perm = {
            "counts": torch.empty(num_experts, **i32),
            "offsets": torch.empty(num_experts + 1, **i32),
            "sorted_pairs": torch.empty(cap, **i32),
            "position": torch.empty(tokens * top_k, **i32),
            "hist": torch.empty(permute_hist_size(tokens * top_k, num_experts), **i32),
        }
        self.x_perm = torch.empty(cap, hidden, **bf)
        self.h = torch.empty(cap, intermediate, **bf)
        self.y = torch.empty(tokens * top_k, hidden, **bf)
        self.flags = torch.zeros(num_experts + 1, **i32)  # moe_gemms' per-expert counters (left zero by it)

    @classmethod
    def for_shape(cls, cache: dict, tokens, top_k, num_experts, hidden, intermediate, device):
        key = (tokens, top_k, num_experts, hidden, intermediate, torch.device(device))
        ws = cache.get(key)
        if ws is None:
            ws = cache[key] = cls(tokens, top_k, num_experts, hidden, intermediate, device)
        return ws


def moe_experts(x, gate_up, down, ids, topk_weights, workspace: MoEWorkspace, out=None):
    """Routed SwiGLU experts for precomputed (ids, weights): permute + gather (count, then scatter with the row copies)
    -> GEMM1+SwiGLU -> GEMM2*w (one launch at decode sizes) -> combine. x [T, D] bf16; gate_up [E, 2I, D]; down [E, D, I]. Returns out [T, D] bf16."""
    T, D = x.shape
    E = gate_up.shape[0]
    k = ids.shape[1]
    ws = workspace
    perm = moe_permute_gather(ids, E, x, ws.x_perm, capacity=ws.capacity, out=ws.perm)
    moe_gemms(ws.x_perm, gate_up, down, perm["offsets"], perm["sorted_pairs"], topk_weights, ws.h, ws.y, ws.flags,
              counts=perm["counts"])
    if out is None:
        out = torch.empty((T, D), device=x.device, dtype=torch.bfloat16)
    return moe_combine(ws.y, k, out)


def gdn_chunk_prefill_workspace_bytes(total_tokens: int, num_seqs: int, heads: int, head_dim: int) -> int:
    """Bytes of device workspace ``gdn_chunk_prefill`` needs (0 for head_dim 64): one 33 KB record of the chunk
    preparation (T, P, decays) per (chunk, head)."""
    return int(_lib.load().zb_gdn_chunk_prefill_workspace_bytes(int(total_tokens), int(num_seqs), int(heads),
                                                                int(head_dim)))


def gdn_chunk_prefill(q, k, v, g, beta, cu_seqlens, *, initial_state=None, output_final_state=True, scale=None,
                      state_slots=None, final_state=None, out=None, workspace=None):
    """Chunked (C = 64) gated delta rule over packed variable-length sequences, fp32 state.

    The call FLA's chunk_gated_delta_rule_fwd makes for OriginalGDN._run_packed
    (servers/sgl/src/zonos3_sgl/models/gdn.py:418-434), with the per-token math of
    model/src/zonos3/reference/lm.py:576-582. q, k [N, H, d] bf16 (L2-normalised), v [N, H, d] bf16, g / beta
    [N, H] fp32 (g = log decay), cu_seqlens [n+1] int32 (device). initial_state / final_state [n or slots, H, d, d]
    fp32 V-first (``state_slots`` [n] int64 maps sequence i to a state row). ``workspace``: optional uint8 device
    buffer of at least ``gdn_chunk_prefill_workspace_bytes(N, n, H, d)`` bytes (allocated per call when absent).
    Returns (out [N, H, d] bf16, final_state or None)."""
    _check_cuda("q", q, torch.bfloat16)
    dev = q.device
    N, H, dk = q.shape
    dv = v.shape[-1]
    for name, t in (("k", k), ("v", v)):
        _check_cuda(name, t, torch.bfloat16, dev)
        _require(t.is_contiguous() and t.shape[:2] == (N, H), f"{name} must be a contiguous [N, H, d] tensor")
    _require(q.is_contiguous(), "q must be contiguous")
    for name, t in (("g", g), ("beta", beta)):
        _check_cuda(name, t, torch.float32, dev)
        _require(t.shape == (N, H) and t.is_contiguous(), f"{name} must be a contiguous [N, H] tensor")
    _check_cuda("cu_seqlens", cu_seqlens, torch.int32, dev)
    n = cu_seqlens.numel() - 1
    _require(n >= 0 and cu_seqlens.is_contiguous(), "cu_seqlens must be a contiguous [n + 1] tensor")
    rows = n
    if state_slots is not None:
        _check_cuda("state_slots", state_slots, torch.int64, dev)
        _require(state_slots.shape == (n,), "state_slots must be [n]")
    for name, t in (("initial_state", initial_state), ("final_state", final_state)):
        if t is not None:
            _check_cuda(name, t, torch.float32, dev)
            _require(t.dim() == 4 and tuple(t.shape[1:]) == (H, dv, dk) and t.is_contiguous(),
                     f"{name} must be a contiguous [*, {H}, {dv}, {dk}] tensor")
            _require(state_slots is not None or t.shape[0] >= n, f"{name} has fewer rows than sequences")
    if output_final_state and final_state is None:
        final_state = torch.empty((rows, H, dv, dk), device=dev, dtype=torch.float32)
    if out is None:
        out = torch.empty((N, H, dv), device=dev, dtype=torch.bfloat16)
    _check_cuda("out", out, torch.bfloat16, dev)
    _require(out.shape == (N, H, dv) and out.is_contiguous(), "out must be a contiguous [N, H, dv] tensor")
    if scale is None:
        scale = dk ** -0.5
    ws_bytes = gdn_chunk_prefill_workspace_bytes(N, n, H, dk)
    if workspace is None:
        workspace = torch.empty(max(ws_bytes, 1), device=dev, dtype=torch.uint8) if ws_bytes else None
    else:
        _check_cuda("workspace", workspace, torch.uint8, dev)
        _require(workspace.is_contiguous() and workspace.numel() >= ws_bytes,
                 f"workspace must be a contiguous uint8 buffer of at least {ws_bytes} bytes")
    ptr = lambda t: None if t is None else t.data_ptr()  # noqa: E731
    _lib.call("zb_gdn_chunk_prefill", q.data_ptr(), k.data_ptr(), v.data_ptr(), g.data_ptr(), beta.data_ptr(),
              cu_seqlens.data_ptr(), n, H, dk, dv, float(scale), ptr(initial_state), ptr(state_slots),
              ptr(final_state) if output_final_state else None, out.data_ptr(), N, ptr(workspace),
              0 if workspace is None else workspace.numel(), _stream(dev))
    return out, (final_state if output_final_state else None)


def gdn_prologue(mixed, conv_weight, A_log, dt_bias, cu_seqlens, seq_of_token, slots, conv_state, *, heads,
                 head_dim, fresh=None, q=None, k=None, v=None, g=None, beta=None):
    """Causal conv + SiLU over the qkv channels, per-head L2 norm of q and k, log decay g and beta from the in_proj
    output rows [qkv | z | a | b] (lm.py:561-573; gdn.py:403-423). conv_state [rows, 3*inner, W-1] (bf16) is read
    as each sequence's history and replaced by its last W-1 inputs; ``fresh`` [n] uint8 starts a sequence from a
    zero history. Returns (q, k, v [N, H, d] bf16, g, beta [N, H] fp32)."""
    _check_cuda("mixed", mixed, torch.bfloat16)
    dev = mixed.device
    N = mixed.shape[0]
    H, D = heads, head_dim
    inner = H * D
    _require(mixed.dim() == 2 and mixed.shape[1] >= 4 * inner + 2 * H and mixed.stride(1) == 1,
             "mixed must be [N, 4*inner + 2*H] with contiguous rows")
    _check_cuda("conv_weight", conv_weight, torch.bfloat16, dev)
    _require(conv_weight.numel() == 3 * inner * 4 and conv_weight.is_contiguous(), "conv_weight must be [3*inner, 1, 4]")
    _check_cuda("conv_state", conv_state, torch.bfloat16, dev)
    _require(conv_state.dim() == 3 and conv_state.shape[1:] == (3 * inner, 3) and conv_state.is_contiguous(),
             "conv_state must be a contiguous [rows, 3*inner, 3] tensor")
    for name, t in (("A_log", A_log), ("dt_bias", dt_bias)):
        _check_cuda(name, t, torch.float32, dev)
    n = cu_seqlens.numel() - 1
    _check_cuda("cu_seqlens", cu_seqlens, torch.int32, dev)
    _check_cuda("seq_of_token", seq_of_token, torch.int32, dev)
    _check_cuda("slots", slots, torch.int64, dev)
    if fresh is not None:
        _check_cuda("fresh", fresh, torch.uint8, dev)
    bf = dict(device=dev, dtype=torch.bfloat16)
    q = torch.empty(N, H, D, **bf) if q is None else q
    k = torch.empty(N, H, D, **bf) if k is None else k
    v = torch.empty(N, H, D, **bf) if v is None else v
    g = torch.empty(N, H, device=dev, dtype=torch.float32) if g is None else g
    beta = torch.empty(N, H, device=dev, dtype=torch.float32) if beta is None else beta
    _lib.call("zb_gdn_prologue", mixed.data_ptr(), mixed.stride(0), conv_weight.data_ptr(), A_log.data_ptr(),
              dt_bias.data_ptr(), cu_seqlens.data_ptr(), seq_of_token.data_ptr(), slots.data_ptr(),
              None if fresh is None else fresh.data_ptr(), conv_state.data_ptr(), conv_state.shape[0], n, N, H, D,
              q.data_ptr(),
              k.data_ptr(), v.data_ptr(), g.data_ptr(), beta.data_ptr(), _stream(dev))
    return q, k, v, g, beta


def gdn_prologue_decode(mixed, conv_weight, A_log, dt_bias, slots, conv_state, *, heads, head_dim, q=None, k=None,
                        v=None, g=None, beta=None):
    """:func:`gdn_prologue` for a decode batch: row i is the one new token of request i, whose conv history is row
    ``slots[i]`` of conv_state (a slot outside [0, rows) is a padding row: zero history, nothing written). The
    history update happens in the same kernel (no second launch). Returns (q, k, v, g, beta)."""
    _check_cuda("mixed", mixed, torch.bfloat16)
    dev = mixed.device
    N = mixed.shape[0]
    H, D = heads, head_dim
    inner = H * D
    _require(mixed.dim() == 2 and mixed.shape[1] >= 4 * inner + 2 * H and mixed.stride(1) == 1,
             "mixed must be [N, 4*inner + 2*H] with contiguous rows")
    _check_cuda("conv_weight", conv_weight, torch.bfloat16, dev)
    _require(conv_weight.numel() == 3 * inner * 4 and conv_weight.is_contiguous(), "conv_weight must be [3*inner, 1, 4]")
    _check_cuda("conv_state", conv_state, torch.bfloat16, dev)
    _require(conv_state.dim() == 3 and conv_state.shape[1:] == (3 * inner, 3) and conv_state.is_contiguous(),
             "conv_state must be a contiguous [rows, 3*inner, 3] tensor")
    for name, t in (("A_log", A_log), ("dt_bias", dt_bias)):
        _check_cuda(name, t, torch.float32, dev)
    _check_cuda("slots", slots, torch.int64, dev)
    _require(slots.numel() == N, f"slots must hold one row per token ({N}), got {slots.numel()}")
    bf = dict(device=dev, dtype=torch.bfloat16)
    q = torch.empty(N, H, D, **bf) if q is None else q
    k = torch.empty(N, H, D, **bf) if k is None else k
    v = torch.empty(N, H, D, **bf) if v is None else v
    g = torch.empty(N, H, device=dev, dtype=torch.float32) if g is None else g
    beta = torch.empty(N, H, device=dev, dtype=torch.float32) if beta is None else beta
    _lib.call("zb_gdn_prologue_decode", mixed.data_ptr(), mixed.stride(0), conv_weight.data_ptr(), A_log.data_ptr(),
              dt_bias.data_ptr(), slots.data_ptr(), conv_state.data_ptr(), conv_state.shape[0], N, H, D,
              q.data_ptr(), k.data_ptr(), v.data_ptr(), g.data_ptr(), beta.data_ptr(), _stream(dev))
    return q, k, v, g, beta


def gdn_gated_norm(o, z, weight, eps=1e-5, out=None):
    """Per-head RMSNorm(o; weight, eps) * SiLU(z), rounded once to bf16 (gdn.py:435-445; lm.py:585-587).
    o [N, H, d] bf16; z [N, H*d] bf16 view (row stride allowed); returns [N, H*d] bf16."""
    _check_cuda("o", o, torch.bfloat16)
    dev = o.device
    N, H, D = o.shape
    _require(o.is_contiguous(), "o must be contiguous")
    _check_cuda("z", z, torch.bfloat16, dev)
    _require(z.shape == (N, H * D) and z.stride(1) == 1, "z must be [N, H*d] with contiguous rows")
    _check_cuda("weight", weight, torch.bfloat16, dev)
    if out is None:
        out = torch.empty(N, H * D, device=dev, dtype=torch.bfloat16)
    _lib.call("zb_gdn_gated_norm", o.data_ptr(), z.data_ptr(), z.stride(0) if N > 1 else H * D, weight.data_ptr(),
              float(eps), N, H, D, out.data_ptr(), _stream(dev))
    return out


# ----------------------------------------------------------------------------- dense projections (tcgen05)

_PROJ_WS: dict = {}  # device -> the current split-K workspace (uint8, ticket counters zero between launches)
_PROJ_WS_RETIRED: list = []  # replaced workspaces stay alive: a captured graph may still hold their address


def _proj_workspace(dev: torch.device, nbytes: int) -> torch.Tensor | None:
    """The device's split-K workspace, grown (zeroed) when a launch needs more; launches use it in stream order."""
    if nbytes <= 0:
        return None
    ws = _PROJ_WS.get(dev)
    if ws is None or ws.numel() < nbytes:
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError("the projection GEMM's workspace must be sized before graph capture: run the step "
                               "once eagerly (a warm-up) before capturing it")
        if ws is not None:
            _PROJ_WS_RETIRED.append(ws)
        ws = torch.zeros(nbytes, device=dev, dtype=torch.uint8)
        _PROJ_WS[dev] = ws
    return ws


def _proj_rows(name: str, x: torch.Tensor, K: int) -> int:
    _check_cuda(name, x, torch.bfloat16)
    _require(x.dim() == 2 and x.shape[1] == K and x.stride(1) == 1, f"{name} must be [T, {K}] with contiguous rows")
    stride = x.stride(0) if x.shape[0] > 1 else K
    _require(stride % 8 == 0 and x.data_ptr() % 16 == 0, f"{name}: rows must start on 16-byte boundaries")
    return stride


def proj_gemm(x, weight, out=None, *, block_n: int = 0, splits: int = 0):
    """out = x @ weight^T on the tensor cores (tcgen05 CTA pairs, fp32 accumulation, one bf16 rounding): the decode
    step's dense projections (F.linear of the DeltaNet / attention wo, the attention projection and the codebook
    head; gdn.py:447, zonos3.py:326-390, :1341-1360). x [T, K] bf16, weight [N, K] bf16 contiguous, out [T, N] bf16
    (a row stride allowed). ``block_n`` (64 / 128 / 256) and ``splits`` (K slices) pick the tiling; 0 = chosen from
    the shape. K must be a multiple of 128 and N of 8."""
    _check_cuda("weight", weight, torch.bfloat16)
    dev = weight.device
    _require(weight.dim() == 2 and weight.is_contiguous(), "weight must be a contiguous [N, K] tensor")
    N, K = weight.shape
    xs = _proj_rows("x", x, K)
    T = x.shape[0]
    if out is None:
        out = torch.empty(T, N, device=dev, dtype=torch.bfloat16)
    _check_cuda("out", out, torch.bfloat16, dev)
    _require(out.dim() == 2 and out.shape == (T, N) and out.stride(1) == 1, f"out must be [{T}, {N}] with contiguous rows")
    os_ = out.stride(0) if T > 1 else N
    lib = _lib.load()
    nbytes = int(lib.zb_proj_gemm_workspace_bytes(T, N, K, int(block_n), int(splits))) if T else 0
    ws = _proj_workspace(dev, nbytes)
    _lib.call("zb_proj_gemm", x.data_ptr(), xs, T, K, weight.data_ptr(), N, out.data_ptr(), os_, int(block_n),
              int(splits), None if ws is None else ws.data_ptr(), 0 if ws is None else ws.numel(), _stream(dev))
    return out


def gdn_in_proj_decode(x, in_proj, conv_weight, A_log, dt_bias, slots, conv_state, *, heads, head_dim,
                       splits: int = 0, q=None, k=None, v=None, z=None, g=None, beta=None):
    """The DeltaNet in_proj GEMM fused with its decode prologue (gdn.py:399-434): row i of x is the new token of the
    request whose conv history is row ``slots[i]`` of conv_state (outside [0, rows): a padding row, zero history,
    nothing written). The in_proj output is never stored: the GEMM's epilogue runs the causal conv (shifting the
    history in place), SiLU, the per-head L2 norm of q and k, g and beta, and stores z for the gated norm.
    Returns (q, k, v [T, H, d] bf16, z [T, H*d] bf16, g, beta [T, H] fp32)."""
    _check_cuda("in_proj", in_proj, torch.bfloat16)
    dev = in_proj.device
    H, D = heads, head_dim
    inner = H * D
    N, K = in_proj.shape
    _require(N == 4 * inner + 2 * H and in_proj.is_contiguous(), f"in_proj must be a contiguous [{4 * inner + 2 * H}, K] tensor")
    xs = _proj_rows("x", x, K)
    T = x.shape[0]
    _check_cuda("conv_weight", conv_weight, torch.bfloat16, dev)
    _require(conv_weight.numel() == 3 * inner * 4 and conv_weight.is_contiguous(), "conv_weight must be [3*inner, 1, 4]")
    _check_cuda("conv_state", conv_state, torch.bfloat16, dev)
    _require(conv_state.dim() == 3 and conv_state.shape[1:] == (3 * inner, 3) and conv_state.is_contiguous(),
             "conv_state must be a contiguous [rows, 3*inner, 3] tensor")
    for name, t in (("A_log", A_log), ("dt_bias", dt_bias)):
        _check_cuda(name, t, torch.float32, dev)
    _check_cuda("slots", slots, torch.int64, dev)
    _require(slots.numel() == T and slots.is_contiguous(), f"slots must hold one row per token ({T})")
    bf = dict(device=dev, dtype=torch.bfloat16)
    q = torch.empty(T, H, D, **bf) if q is None else q
    k = torch.empty(T, H, D, **bf) if k is None else k
    v = torch.empty(T, H, D, **bf) if v is None else v
    z = torch.empty(T, inner, **bf) if z is None else z
    g = torch.empty(T, H, device=dev, dtype=torch.float32) if g is None else g
    beta = torch.empty(T, H, device=dev, dtype=torch.float32) if beta is None else beta
    for name, t in (("q", q), ("k", k), ("v", v), ("z", z)):
        _check_cuda(name, t, torch.bfloat16, dev)
        _require(t.is_contiguous() and t.numel() == T * inner, f"{name} must be a contiguous [T, {inner}] buffer")
    for name, t in (("g", g), ("beta", beta)):
        _check_cuda(name, t, torch.float32, dev)
        _require(t.is_contiguous() and t.numel() == T * H, f"{name} must be a contiguous [T, {H}] buffer")
    lib = _lib.load()
    nbytes = int(lib.zb_proj_gemm_workspace_bytes(T, N, K, 128, int(splits))) if T else 0  # its column tile
    ws = _proj_workspace(dev, nbytes)
    _lib.call("zb_gdn_in_proj_decode", x.data_ptr(), xs, T, K, in_proj.data_ptr(), conv_weight.data_ptr(),
              A_log.data_ptr(), dt_bias.data_ptr(), slots.data_ptr(), conv_state.data_ptr(), conv_state.shape[0], H, D,
              q.data_ptr(), k.data_ptr(), v.data_ptr(), z.data_ptr(), g.data_ptr(), beta.data_ptr(), int(splits),
              None if ws is None else ws.data_ptr(), 0 if ws is None else ws.numel(), _stream(dev))
    return q, k, v, z, g, beta


# ------------------------------------------------------------------------------------- GQA decode attention


def kv_store(k_cache, v_cache, slots, k, v):
    """Row i of k and v ([N, Hkv, hd] bf16) into slot slots[i] of k_cache and v_cache ([slots, Hkv, hd] bf16, slot
    stride allowed); a slot outside [0, slots) stores nothing. The store of MHAKVCache.store_kv
    (servers/sgl/src/zonos3_sgl/kvcache/mha_pool.py:58-67, kernel/store.py:30-43)."""
    dev = k.device
    for name, t in (("k_cache", k_cache), ("v_cache", v_cache), ("k", k), ("v", v)):
        _check_cuda(name, t, torch.bfloat16, dev)
    _check_cuda("slots", slots, torch.int32, dev)
    N, Hkv, hd = k.shape
    ks = _rows("k", k, (Hkv, hd))
    vs = _rows("v", v, (Hkv, hd))
    cs = _rows("k_cache", k_cache, (Hkv, hd))
    _require(v_cache.shape == k_cache.shape and v_cache.stride() == k_cache.stride(),
             "v_cache must match k_cache's shape and strides")
    _require(slots.shape == (N,) and slots.is_contiguous(), f"slots must be a contiguous [{N}] tensor")
    _lib.call("zb_kv_store", k_cache.data_ptr(), v_cache.data_ptr(), cs, k_cache.shape[0], slots.data_ptr(),
              k.data_ptr(), ks, v.data_ptr(), vs, N, Hkv, hd, _stream(dev))


def gqa_tile(head_dim: int) -> int:
    """Key positions of one tile of the decode attention kernel (split lengths are multiples of it): 128 for head
    dim 128 (tensor-core kernel), 32 otherwise."""
    return 128 if head_dim == 128 else 32


def gqa_splits(batch: int, kv_heads: int, max_len: int, num_splits: int = 1, head_dim: int = 128) -> tuple[int, int]:
    """(splits, split_len) covering max_len keys. num_splits = 1 runs unsplit, as the reference does for this model
    (servers/sgl/src/zonos3_sgl/attention/fa.py:41-50); 0 picks enough splits for about two CTAs per resident CTA
    slot (148 SMs x 1 CTA for head dim 128, x 3 otherwise), at least 256 keys each; n > 1 forces n."""
    max_len = max(int(max_len), 1)
    tile = gqa_tile(head_dim)
    if num_splits == 0:
        slots = 148 * (1 if head_dim == 128 else 3)
        want = -(-2 * slots // max(batch * kv_heads, 1))
        num_splits = max(1, min(want, max_len // 256))
    split_len = -(-max_len // num_splits)
    split_len = -(-split_len // tile) * tile
    return -(-max_len // split_len), split_len


def gqa_decode(q, k_cache, v_cache, page_table, cache_seqlens, *, softmax_scale=None, num_splits=1, out=None,
               workspace=None, gate=None):
    """Decode attention over a slot-indexed KV cache: the flash_attn_with_kvcache call of the FA backend for a
    decode batch (servers/sgl/src/zonos3_sgl/attention/fa.py:64-81, :171-212; causal, one query row per request,
    one token per page).

    q [B, Hq, hd] bf16; k_cache, v_cache [slots, Hkv, hd] bf16 (slot stride allowed); page_table [B, max_pages]
    int32 (slot of each key position; an entry outside [0, slots) masks that key); cache_seqlens [B] int32 (keys
    per request, clamped to max_pages). Query head h
    reads KV head h // (Hq / Hkv). softmax_scale defaults to hd ** -0.5. num_splits as :func:`gqa_splits`;
    workspace: optional fp32 tensor of at least B * Hq * splits * (hd + 2) elements (allocated when absent and
    needed). gate: optional [B, Hq] bf16 gate logits (row stride allowed): the output is multiplied by
    sigmoid(gate) per head, with torch's bf16 rounding points (the attention layer's output gate). Returns out
    [B, Hq, hd] bf16."""
    dev = q.device
    _check_cuda("q", q, torch.bfloat16)
    B, Hq, hd = q.shape
    for name, t in (("k_cache", k_cache), ("v_cache", v_cache)):
        _check_cuda(name, t, torch.bfloat16, dev)
    _require(k_cache.dim() == 3 and k_cache.shape[2] == hd, f"k_cache must be [slots, Hkv, {hd}]")
    Hkv = k_cache.shape[1]
    _require(Hq % Hkv == 0, f"{Hq} query heads do not group over {Hkv} KV heads")
    qs = _rows("q", q, (Hq, hd))
    cs = _rows("k_cache", k_cache, (Hkv, hd))
    _require(v_cache.shape == k_cache.shape and v_cache.stride() == k_cache.stride(),
             "v_cache must match k_cache's shape and strides")
    _check_cuda("page_table", page_table, torch.int32, dev)
    _check_cuda("cache_seqlens", cache_seqlens, torch.int32, dev)
    _require(page_table.dim() == 2 and page_table.shape[0] == B and page_table.stride(1) == 1,
             f"page_table must be [{B}, max_pages] with contiguous rows")
    _require(cache_seqlens.shape == (B,) and cache_seqlens.is_contiguous(), f"cache_seqlens must be [{B}]")
    if out is None:
        out = torch.empty(B, Hq, hd, device=dev, dtype=torch.bfloat16)
    _check_cuda("out", out, torch.bfloat16, dev)
    os_ = _rows("out", out, (Hq, hd))
    splits, split_len = gqa_splits(B, Hkv, page_table.shape[1], num_splits, hd)
    need = B * Hq * splits * (hd + 2) if splits > 1 else 0
    if need and (workspace is None or workspace.numel() < need):
        workspace = torch.empty(need, device=dev, dtype=torch.float32)
    if need:
        _check_cuda("workspace", workspace, torch.float32, dev)
    scale = float(hd ** -0.5 if softmax_scale is None else softmax_scale)
    gs = 0
    if gate is not None:
        _check_cuda("gate", gate, torch.bfloat16, dev)
        _require(gate.dim() == 2 and gate.shape == (B, Hq) and gate.stride(1) == 1, f"gate must be [{B}, {Hq}]")
        gs = gate.stride(0) if B > 1 else Hq
    _lib.call("zb_gqa_decode", q.data_ptr(), qs, k_cache.data_ptr(), v_cache.data_ptr(), cs, k_cache.shape[0],
              page_table.data_ptr(), page_table.stride(0) if B > 1 else page_table.shape[1], cache_seqlens.data_ptr(),
              page_table.shape[1], B, Hq, Hkv, hd, scale, splits, split_len, workspace.data_ptr() if need else None,
              need * 4, out.data_ptr(), os_, None if gate is None else gate.data_ptr(), gs, _stream(dev))
    return out


# ------------------------------------------------------------------------------------------------ TTS sampler


def _host_list(t) -> list:
    return t.tolist() if isinstance(t, torch.Tensor) else list(t)


def sample_tts(logits, temperatures, top_ks, top_ps, min_ps, *, codebook_size, audio_pad_id, stop_token_ids,
               repetition_token_ids=None, repetition_penalties=None, codebook_sizes=None, text_vocab=0, seed=0,
               offset=0, stop_blocked=None, stop_bias=None, probs_out=None, out=None, device_temperatures=None,
               softcap=0.0, offset_dev=None):
    """Next codes from logits [B, C, V] (bf16 or fp32, CUDA): sample_tts (model/src/zonos3/tts/sampler.py:159-372)
    as one kernel per (request, codebook) row, with the reference's masks, stop bias, repetition penalty, greedy
    path and top-k / top-p / min-p filters. temperatures, top_ks, top_ps, min_ps, stop_token_ids: [B] tensors or
    lists; their values pick host-side branches as in the reference (greedy when every temperature <= 0, the batch's
    min top-k, max top-p and max min-p), so pass CPU tensors to keep the host from waiting on the GPU. The draw uses
    Philox4x32-10 keyed by ``seed`` at counter (row, ``offset`` + ``offset_dev[0]``): advance ``offset`` every step,
    or, inside a captured graph, the one-element int64 device counter ``offset_dev``. Returns
    [B, C + 1] int32 (codes, then ``text_vocab``); ``probs_out`` ([B * C, V] fp32) receives the final
    distributions. Per-row inputs already on the device (int32 stop ids, fp32 ``device_temperatures``, ...) are
    used as they are, so a call can be captured in a CUDA graph. ``softcap`` > 0 applies the head's soft cap
    (cap * tanh(x / cap), zonos3.py:1341-1360) to the raw head output first, with torch's bf16 rounding points."""
    _require(isinstance(logits, torch.Tensor) and logits.is_cuda, "logits must be a CUDA tensor")
    _require(logits.dtype in (torch.bfloat16, torch.float32), "logits must be bf16 or fp32")
    dev = logits.device
    B, C, V = logits.shape
    _require(logits.stride(2) == 1 and logits.stride(1) >= V and logits.stride(0) >= (C - 1) * logits.stride(1) + V,
             "logits must be [B, C, V] with contiguous, non-overlapping rows")
    temps = _host_list(temperatures)
    greedy = all(float(t) <= 0 for t in temps)
    top_k = int(min(int(k) for k in _host_list(top_ks))) if B else 0
    top_p = float(max(float(v) for v in _host_list(top_ps))) if B else 1.0
    min_p = float(max(float(v) for v in _host_list(min_ps))) if B else 0.0
    i32 = dict(device=dev, dtype=torch.int32)
    f32 = dict(device=dev, dtype=torch.float32)
    dev_t = lambda v, kw: v.to(**kw) if isinstance(v, torch.Tensor) else torch.tensor(v, **kw)  # noqa: E731
    temp_d = dev_t(temperatures if device_temperatures is None else device_temperatures, f32)
    stop_d = dev_t(stop_token_ids, i32)
    sizes_d = None if codebook_sizes is None else dev_t(codebook_sizes, i32)
    blocked_d = None if stop_blocked is None else dev_t(stop_blocked, dict(device=dev, dtype=torch.uint8))
    bias_d = None if stop_bias is None else dev_t(stop_bias, f32)
    W = 0
    rep_d = pen_d = None
    if repetition_token_ids is not None and repetition_penalties is not None and repetition_token_ids.numel():
        rep_d = dev_t(repetition_token_ids, i32).contiguous()
        _require(rep_d.shape[:2] == (B, C), f"repetition_token_ids must be [{B}, {C}, W]")
        W = rep_d.shape[2]
        pen_d = dev_t(repetition_penalties, f32)
    if out is None:
        out = torch.empty(B, C + 1, **i32)
    if offset_dev is not None:
        _check_cuda("offset_dev", offset_dev, torch.int64, dev)
        _require(offset_dev.numel() >= 1, "offset_dev must hold one counter")
    ptr = lambda t: None if t is None else t.data_ptr()  # noqa: E731
    _lib.call("zb_sample_tts", logits.data_ptr(), int(logits.dtype == torch.float32), float(softcap), logits.stride(1),
              logits.stride(0), B, C, V,
              temp_d.data_ptr(), int(greedy), top_k, top_p, min_p, int(codebook_size), int(audio_pad_id),
              stop_d.data_ptr(), ptr(sizes_d), ptr(blocked_d), ptr(bias_d), ptr(rep_d), W, ptr(pen_d),
              int(seed) & (2**64 - 1), int(offset) & (2**64 - 1), ptr(offset_dev), int(text_vocab), out.data_ptr(),
              ptr(probs_out), _stream(dev))
    return out


# ------------------------------------------------------------------------------------------- input embedding


def embed_norm(ids, tables, *, eps=1e-5, norm_weight=None, normalize=True, out=None):
    """Layer-stack input rows: RMSNorm(sum_c tables[c][ids[:, c]]) (MultiEmbedding.forward + emb_norm,
    servers/sgl/src/zonos3_sgl/models/zonos3.py:225-255, :1218), one kernel. ids [N, C] int32 on the device (row
    stride allowed); tables: C bf16 [rows_c, D] tensors; the columns are summed one add at a time in bf16 as the
    reference does. An id outside its table reads zeros and sets bit 32 of ``device_status()``."""
    _require(isinstance(ids, torch.Tensor) and ids.is_cuda and ids.dtype == torch.int32 and ids.dim() == 2,
             "ids must be a [N, C] int32 CUDA tensor")
    dev = ids.device
    N, C = ids.shape
    _require(ids.stride(1) == 1 or C == 1, "ids columns must be contiguous")
    _require(len(tables) == C, f"{C} id columns need {C} tables, got {len(tables)}")
    D = tables[0].shape[1]
    for i, t in enumerate(tables):
        _check_cuda(f"tables[{i}]", t, torch.bfloat16, dev)
        _require(t.dim() == 2 and t.shape[1] == D and t.is_contiguous(), f"tables[{i}] must be a contiguous [rows, {D}]")
    if norm_weight is not None:
        _check_cuda("norm_weight", norm_weight, torch.bfloat16, dev)
        _require(norm_weight.shape == (D,) and norm_weight.is_contiguous(), f"norm_weight must be [{D}]")
    if out is None:
        out = torch.empty(N, D, device=dev, dtype=torch.bfloat16)
    _check_cuda("out", out, torch.bfloat16, dev)
    _require(out.shape == (N, D) and out.stride(1) == 1, f"out must be [{N}, {D}] with contiguous rows")
    ptrs = (ctypes.c_void_p * C)(*[t.data_ptr() for t in tables])
    rows = (ctypes.c_int32 * C)(*[t.shape[0] for t in tables])
    _lib.call("zb_embed_norm", ids.data_ptr(), ids.stride(0) if N > 1 else C, C, ctypes.cast(ptrs, ctypes.c_void_p),
              ctypes.cast(rows, ctypes.c_void_p), None if norm_weight is None else norm_weight.data_ptr(), float(eps),
              int(bool(normalize)), N, D, out.data_ptr(), out.stride(0) if N > 1 else D, _stream(dev))
    return out


def gqa_prologue_decode(proj, temp, positions, k_cache, v_cache, out_loc, *, heads, kv_heads, rope_theta=10000.0,
                        eps=1e-6, q_out=None):
    """The attention layer's decode prologue (Attention.forward, servers/sgl/src/zonos3_sgl/models/zonos3.py:340-375)
    in one kernel: proj [N, >= (heads + 2 kv_heads) * 128] bf16 holds q | k | v (rows contiguous, row stride
    allowed); q gets RMSNorm (eps) x |temp| and interleaved RoPE at ``positions`` ([N] int32), k RMSNorm and RoPE;
    k and v go to slot ``out_loc[t]`` of k_cache / v_cache ([slots, kv_heads, 128] bf16). Returns q [N, heads, 128]."""
    dev = proj.device
    _check_cuda("proj", proj, torch.bfloat16)
    N = proj.shape[0]
    hd = 128
    _require(proj.dim() == 2 and proj.stride(1) == 1 and proj.shape[1] >= (heads + 2 * kv_heads) * hd,
             "proj must be [N, >= (heads + 2 kv_heads) * 128] with contiguous rows")
    for name, t in (("temp", temp), ("k_cache", k_cache), ("v_cache", v_cache)):
        _check_cuda(name, t, torch.bfloat16, dev)
    _require(temp.numel() == heads and temp.is_contiguous(), f"temp must hold {heads} values")
    _check_cuda("positions", positions, torch.int32, dev)
    _check_cuda("out_loc", out_loc, torch.int32, dev)
    _require(positions.shape == (N,) and out_loc.shape == (N,), "positions and out_loc must be [N]")
    cs = _rows("k_cache", k_cache, (kv_heads, hd))
    _require(v_cache.shape == k_cache.shape and v_cache.stride() == k_cache.stride(), "v_cache must match k_cache")
    if q_out is None:
        q_out = torch.empty(N, heads, hd, device=dev, dtype=torch.bfloat16)
    _check_cuda("q_out", q_out, torch.bfloat16, dev)
    _require(q_out.shape == (N, heads, hd) and q_out.is_contiguous(), f"q_out must be a contiguous [{N}, {heads}, 128]")
    _lib.call("zb_gqa_prologue_decode", proj.data_ptr(), proj.stride(0) if N > 1 else proj.shape[1], temp.data_ptr(),
              positions.data_ptr(), float(rope_theta), float(eps), q_out.data_ptr(), k_cache.data_ptr(),
              v_cache.data_ptr(), cs, k_cache.shape[0], out_loc.data_ptr(), N, heads, kv_heads, hd, _stream(dev))
    return q_out


def decode_advance(codes, ids, positions, cache_seqlens, out_loc, page_table, counter, *, history=None, ring=None):
    """The bookkeeping between two decode steps in one kernel (zb_decode_advance): the sampled codes [B, >= cols]
    become the next ids [B, cols]; the first C codes enter the repetition window history [B, C, W] at column
    ring[0]; positions and cache_seqlens advance by one (lengths capped at the page table's width); out_loc takes
    each stream's next page-table slot; ring and the sampler's draw counter (int64 [1]) advance."""
    dev = codes.device
    for name, t in (("codes", codes), ("ids", ids), ("positions", positions), ("cache_seqlens", cache_seqlens),
                    ("out_loc", out_loc), ("page_table", page_table)):
        _check_cuda(name, t, torch.int32, dev)
        _require(t.is_contiguous() or name == "page_table", f"{name} must be contiguous")
    _check_cuda("counter", counter, torch.int64, dev)
    B = codes.shape[0]
    _require(ids.shape[0] == B and ids.shape[1] <= codes.shape[1], "ids must be [B, <= codes columns]")
    _require(page_table.dim() == 2 and page_table.shape[0] == B and page_table.stride(1) == 1, "page_table [B, L]")
    C = W = 0
    if history is not None:
        _check_cuda("history", history, torch.int32, dev)
        _check_cuda("ring", ring, torch.int64, dev)
        _require(history.dim() == 3 and history.shape[0] == B and history.is_contiguous(), "history [B, C, W]")
        C, W = history.shape[1], history.shape[2]
    ptr = lambda t: None if t is None else t.data_ptr()  # noqa: E731
    _lib.call("zb_decode_advance", codes.data_ptr(), codes.shape[1], ids.data_ptr(), ids.shape[1], ptr(history), C, W,
              ptr(ring), counter.data_ptr(), positions.data_ptr(), cache_seqlens.data_ptr(), out_loc.data_ptr(),
              page_table.data_ptr(), page_table.stride(0), page_table.shape[1], B, _stream(dev))

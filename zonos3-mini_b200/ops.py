"""Thin torch-facing wrappers over the C-ABI entry points.

Each wrapper validates shapes, dtypes and devices (raising ``ValueError`` the way the reference's layers do), then
passes raw device pointers, strides and the current CUDA stream to ``libzonos3_b200.so``. Outputs are written into
caller-provided tensors when given, so a wrapper allocates nothing inside a CUDA-graph capture.
"""

from __future__ import annotations

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
) -> torch.Tensor:
    """Full AttnRes route over ``bank[:num_sources]`` (+ ``source`` as the last source) for every token.

    bank [>= num_sources, T, D] bf16 (rows contiguous [T, D]); source [T, D] bf16; query [D] bf16. The mix follows
    full_attnres_route (model/src/zonos3/reference/lm.py:384-389) with the fused Triton kernel's bf16 rounding
    points. ``norm_weight`` fuses the RMSNorm after the route (out = RMSNorm(mix) and, if given, mix_out = mix);
    ``append_to`` (a [T, D] bank row) receives ``source`` in the same pass.
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
    ptr = lambda t: None if t is None else t.data_ptr()  # noqa: E731
    _lib.call(
        "zb_attnres_route",
        ptr(bank) if num_sources else None, bank_stride, num_sources, ptr(source), ptr(append_to),
        query.data_ptr(), float(eps), ptr(norm_weight), float(norm_eps), out.data_ptr(), ptr(mix_out), T, D,
        _stream(dev),
    )
    return out


def device_status(clear: bool = True) -> int:
    """Bits set by kernels whose bounded device-side waits expired on the current device (synchronous)."""
    import ctypes

    flags = ctypes.c_uint(0)
    _lib.call("zb_device_status", ctypes.byref(flags), int(clear))
    return flags.value

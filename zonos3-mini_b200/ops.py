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

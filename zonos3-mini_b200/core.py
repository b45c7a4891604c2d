"""The per-step batch context the layer modules read, with the field names the reference's layers use
(servers/sgl/src/zonos3_sgl/core.py; read by OriginalGDN.forward, servers/sgl/src/zonos3_sgl/models/gdn.py:235-257,
and Attention.forward, servers/sgl/src/zonos3_sgl/models/zonos3.py:315-390): ``get_global_ctx().batch`` with
``is_decode``, ``reqs`` (each with ``table_idx``, ``extend_len``, ``cached_len``, ``device_len``, ``uid``,
``is_cfg_uncond``), ``padded_size``, ``input_ids`` and ``attn_metadata``; ``get_global_ctx().attn_backend`` is the
KV pool of the global-attention layers."""

from __future__ import annotations

import contextlib
from dataclasses import dataclass, field

import torch  # noqa: F401  (annotations)


@dataclass
class Req:
    table_idx: int  # the request's state slot
    extend_len: int  # new rows in this forward
    cached_len: int = 0  # rows already in the state before this forward
    uid: int = 0
    is_cfg_uncond: bool = False

    @property
    def device_len(self) -> int:
        return self.cached_len + self.extend_len


@dataclass
class AttnMetadata:
    """Where the global-attention layers read and write the KV cache (page size 1, the FA backend's layout,
    servers/sgl/src/zonos3_sgl/attention/fa.py): every new row t has a position and a cache slot; request b reads
    keys page_table[b, :cache_seqlens[b]] (its new rows included)."""

    positions: "torch.Tensor"  # [N] int32
    out_loc: "torch.Tensor"  # [N] int32
    page_table: "torch.Tensor"  # [B, max_len] int32
    cache_seqlens: "torch.Tensor"  # [B] int32
    cu_seqlens_q: list[int] | None = None  # prefill: request b's new rows are [cu[b], cu[b+1])


@dataclass
class Batch:
    reqs: list[Req]
    is_decode: bool
    padded_size: int | None = None  # decode graph batch size (>= len(reqs))
    gdn_prefill: object = None
    input_ids: "torch.Tensor | None" = None  # [N, n_codebooks + 1] int32
    attn_metadata: AttnMetadata | None = None

    @property
    def padded_reqs(self) -> list[Req]:
        return self.reqs


@dataclass
class Context:
    batch: Batch | None = None
    attn_backend: object = None  # attention.SlotKVPool of the model being run
    extra: dict = field(default_factory=dict)


_CTX = Context()


def _reference_context():
    """The reference server's get_global_ctx (servers/sgl/src/zonos3_sgl/core.py) when that package imports, so the
    modules dropped into the server read the server's batch; None otherwise (this package's own context)."""
    try:
        from zonos3_sgl.core import get_global_ctx as reference_ctx  # noqa: PLC0415
    except Exception:  # the reference server is not installed (or its native dependencies are missing)
        return None
    return reference_ctx


_REFERENCE_CTX = _reference_context()


def get_global_ctx() -> Context:
    return _REFERENCE_CTX() if _REFERENCE_CTX is not None else _CTX


@contextlib.contextmanager
def forward_batch(batch: Batch):
    """Make ``batch`` the current batch for the duration of one model forward."""
    ctx = get_global_ctx()
    previous = ctx.batch
    ctx.batch = batch
    try:
        yield batch
    finally:
        ctx.batch = previous

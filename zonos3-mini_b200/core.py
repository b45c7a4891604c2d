"""The per-step batch context the layer modules read, with the field names the reference's layers use
(servers/sgl/src/zonos3_sgl/core.py; read by OriginalGDN.forward, servers/sgl/src/zonos3_sgl/models/gdn.py:235-257):
``get_global_ctx().batch`` with ``is_decode``, ``reqs`` (each with ``table_idx``, ``extend_len``, ``cached_len``,
``device_len``, ``uid``, ``is_cfg_uncond``) and ``padded_size``."""

from __future__ import annotations

import contextlib
from dataclasses import dataclass, field


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
class Batch:
    reqs: list[Req]
    is_decode: bool
    padded_size: int | None = None  # decode graph batch size (>= len(reqs))
    gdn_prefill: object = None

    @property
    def padded_reqs(self) -> list[Req]:
        return self.reqs


@dataclass
class Context:
    batch: Batch | None = None
    extra: dict = field(default_factory=dict)


_CTX = Context()


def get_global_ctx() -> Context:
    return _CTX


@contextlib.contextmanager
def forward_batch(batch: Batch):
    """Make ``batch`` the current batch for the duration of one model forward."""
    previous = _CTX.batch
    _CTX.batch = batch
    try:
        yield batch
    finally:
        _CTX.batch = previous

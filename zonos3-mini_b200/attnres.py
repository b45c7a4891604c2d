"""Full AttnRes with the reference's module-level API, on the B200 route kernel (``zb_attnres_route``).

Drop-in names and signatures:

* ``full_attnres_route(sources, query, norm_eps)`` — servers/sgl/src/zonos3_sgl/models/zonos3.py:99-113
  (and model/src/zonos3/reference/lm.py:384-389, which takes a list of sources);
* ``FusedBlockAttnResContext(max_completed_blocks, reference, gradient_dtype)`` — the persistent bank of
  servers/sgl/src/zonos3_sgl/models/training_attnres_kernels.py:1438-1513 (forward use: ``blocks``,
  ``completed_count``, ``call_count``, ``validate_owner``, ``completed_view``);
* ``fused_full_attnres(state, source, query, norm_eps, append_current)`` — training_attnres_kernels.py:2826-2840.

A forward that knows its route queries up front (``forward_layers_full`` does) registers them with
``FusedBlockAttnResContext.register_queries``: each route then computes the next route's logits of the rows it
mixes, while they stream through registers, and leaves them in a [routes, T, rows] fp32 table, so that a route
computes only its current source's logit before its softmax and reads the bank once (``zb_attnres_route_tabled``).
A (source, route) logit depends on nothing but the source row, the route's query and the eps, so the table holds
exactly what the reference's route recomputes.

Inference only: the reference's autograd backward (used by its trainer) is not part of the serving hot path.
The bank append happens inside the route kernel, and when the caller already wrote ``source`` into the next bank
row (``state.next_row()``), the route reads it from there and nothing is copied.
"""

from __future__ import annotations

import torch

from . import ops


def full_attnres_route(sources, query: torch.Tensor, norm_eps: float) -> torch.Tensor:
    """One softmax mix over every source: ``sources`` is a [S, T, D] bf16 bank (or a list of [T, D] rows)."""
    if not isinstance(sources, torch.Tensor):
        sources = torch.stack(list(sources))
    if sources.dim() != 3:
        raise ValueError(f"sources must be [S, T, D], got {tuple(sources.shape)}")
    return ops.attnres_route(sources, sources.shape[0], query, norm_eps)


class FusedBlockAttnResContext:
    """One forward's bank of completed sources, allocated once and reused (graph-safe)."""

    TABLED_MAX_DIM = 4096  # hidden sizes the route over a logit table supports

    def __init__(self, max_completed_blocks: int, reference: torch.Tensor, gradient_dtype=torch.float32, **_):
        if not reference.is_cuda:
            raise RuntimeError("fused AttnRes requires CUDA")
        if reference.dtype != torch.bfloat16:
            raise RuntimeError("fused AttnRes runs on bf16 activations")
        self.token_shape = tuple(reference.shape[:-1])
        self.dim = int(reference.shape[-1])
        self.bt = 1
        for n in self.token_shape:
            self.bt *= int(n)
        self.max_completed_blocks = int(max_completed_blocks)
        self.gradient_dtype = gradient_dtype
        self.blocks = torch.empty((self.max_completed_blocks, self.bt, self.dim), device=reference.device,
                                  dtype=reference.dtype)
        # key inverse RMS of every bank row (and of the routed source), filled by the route kernel: each row's sum
        # of squares is read from HBM once per forward instead of once per later route
        self.rms_cache = torch.empty((self.bt, (self.max_completed_blocks + 4) // 4 * 4), device=reference.device,
                                     dtype=torch.float32)
        self._rms_eps = None
        self._queries = None  # registered route queries [R, D] (call order) and their logit table
        self._table = None
        self._table_eps = None
        self.completed_count = 0
        self.call_count = 0

    def reset(self) -> None:
        """Starts a new forward (the registered queries stay registered)."""
        self.completed_count = 0
        self.call_count = 0
        self._rms_eps = None

    def register_queries(self, queries: torch.Tensor | None, norm_eps: float | None = None) -> None:
        """Registers the queries of the forward's routes in call order (contiguous [R, D] bf16 on this device) and
        the key RMSNorm eps they run with: route number ``call_count`` must then pass ``queries[call_count]`` (this
        storage) and that eps. ``None`` unregisters."""
        if queries is None:
            self._queries = self._table = self._table_eps = None
            return
        if self.dim > self.TABLED_MAX_DIM:
            raise RuntimeError(f"registered route queries need a hidden size <= {self.TABLED_MAX_DIM}")
        if queries.dtype != torch.bfloat16 or queries.device != self.blocks.device or queries.dim() != 2 \
                or queries.shape[1] != self.dim or not queries.is_contiguous():
            raise RuntimeError(f"route queries must be a contiguous [R, {self.dim}] bf16 tensor on "
                               f"{self.blocks.device}, got {tuple(queries.shape)} {queries.dtype} {queries.device}")
        if norm_eps is None:
            raise RuntimeError("register_queries needs the eps the routes run with")
        rows = (self.max_completed_blocks + 3) // 4 * 4
        shape = (queries.shape[0], self.bt, rows)
        if self._table is None or tuple(self._table.shape) != shape:
            self._table = torch.zeros(shape, device=self.blocks.device, dtype=torch.float32)
        self._queries = queries
        self._table_eps = float(norm_eps)

    def validate_owner(self, partial: torch.Tensor) -> None:
        if tuple(partial.shape[:-1]) != self.token_shape or partial.shape[-1] != self.dim:
            raise RuntimeError(
                "Block AttnRes context shape changed within one model forward: "
                f"expected {(*self.token_shape, self.dim)}, got {tuple(partial.shape)}"
            )
        if partial.device != self.blocks.device:
            raise RuntimeError(f"Block AttnRes context device changed: {partial.device} vs {self.blocks.device}")
        if partial.dtype != self.blocks.dtype:
            raise RuntimeError(f"Block AttnRes context dtype changed: {partial.dtype} vs {self.blocks.dtype}")

    def completed_view(self) -> torch.Tensor:
        return self.blocks[: self.completed_count]

    def next_row(self) -> torch.Tensor:
        """The bank row the next appended source lands in: a producer can write its output here directly."""
        if self.completed_count >= self.max_completed_blocks:
            raise RuntimeError("Block AttnRes completed-block buffer overflow")
        return self.blocks[self.completed_count]

    def route(self, source: torch.Tensor, query: torch.Tensor, norm_eps: float, append_current: bool, *,
              norm_weight: torch.Tensor | None = None, out: torch.Tensor | None = None,
              mix_out: torch.Tensor | None = None) -> torch.Tensor:
        """Route over the completed rows + ``source`` (then append it when ``append_current``); with
        ``norm_weight`` the following RMSNorm is fused and ``out`` is the normalised mix."""
        src = source.reshape(self.bt, self.dim)
        self.validate_owner(source)
        completed = self.completed_count
        if append_current and completed >= self.max_completed_blocks:
            raise RuntimeError("Block AttnRes completed-block buffer overflow")
        in_place = completed < self.max_completed_blocks and src.data_ptr() == self.blocks[completed].data_ptr()
        if out is not None:
            out = out.reshape(self.bt, self.dim)
        if self._queries is not None:
            c = self.call_count
            if c >= self._queries.shape[0] or query.data_ptr() != self._queries[c].data_ptr() \
                    or float(norm_eps) != self._table_eps:
                raise RuntimeError(f"route {c} does not match the registered route queries / eps")
            result = ops.attnres_route_tabled(
                self.blocks if completed else None, completed, src if in_place else src.contiguous(),
                self._queries, c, self._table, self.rms_cache, norm_eps, source_in_bank=in_place and append_current,
                append_to=self.blocks[completed] if append_current and not in_place else None,
                norm_weight=norm_weight, norm_eps=norm_eps, out=out, mix_out=mix_out)
            if append_current:
                self.completed_count += 1
            self.call_count += 1
            return result.view(*self.token_shape, self.dim)
        cached = completed if self._rms_eps == norm_eps else 0  # cached rows hold 1 / rms at this eps
        self._rms_eps = norm_eps
        if in_place:
            result = ops.attnres_route(self.blocks, completed + 1, query, norm_eps, norm_weight=norm_weight,
                                       norm_eps=norm_eps, out=out, mix_out=mix_out, rms_cache=self.rms_cache,
                                       cached=cached)
        else:
            result = ops.attnres_route(
                self.blocks if completed else None, completed, query, norm_eps, source=src.contiguous(),
                append_to=self.blocks[completed] if append_current else None, norm_weight=norm_weight,
                norm_eps=norm_eps, out=out, mix_out=mix_out, rms_cache=self.rms_cache, cached=cached)
        if append_current:
            self.completed_count += 1
        self.call_count += 1
        return result.view(*self.token_shape, self.dim)


def fused_full_attnres(state: FusedBlockAttnResContext, source: torch.Tensor, query: torch.Tensor,
                       norm_eps: float, append_current: bool) -> torch.Tensor:
    """Route ``source`` with every completed bank row (training_attnres_kernels.py:2826)."""
    return state.route(source, query, float(norm_eps), bool(append_current))


def forward_layers_full(layers, x: torch.Tensor, queries: torch.Tensor, eps: float, state: FusedBlockAttnResContext,
                        out_norm_weight: torch.Tensor, router_states=None) -> torch.Tensor:
    """The Full AttnRes layer schedule (servers/sgl/src/zonos3_sgl/models/training_attnres.py:59-78; lm.py:699-721):
    before each sublayer one route over the bank with the sublayer's RMSNorm fused (attention_norm, ffn_norm), the
    sublayer's input appended to the bank by the same kernel; a final route with out_norm. ``layers`` expose
    ``attention_norm.weight``, ``ffn_norm.weight``, ``attention.forward(x)`` and ``feed_forward.forward(x,
    router_states) -> (out, router_states)`` (MoE) or ``feed_forward.forward(x)`` (dense, ``is_moe`` False).
    Returns the normalised final mix [T, D]. The 2L+1 route queries are registered with the context, so each route
    leaves the next route's logits in the context's table."""
    state.reset()
    if queries.dtype == torch.bfloat16 and queries.is_contiguous() and queries.device == state.blocks.device \
            and state.dim <= state.TABLED_MAX_DIM:
        state.register_queries(queries, eps)
    else:
        state.register_queries(None)
    source = x
    for i, layer in enumerate(layers):
        h = state.route(source, queries[2 * i], eps, True, norm_weight=layer.attention_norm.weight)
        attention_out = layer.attention.forward(h)
        h = state.route(attention_out, queries[2 * i + 1], eps, True, norm_weight=layer.ffn_norm.weight)
        if getattr(layer, "is_moe", True):
            source, router_states = layer.feed_forward.forward(h, router_states)
        else:
            source = layer.feed_forward.forward(h)
            router_states = None
    return state.route(source, queries[-1], eps, False, norm_weight=out_norm_weight)

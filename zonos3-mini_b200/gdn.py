"""``OriginalGDN``: the gated-DeltaNet mixer with the reference's forward signature, checkpoint names and cache
methods (servers/sgl/src/zonos3_sgl/models/gdn.py:121-450), on the B200 kernels.

forward(x [N, D] bf16) reads ``get_global_ctx().batch`` like the reference. Per call:

    mixed = x @ in_proj^T                                    (cuBLAS, as the reference)
    q, k, v, g, beta = zb_gdn_prologue(mixed, conv state)    (conv + SiLU, L2 norms, gate, beta; history update)
    o = zb_gdn_decode_step(...)        decode: one recurrent update per request, state updated in place
      | zb_gdn_chunk_prefill(...)      prefill / extend: chunked scan from the request's state
    gated = zb_gdn_gated_norm(o, z, out_weight)              (RMSNorm * SiLU(z))
    y = gated @ wo^T                                         (cuBLAS)

``fused_in_proj = True`` (class or instance attribute) runs a decode batch's in_proj GEMM and prologue as one
tcgen05 kernel instead (zb_gdn_in_proj_decode: the in_proj output never reaches global memory). It is off by
default: on a B200 at the 256-stream decode shape the cuBLAS GEMM plus the prologue kernel take 18.8 us per layer
and the fused kernel 31 us (its GEMM alone runs 13.7 us against cuBLAS's 9.7 us).

State is exact per request: the recurrence is the reference oracle's per-token update (lm.py:576-582), so a
decode step costs one state read + write instead of the server's 64-row window replay (gdn.py:329-355). The
state pool is V-first fp32 [capacity, H, dv, dk] (LMCache.gdn_state's layout) and the conv history is
[capacity, 3 * inner, 3] (LMCache.conv_state's). Requests address rows through their slot (``table_idx``);
nothing is gathered or scattered around the kernels.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn.functional as F

from . import ops
from .base import BaseOP, Weight
from .core import get_global_ctx

CONV_WIDTH = 4
CHUNK = 64  # the chunk length of the reference's training kernel and of the padded prefill layout


def chunk_tables(lengths: list[int], device) -> tuple[torch.Tensor, torch.Tensor]:
    """(cu_seqlens [n + 1], chunk indices [chunks, 2] = (sequence, chunk within it)) of packed sequences of
    ``lengths`` rows, int32 on ``device`` in one copy (servers/sgl/src/zonos3_sgl/models/gdn.py:49-59). The B200
    chunked prefill needs only cu_seqlens; the chunk indices are kept for callers of the reference interface."""
    cu = [0]
    chunks: list[int] = []
    for i, n in enumerate(lengths):
        cu.append(cu[-1] + n)
        for j in range(-(-n // CHUNK)):
            chunks += (i, j)
    packed = torch.tensor(cu + chunks, dtype=torch.int32).to(device)
    return packed[: len(cu)], packed[len(cu):].view(-1, 2)


@dataclass(frozen=True)
class PrefillLayout:
    """Static tables of a padded prefill of fresh requests (the reference's PrefillLayout, gdn.py:62-104): request i
    owns ``CHUNK * (whole[i] + 1)`` rows of the batch from ``starts[i]``, its real rows first (more than
    ``CHUNK * whole[i]``, at most all of them), padding after. Every tensor's shape depends on ``whole`` only, so a
    forward over the layout can be captured in a CUDA graph and replayed for any real lengths that fit it."""

    whole: tuple[int, ...]
    starts: torch.Tensor  # [b] int64: first batch row of each request
    cu_seqlens: torch.Tensor  # [b + 1] int32: the padded blocks as packed sequences
    seq_of_token: torch.Tensor  # [N] int32: request of each batch row
    row_in_seq: torch.Tensor  # [N] int64: position of each batch row within its request's block
    fresh: torch.Tensor  # [b] uint8 ones: every request starts from a zero state

    @classmethod
    def build(cls, whole: list[int], device) -> "PrefillLayout":
        sizes = [CHUNK * (w + 1) for w in whole]
        cu = [0]
        for n in sizes:
            cu.append(cu[-1] + n)
        dev = torch.device(device)
        return cls(
            whole=tuple(int(w) for w in whole),
            starts=torch.tensor(cu[:-1], dtype=torch.int64, device=dev),
            cu_seqlens=torch.tensor(cu, dtype=torch.int32, device=dev),
            seq_of_token=torch.tensor([i for i, n in enumerate(sizes) for _ in range(n)], dtype=torch.int32,
                                      device=dev),
            row_in_seq=torch.tensor([r for n in sizes for r in range(n)], dtype=torch.int64, device=dev),
            fresh=torch.ones(len(sizes), dtype=torch.uint8, device=dev),
        )

    @property
    def rows(self) -> int:
        return sum(CHUNK * (w + 1) for w in self.whole)

    def tensors(self) -> list[torch.Tensor]:
        """The layout's device tables (what a graph replay reads)."""
        return [self.starts, self.cu_seqlens, self.seq_of_token, self.row_in_seq, self.fresh]


@dataclass
class PrefillInputs:
    """A padded prefill's GDN inputs (``batch.gdn_prefill``, gdn.py:107-113): the layout and the graph's per-replay
    buffers."""

    layout: PrefillLayout
    slots: torch.Tensor  # [b] int64: the requests' state slots
    lengths: torch.Tensor  # [b] int64: the requests' real rows


class OriginalGDN(BaseOP):
    _fp32 = ("A_log", "dt_bias")
    fused_in_proj = False  # decode: zb_gdn_in_proj_decode instead of cuBLAS in_proj + prologue (module docstring)

    def __init__(self, config, layer_id: int):
        H, d = getattr(config, "gdn_num_heads", 4), getattr(config, "gdn_head_dim", 128)
        inner = H * d
        self._layer_id = layer_id
        self._hidden = config.hidden_size
        self._heads, self._head_dim = H, d
        self.in_proj = Weight((4 * inner + 2 * H, config.hidden_size))
        self.conv = Weight((3 * inner, 1, CONV_WIDTH))
        self.out_weight = torch.empty(d)
        self.A_log = torch.empty(H, dtype=torch.float32)
        self.dt_bias = torch.empty(H, dtype=torch.float32)
        self.wo = Weight((config.hidden_size, inner))
        self._capacity = 0
        self._static_mode = False
        self._graph_slots: torch.Tensor | None = None
        self._static: dict[int, tuple[torch.Tensor, torch.Tensor]] = {}

    # ------------------------------------------------------------------ caches
    def allocate_cache(self, capacity, device, dtype):
        if self._capacity:
            raise RuntimeError("GDN cache already allocated")
        H, d = self._heads, self._head_dim
        self._conv_state = torch.zeros((capacity, 3 * H * d, CONV_WIDTH - 1), device=device, dtype=torch.bfloat16)
        self._recurrent_state = torch.zeros((capacity, H, d, d), device=device, dtype=torch.float32)
        self._owners = [None] * capacity
        self._lengths = [0] * capacity
        self._capacity = capacity

    # ------------------------------------------------------------------ CUDA graphs (decode)
    @staticmethod
    def static_tables(device, bs_list):
        """Per decode batch size: (cu_seqlens = 0..bs, sequence of every token = 0..bs-1), built once and shared by
        every layer, so a captured decode step reads only device tables."""
        tables = {}
        for bs in bs_list:
            cu = torch.arange(bs + 1, device=device, dtype=torch.int32)
            tables[bs] = (cu, cu[:-1].clone())
        return tables

    def enable_graph_decode(self, slots: torch.Tensor, tables) -> None:
        """``slots`` is the engine's static [max_bs] int64 slot buffer (padding rows = -1)."""
        self._graph_slots = slots
        self._static.update(tables)

    @staticmethod
    def pin_fla_cache(static_tensors, pinned: dict) -> int:
        """No third-party tensor caches to keep alive: the kernels take their tables as plain device pointers."""
        return 0

    def set_static_mode(self, enabled: bool) -> None:
        self._static_mode = bool(enabled)

    def note_graph_forward(self, reqs) -> None:
        for r in reqs:
            self._owners[r.table_idx] = (r.uid, r.is_cfg_uncond)
            self._lengths[r.table_idx] = r.device_len

    # ------------------------------------------------------------------ forward
    def forward(self, x: torch.Tensor) -> torch.Tensor:
        batch = get_global_ctx().batch
        if batch.is_decode and self._static_mode:
            return self._forward_decode_static(x, batch.padded_size)
        if getattr(batch, "gdn_prefill", None) is not None:
            return self._forward_prefill_static(x, batch.gdn_prefill)
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError("GDN ragged path cannot be captured; graphs use the static decode / prefill paths")
        reqs = batch.reqs
        slots = [r.table_idx for r in reqs]
        lengths = [r.extend_len for r in reqs]
        if (
            not self._capacity
            or len(set(slots)) != len(slots)
            or any(s < 0 or s >= self._capacity for s in slots)
            or any(n <= 0 for n in lengths)
            or sum(lengths) != x.shape[0]
        ):
            raise RuntimeError("Invalid GDN request slots or packed lengths")
        if batch.is_decode and any(n != 1 for n in lengths):
            raise RuntimeError("GDN decode expects one new token per request")
        for r in reqs:
            s = r.table_idx
            owner = (r.uid, r.is_cfg_uncond)
            if r.cached_len and (self._owners[s] != owner or self._lengths[s] != r.cached_len):
                raise RuntimeError(
                    f"GDN layer {self._layer_id}: missing/stale state at slot {s}; "
                    f"expected {(owner, r.cached_len)}, found {(self._owners[s], self._lengths[s])}"
                )
        cu = [0]
        for n in lengths:
            cu.append(cu[-1] + n)
        seq_of_token = [i for i, n in enumerate(lengths) for _ in range(n)]
        fresh = [0 if r.cached_len else 1 for r in reqs]
        dev = x.device
        host = torch.tensor(cu + seq_of_token, dtype=torch.int32).pin_memory()
        tables = host.to(dev, non_blocking=True)
        cu_t, sot_t = tables[: len(cu)], tables[len(cu):]
        slots_t = torch.tensor(slots, dtype=torch.int64).pin_memory().to(dev, non_blocking=True)
        fresh_t = torch.tensor(fresh, dtype=torch.uint8).pin_memory().to(dev, non_blocking=True)
        y = self._run(x, cu_t, sot_t, slots_t, fresh_t, decode=batch.is_decode,
                      any_fresh=any(fresh))
        for r in reqs:
            self._owners[r.table_idx] = (r.uid, r.is_cfg_uncond)
            self._lengths[r.table_idx] = r.device_len
        return y

    def _forward_decode_static(self, x, bs):
        """One new row per padded request; every tensor shape depends on ``bs`` only and the slot buffer's padding
        rows (-1) touch no state: capturable in a CUDA graph."""
        if self._graph_slots is None or bs not in self._static:
            raise RuntimeError(f"GDN static decode is not prepared for batch size {bs}")
        cu, sot = self._static[bs]
        return self._run(x, cu, sot, self._graph_slots[:bs], None, decode=True, any_fresh=False)

    def _forward_prefill_static(self, x, inputs: PrefillInputs):
        """A padded prefill of fresh requests (PrefillLayout): one chunked pass over every request's padded block
        from a zero state. Padding rows are zeroed and enter the recurrence as identity updates (decay 1, beta 0),
        so each request's final state is its state after its real rows; its conv history is rewritten from its last
        CONV_WIDTH - 1 real rows (zeros before its first). Every shape depends on the layout only (capturable)."""
        layout, slots = inputs.layout, inputs.slots
        if x.shape[0] != layout.rows or slots.numel() != len(layout.whole):
            raise RuntimeError(f"padded prefill of {x.shape[0]} rows does not match its layout ({layout.rows} rows, "
                               f"{len(layout.whole)} requests)")
        H, d = self._heads, self._head_dim
        inner = H * d
        lengths = inputs.lengths.to(torch.int64)
        real = layout.row_in_seq < lengths.index_select(0, layout.seq_of_token.to(torch.int64))
        x = x * real.unsqueeze(1).to(x.dtype)
        mixed = F.linear(x, self.in_proj.weight)
        q, k, v, g, beta = ops.gdn_prologue(mixed, self.conv.weight, self.A_log, self.dt_bias, layout.cu_seqlens,
                                            layout.seq_of_token, slots, self._conv_state, heads=H, head_dim=d,
                                            fresh=layout.fresh)
        keep = real.unsqueeze(1)
        g = g.masked_fill(~keep, 0.0)
        beta = beta.masked_fill(~keep, 0.0)
        self._recurrent_state.index_fill_(0, slots, 0.0)
        o, _ = ops.gdn_chunk_prefill(q, k, v, g, beta, layout.cu_seqlens, initial_state=self._recurrent_state,
                                     final_state=self._recurrent_state, state_slots=slots)
        # conv history: the q/k/v channels of the last CONV_WIDTH - 1 real rows, oldest first
        W1 = CONV_WIDTH - 1
        offs = torch.arange(-W1, 0, device=x.device, dtype=torch.int64)
        rows = layout.starts.unsqueeze(1) + lengths.unsqueeze(1) + offs.unsqueeze(0)  # [b, W1]
        inside = rows >= layout.starts.unsqueeze(1)
        hist = mixed[:, : 3 * inner].index_select(0, rows.clamp(min=0).reshape(-1)).view(-1, W1, 3 * inner)
        hist = hist * inside.unsqueeze(2).to(hist.dtype)
        self._conv_state.index_copy_(0, slots, hist.transpose(1, 2).to(self._conv_state.dtype))
        gated = ops.gdn_gated_norm(o, mixed[:, 3 * inner:4 * inner], self.out_weight, 1e-5)
        return F.linear(gated, self.wo.weight)

    def _fused_decode(self, x) -> bool:
        """Whether a decode batch runs the fused in_proj + prologue kernel (opt-in; the shapes it takes)."""
        H, d = self._heads, self._head_dim
        return self.fused_in_proj and x.shape[1] % 128 == 0 and (H * d) % 128 == 0 and d in (64, 128) and H <= 64

    def _run(self, x, cu, seq_of_token, slots, fresh, *, decode: bool, any_fresh: bool):
        H, d = self._heads, self._head_dim
        inner = H * d
        if decode and not any_fresh and self._fused_decode(x):
            q, k, v, z, g, beta = ops.gdn_in_proj_decode(x, self.in_proj.weight, self.conv.weight, self.A_log,
                                                         self.dt_bias, slots, self._conv_state, heads=H, head_dim=d)
            o = ops.gdn_decode_step(q, k, v, g, beta, self._recurrent_state, slots=slots)
            return F.linear(ops.gdn_gated_norm(o, z, self.out_weight, 1e-5), self.wo.weight)
        mixed = F.linear(x, self.in_proj.weight)
        if decode and not any_fresh:  # one token per request: the history update rides in the prologue kernel
            q, k, v, g, beta = ops.gdn_prologue_decode(mixed, self.conv.weight, self.A_log, self.dt_bias, slots,
                                                       self._conv_state, heads=H, head_dim=d)
        else:
            q, k, v, g, beta = ops.gdn_prologue(mixed, self.conv.weight, self.A_log, self.dt_bias, cu, seq_of_token,
                                                slots, self._conv_state, heads=H, head_dim=d, fresh=fresh)
        if decode:
            o = ops.gdn_decode_step(q, k, v, g, beta, self._recurrent_state, slots=slots)
        else:
            if any_fresh:  # a request without cached rows starts from a zero state
                rows = slots[fresh.bool()]
                self._recurrent_state.index_fill_(0, rows, 0.0)
            o, _ = ops.gdn_chunk_prefill(q, k, v, g, beta, cu, initial_state=self._recurrent_state,
                                         final_state=self._recurrent_state, state_slots=slots)
        gated = ops.gdn_gated_norm(o, mixed[:, 3 * inner:4 * inner], self.out_weight, 1e-5)
        return F.linear(gated, self.wo.weight)

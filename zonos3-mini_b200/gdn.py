"""``OriginalGDN``: the gated-DeltaNet mixer with the reference's forward signature, checkpoint names and cache
methods (servers/sgl/src/zonos3_sgl/models/gdn.py:121-450), on the B200 kernels.

forward(x [N, D] bf16) reads ``get_global_ctx().batch`` like the reference. Per call:

    mixed = x @ in_proj^T                                    (cuBLAS, as the reference)
    q, k, v, g, beta = zb_gdn_prologue(mixed, conv state)    (conv + SiLU, L2 norms, gate, beta; history update)
    o = zb_gdn_decode_step(...)        decode: one recurrent update per request, state updated in place
      | zb_gdn_chunk_prefill(...)      prefill / extend: chunked scan from the request's state
    gated = zb_gdn_gated_norm(o, z, out_weight)              (RMSNorm * SiLU(z))
    y = gated @ wo^T                                         (cuBLAS)

State is exact per request: the recurrence is the reference oracle's per-token update (lm.py:576-582), so a
decode step costs one state read + write instead of the server's 64-row window replay (gdn.py:329-355). The
state pool is V-first fp32 [capacity, H, dv, dk] (LMCache.gdn_state's layout) and the conv history is
[capacity, 3 * inner, 3] (LMCache.conv_state's). Requests address rows through their slot (``table_idx``);
nothing is gathered or scattered around the kernels.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from . import ops
from .base import BaseOP, Weight
from .core import get_global_ctx

CONV_WIDTH = 4


class OriginalGDN(BaseOP):
    _fp32 = ("A_log", "dt_bias")

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
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError("GDN ragged path cannot be captured; graphs use the static decode path")
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

    def _run(self, x, cu, seq_of_token, slots, fresh, *, decode: bool, any_fresh: bool):
        H, d = self._heads, self._head_dim
        inner = H * d
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

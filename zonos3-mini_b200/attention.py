"""The global-attention layer of the hybrid stack (one layer in four at cfg5) with the reference's forward signature
and checkpoint names (``Attention``, servers/sgl/src/zonos3_sgl/models/zonos3.py:258-390), and the slot-indexed KV
pool it reads (``SlotKVPool``; the FA backend's page-size-1 cache, servers/sgl/src/zonos3_sgl/attention/fa.py and
kvcache/mha_pool.py).

forward(x [N, D] bf16) reads ``get_global_ctx().batch.attn_metadata`` and ``get_global_ctx().attn_backend``:

    p = x @ [wq; wkv; gater]^T                              (one cuBLAS GEMM over the concatenated weights)
    decode:  q = zb_gqa_prologue_decode(p)                  (q / k RMSNorm eps 1e-6, q x |temp|, interleaved RoPE,
                                                             k and v stored at the rows' cache slots)
             o = zb_gqa_decode(q, cache, page_table, gate)  (tcgen05 decode attention, unsplit, the output gate
                                                             sigmoid(gate) applied in its store)
    prefill: the same prologue in torch, zb_kv_store, causal softmax attention per request in torch
    y = (o * sigmoid(gate)) @ wo^T                          (cuBLAS; decode: the gate already applied)

The prefill attention is plain torch: the north_star path is the decode step, and the reference runs its prefill
attention through flash_attn_varlen_func (fa.py), a library kernel this package does not replace.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from . import ops
from .base import BaseOP, Weight
from .core import get_global_ctx

QK_NORM_EPS = 1e-6  # zonos3.py:362-363


class SlotKVPool:
    """K and V caches of every global-attention layer: ``[slots, kv_heads, head_dim]`` bf16 each, one token per slot
    (page size 1). ``layer_ids`` lists the model's attention layers; a layer's cache is ``k(layer_id)``."""

    def __init__(self, layer_ids, slots: int, kv_heads: int, head_dim: int, device, dtype=torch.bfloat16):
        self.layer_ids = list(layer_ids)
        self._index = {layer: i for i, layer in enumerate(self.layer_ids)}
        shape = (len(self.layer_ids), slots, kv_heads, head_dim)
        self.k_buffer = torch.zeros(shape, device=device, dtype=dtype)
        self.v_buffer = torch.zeros(shape, device=device, dtype=dtype)
        self.slots = slots

    def k(self, layer_id: int) -> torch.Tensor:
        return self.k_buffer[self._index[layer_id]]

    def v(self, layer_id: int) -> torch.Tensor:
        return self.v_buffer[self._index[layer_id]]


def rope_interleaved(x: torch.Tensor, positions: torch.Tensor, theta: float) -> torch.Tensor:
    """Interleaved-pair rotary embedding (is_neox=False): pair (2i, 2i+1) rotated by position * theta^(-2i/hd),
    in fp32, rounded to x's dtype."""
    hd = x.shape[-1]
    freqs = theta ** (-torch.arange(0, hd, 2, device=x.device, dtype=torch.float32) / hd)
    ang = positions.float()[:, None] * freqs[None, :]
    cos, sin = ang.cos()[:, None, :], ang.sin()[:, None, :]
    pairs = x.float().reshape(*x.shape[:-1], hd // 2, 2)
    a, b = pairs[..., 0], pairs[..., 1]
    return torch.stack((a * cos - b * sin, a * sin + b * cos), -1).flatten(-2).to(x.dtype)


class Attention(BaseOP):
    """Gated GQA with q / k RMSNorm and a learned |temperature| on q (zonos3.py:258-390)."""

    def __init__(self, config, layer_id: int):
        self.num_heads = config.num_qo_heads
        self.num_kv_heads = config.num_kv_heads
        self.head_dim = config.head_dim
        self._layer_id = layer_id
        self._theta = float(getattr(config, "rope_theta", 10000.0))
        D = config.hidden_size
        self.wq = Weight((self.num_heads * self.head_dim, D))
        self.wkv = Weight((2, self.num_kv_heads * self.head_dim, D))
        self.wo = Weight((D, self.num_heads * self.head_dim))
        self.temp = torch.ones(1, self.num_heads, 1)
        self.gater = Weight((self.num_heads, D))
        self._proj = None  # [wq; wk; wv; gater] concatenated (prepare())
        self._temp = None
        self._q = self._o = None

    def prepare(self) -> None:
        """Builds the concatenated projection weight (call after loading and moving the weights, before capture)."""
        kv = self.num_kv_heads * self.head_dim
        self._proj = torch.cat([self.wq.weight, self.wkv.weight.reshape(2 * kv, -1), self.gater.weight]).contiguous()
        self._temp = self.temp.reshape(-1).to(self._proj.dtype).contiguous()

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        ctx = get_global_ctx()
        batch, pool = ctx.batch, ctx.attn_backend
        meta = batch.attn_metadata
        if pool is None or meta is None:
            raise RuntimeError("Attention needs the batch's attn_metadata and the KV pool (get_global_ctx().attn_backend)")
        if self._proj is None or self._proj.device != x.device:
            if torch.cuda.is_current_stream_capturing():
                raise RuntimeError("Attention.prepare() must run before graph capture")
            self.prepare()
        n, H, Hkv, hd = x.shape[0], self.num_heads, self.num_kv_heads, self.head_dim
        kc, vc = pool.k(self._layer_id), pool.v(self._layer_id)
        p = F.linear(x, self._proj)  # q | k | v | gate
        gate = p[:, (H + 2 * Hkv) * hd:]
        if batch.is_decode:  # the output gate rides in the attention kernel's store
            q = ops.gqa_prologue_decode(p, self._temp, meta.positions, kc, vc, meta.out_loc, heads=H, kv_heads=Hkv,
                                        rope_theta=self._theta, eps=QK_NORM_EPS)
            o = ops.gqa_decode(q, kc, vc, meta.page_table, meta.cache_seqlens, softmax_scale=hd ** -0.5, gate=gate)
        else:
            o = self._prefill(p, kc, vc, meta).view(n, H, hd) * torch.sigmoid(gate).unsqueeze(-1)
        return F.linear(o.reshape(n, H * hd), self.wo.weight)

    def _prefill(self, p, kc, vc, meta):
        n, H, Hkv, hd = p.shape[0], self.num_heads, self.num_kv_heads, self.head_dim
        q = p[:, : H * hd].reshape(n, H, hd)
        k = p[:, H * hd:(H + Hkv) * hd].reshape(n, Hkv, hd)
        v = p[:, (H + Hkv) * hd:(H + 2 * Hkv) * hd].reshape(n, Hkv, hd).contiguous()
        q = F.rms_norm(q, (hd,), eps=QK_NORM_EPS) * self._temp.abs().view(1, H, 1)
        k = F.rms_norm(k, (hd,), eps=QK_NORM_EPS)
        q = rope_interleaved(q, meta.positions, self._theta)
        k = rope_interleaved(k, meta.positions, self._theta).contiguous()
        ops.kv_store(kc, vc, meta.out_loc, k, v)
        cu = meta.cu_seqlens_q
        if cu is None:
            raise RuntimeError("a prefill batch needs attn_metadata.cu_seqlens_q")
        lengths = meta.cache_seqlens.tolist()
        out = torch.empty(n, H, hd, device=p.device, dtype=p.dtype)
        for b in range(len(cu) - 1):
            rows = cu[b + 1] - cu[b]
            if rows == 0:
                continue
            total = lengths[b]
            table = meta.page_table[b, :total].long()
            key = kc[table].repeat_interleave(H // Hkv, 1).transpose(0, 1)
            value = vc[table].repeat_interleave(H // Hkv, 1).transpose(0, 1)
            # row i of this request sits at key position total - rows + i and sees keys up to it
            mask = torch.arange(total, device=p.device)[None, :] <= (total - rows + torch.arange(rows, device=p.device))[:, None]
            o = F.scaled_dot_product_attention(q[cu[b]:cu[b + 1]].transpose(0, 1), key, value, attn_mask=mask,
                                               scale=hd ** -0.5)
            out[cu[b]:cu[b + 1]] = o.transpose(0, 1)
        return out

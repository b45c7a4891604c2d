"""Decode-attention oracle (CPU, float32): the attention core of a global-attention layer for one new query row per
request over its cached keys, with the cache addressed through a page table of token slots.

Restates model/src/zonos3/reference/lm.py:526-531 (GQA: query head h reads KV head h // (Hq / Hkv), softmax scale
head_dim ** -0.5, causal mask — for a decode row every cached key is visible) and the cache addressing of the FA
backend (servers/sgl/src/zonos3_sgl/attention/fa.py:64-81: store row i at slot out_loc[i], read key position j of
request b at slot page_table[b, j], cache_seqlens[b] keys). The product kernel's attention library counterpart is
FlashAttention-3's flash_attn_with_kvcache (sgl-kernel, not vendored in the reference), whose published algorithm
is exact softmax attention; parity is therefore against this exact fp32 restatement within a bf16 tolerance.
Test infrastructure only (see ``oracle/__init__.py``).
"""

from __future__ import annotations

import torch


def store_kv(k_cache, v_cache, slots, k, v):
    """k_cache[slots[i]] = k[i], v_cache[slots[i]] = v[i] for each slot in range (store.cu:28-50), in place."""
    keep = (slots >= 0) & (slots < k_cache.shape[0])
    k_cache[slots[keep].long()] = k[keep]
    v_cache[slots[keep].long()] = v[keep]


def decode_attention(q, k_cache, v_cache, page_table, seq_lens, scale=None):
    """out[b, h] = softmax(q[b, h] . K_b^T * scale) V_b (fp32), K_b / V_b the cache rows page_table[b, :seq_lens[b]]
    of KV head h // (Hq / Hkv). An entry of the table outside the cache masks its key; a request without keys gets
    zeros. q [B, Hq, hd]; caches [slots, Hkv, hd]; returns [B, Hq, hd] float32."""
    B, Hq, hd = q.shape
    Hkv = k_cache.shape[1]
    rep = Hq // Hkv
    scale = hd ** -0.5 if scale is None else scale
    out = torch.zeros(B, Hq, hd, dtype=torch.float32)
    for b in range(B):
        n = min(int(seq_lens[b]), page_table.shape[1])
        idx = page_table[b, :n].long()
        idx = idx[(idx >= 0) & (idx < k_cache.shape[0])]
        if len(idx) == 0:
            continue
        key = k_cache[idx].float().repeat_interleave(rep, 1).transpose(0, 1)  # [Hq, n, hd]
        value = v_cache[idx].float().repeat_interleave(rep, 1).transpose(0, 1)
        w = torch.softmax(torch.einsum("hd,hnd->hn", q[b].float(), key) * scale, dim=-1)
        out[b] = torch.einsum("hn,hnd->hd", w, value)
    return out

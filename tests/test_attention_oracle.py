"""CPU: the decode-attention oracle (slot-indexed cache through a page table) equals the reference's contiguous-cache
attention math (model/src/zonos3/reference/lm.py:524-531: repeat_interleave GQA, causal mask, scale hd ** -0.5) for
the last query row, and the KV store places rows where the page table later finds them."""

from __future__ import annotations

import torch
import torch.nn.functional as F

from oracle import attention


def test_decode_attention_matches_contiguous_sdpa():
    gen = torch.Generator().manual_seed(3)
    B, Hq, Hkv, hd, slots = 3, 8, 2, 64, 200
    lens = [1, 17, 70]
    k_cache = torch.zeros(slots, Hkv, hd)
    v_cache = torch.zeros(slots, Hkv, hd)
    table = torch.full((B, 80), -1, dtype=torch.int32)
    perm = torch.randperm(slots, generator=gen)
    used = 0
    keys, values = [], []
    for b, n in enumerate(lens):
        k = torch.randn(n, Hkv, hd, generator=gen)
        v = torch.randn(n, Hkv, hd, generator=gen)
        loc = perm[used: used + n].to(torch.int32)
        used += n
        attention.store_kv(k_cache, v_cache, loc, k, v)
        table[b, :n] = loc
        keys.append(k)
        values.append(v)
    q = torch.randn(B, Hq, hd, generator=gen)
    got = attention.decode_attention(q, k_cache, v_cache, table, torch.tensor(lens, dtype=torch.int32))
    for b, n in enumerate(lens):
        rep = Hq // Hkv
        key = keys[b].repeat_interleave(rep, 1).transpose(0, 1)
        value = values[b].repeat_interleave(rep, 1).transpose(0, 1)
        pos = torch.tensor([n - 1])
        mask = torch.arange(n)[None, :] <= pos[:, None]
        ref = F.scaled_dot_product_attention(q[b][:, None], key, value, attn_mask=mask, scale=hd ** -0.5)[:, 0]
        torch.testing.assert_close(got[b], ref, rtol=1e-5, atol=1e-5)


def test_store_skips_out_of_range_slots():
    k_cache = torch.zeros(4, 1, 8)
    v_cache = torch.zeros(4, 1, 8)
    k = torch.ones(3, 1, 8)
    attention.store_kv(k_cache, v_cache, torch.tensor([2, -1, 4], dtype=torch.int32), k, 2 * k)
    assert k_cache[2].eq(1).all() and v_cache[2].eq(2).all()
    assert k_cache[[0, 1, 3]].eq(0).all()


def test_masked_entries_and_empty_requests():
    gen = torch.Generator().manual_seed(5)
    k_cache = torch.randn(10, 1, 8, generator=gen)
    v_cache = torch.randn(10, 1, 8, generator=gen)
    q = torch.randn(2, 2, 8, generator=gen)
    table = torch.tensor([[3, -1, 11, 5], [0, 1, 2, 3]], dtype=torch.int32)
    out = attention.decode_attention(q, k_cache, v_cache, table, torch.tensor([4, 0], dtype=torch.int32))
    ref = attention.decode_attention(q[:1], k_cache, v_cache, torch.tensor([[3, 5]], dtype=torch.int32),
                                     torch.tensor([2], dtype=torch.int32))
    torch.testing.assert_close(out[:1], ref)
    assert out[1].eq(0).all()

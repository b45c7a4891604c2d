"""GPU: GQA decode attention over a slot-indexed KV cache (zb_gqa_decode) and the KV store (zb_kv_store) through the
C ABI, against the fp32 oracle (oracle.attention): random caches addressed through a permuted page table, requests
of 0, 1, tile-edge and long lengths, masked table entries, unsplit / automatic / forced splits, head dims 32 (the
tiny config's attention), 64 and 128 and groups of 1, 2, 4 and 8 query heads per KV head. Attention output within
2e-2 (absolute + relative) of the fp32 oracle — the bf16 rounding of the output and of K and V already in the cache;
the store bit-exact."""

from __future__ import annotations

import pytest
import torch

from oracle import attention

pytestmark = pytest.mark.gpu

ATOL = RTOL = 2e-2


def _case(gen, B, Hq, Hkv, hd, lens, slots, width):
    k_cache = torch.randn(slots, Hkv, hd, generator=gen).bfloat16()
    v_cache = torch.randn(slots, Hkv, hd, generator=gen).bfloat16()
    q = (torch.randn(B, Hq, hd, generator=gen) * 1.5).bfloat16()
    table = torch.randint(0, slots, (B, width), generator=gen, dtype=torch.int32)
    for b in range(B):
        table[b, : lens[b]] = torch.randperm(slots, generator=gen)[: lens[b]].to(torch.int32)
    return q, k_cache, v_cache, table, torch.tensor(lens, dtype=torch.int32)


@pytest.mark.parametrize("Hq,Hkv,hd", [(16, 4, 128), (8, 8, 64), (16, 2, 64), (4, 2, 128), (16, 2, 128), (8, 8, 128),
                                       (8, 2, 32)])
@pytest.mark.parametrize("num_splits", [1, 0, 3])
def test_gqa_decode_matches_oracle(zb, Hq, Hkv, hd, num_splits):
    gen = torch.Generator().manual_seed(Hq * 131 + Hkv * 7 + hd + num_splits)
    lens = [0, 1, 31, 32, 33, 200, 1000, 517]
    # table width 1100: unsplit, a unit spans 9 tiles (one unit per CTA); split, 3 tiles (persistent CTAs)
    B, slots, width = len(lens), 4096, 1100
    q, kc, vc, table, seq = _case(gen, B, Hq, Hkv, hd, lens, slots, width)
    dev = torch.device("cuda")
    out = zb.ops.gqa_decode(q.to(dev), kc.to(dev), vc.to(dev), table.to(dev), seq.to(dev), num_splits=num_splits)
    ref = attention.decode_attention(q, kc, vc, table, seq)
    torch.testing.assert_close(out.float().cpu(), ref, atol=ATOL, rtol=RTOL)
    assert out[0].float().abs().max().item() == 0.0  # no keys: zero output


def test_gqa_decode_masked_entries_and_strides(zb):
    """Table entries outside the cache mask their key; q, out and the cache carry padded strides; page_table rows
    wider than the longest request; seq_lens past the table clamp to it."""
    gen = torch.Generator().manual_seed(11)
    B, Hq, Hkv, hd, slots, width = 5, 16, 4, 128, 600, 96
    lens = [96, 50, 7, 200, 64]  # 200 > width: clamped
    q, kc, vc, table, seq = _case(gen, B, Hq, Hkv, hd, [min(n, width) for n in lens], slots, width)
    seq = torch.tensor(lens, dtype=torch.int32)
    table[0, 5] = -1
    table[0, 40] = slots + 3
    table[2, :7] = -1  # every key of request 2 masked: zero output
    dev = torch.device("cuda")
    kpad = torch.zeros(slots, Hkv * hd + 64, dtype=torch.bfloat16)
    vpad = torch.zeros_like(kpad)
    kpad[:, : Hkv * hd] = kc.reshape(slots, -1)
    vpad[:, : Hkv * hd] = vc.reshape(slots, -1)
    kd = kpad.to(dev).as_strided((slots, Hkv, hd), (Hkv * hd + 64, hd, 1))
    vd = vpad.to(dev).as_strided((slots, Hkv, hd), (Hkv * hd + 64, hd, 1))
    qpad = torch.zeros(B, Hq * hd + 32, dtype=torch.bfloat16)
    qpad[:, : Hq * hd] = q.reshape(B, -1)
    qd = qpad.to(dev).as_strided((B, Hq, hd), (Hq * hd + 32, hd, 1))
    outbuf = torch.full((B, Hq * hd + 16), 7.0, dtype=torch.bfloat16, device=dev)
    out = outbuf.as_strided((B, Hq, hd), (Hq * hd + 16, hd, 1))
    for splits in (1, 2):
        zb.ops.gqa_decode(qd, kd, vd, table.to(dev), seq.to(dev), num_splits=splits, out=out)
        ref = attention.decode_attention(q, kc, vc, table, seq)
        torch.testing.assert_close(out.float().cpu(), ref, atol=ATOL, rtol=RTOL)
        assert out[2].float().abs().max().item() == 0.0
        assert outbuf[:, Hq * hd:].eq(7.0).all()  # the padding between rows is untouched


def test_gqa_decode_scale_and_errors(zb):
    gen = torch.Generator().manual_seed(2)
    q, kc, vc, table, seq = _case(gen, 2, 8, 2, 64, [40, 9], 128, 64)
    dev = torch.device("cuda")
    out = zb.ops.gqa_decode(q.to(dev), kc.to(dev), vc.to(dev), table.to(dev), seq.to(dev), softmax_scale=0.3)
    ref = attention.decode_attention(q, kc, vc, table, seq, scale=0.3)
    torch.testing.assert_close(out.float().cpu(), ref, atol=ATOL, rtol=RTOL)
    with pytest.raises(ValueError):
        zb.ops.gqa_decode(q.to(dev)[:, :5], kc.to(dev), vc.to(dev), table.to(dev), seq.to(dev))  # 5 heads over 2
    # splits that do not cover the table's columns are refused before any launch
    with pytest.raises(ValueError):
        zb._lib.call("zb_gqa_decode", q.to(dev).data_ptr(), 8 * 64, kc.to(dev).data_ptr(), vc.to(dev).data_ptr(),
                     2 * 64, 128, table.to(dev).data_ptr(), 64, seq.to(dev).data_ptr(), 64, 2, 8, 2, 64, 0.125, 1, 32,
                     None, 0, out.data_ptr(), 8 * 64, torch.cuda.current_stream().cuda_stream)
    with pytest.raises(RuntimeError):  # head dim 96 is not built
        zb._lib.call("zb_gqa_decode", q.to(dev).data_ptr(), 8 * 96, kc.to(dev).data_ptr(), vc.to(dev).data_ptr(),
                     2 * 96, 128, table.to(dev).data_ptr(), 64, seq.to(dev).data_ptr(), 64, 2, 8, 2, 96, 0.125, 1, 64,
                     None, 0, out.data_ptr(), 8 * 96, torch.cuda.current_stream().cuda_stream)


@pytest.mark.parametrize("Hkv,hd", [(4, 128), (2, 64)])
def test_kv_store_bit_exact(zb, Hkv, hd):
    gen = torch.Generator().manual_seed(Hkv + hd)
    slots, N = 300, 77
    kc = torch.randn(slots, Hkv, hd, generator=gen).bfloat16()
    vc = torch.randn(slots, Hkv, hd, generator=gen).bfloat16()
    k = torch.randn(N, Hkv, hd, generator=gen).bfloat16()
    v = torch.randn(N, Hkv, hd, generator=gen).bfloat16()
    loc = torch.randperm(slots, generator=gen)[:N].to(torch.int32)
    loc[4], loc[9] = -1, slots + 2  # not stored
    dev = torch.device("cuda")
    kd, vd = kc.to(dev), vc.to(dev)
    # k and v as views of one fused kv projection row: [N, 2 * Hkv * hd], stride 2 * Hkv * hd
    kv = torch.cat((k.reshape(N, -1), v.reshape(N, -1)), 1).to(dev)
    zb.ops.kv_store(kd, vd, loc.to(dev), kv.as_strided((N, Hkv, hd), (2 * Hkv * hd, hd, 1)),
                    kv.as_strided((N, Hkv, hd), (2 * Hkv * hd, hd, 1), Hkv * hd))
    attention.store_kv(kc, vc, loc, k, v)
    assert torch.equal(kd.cpu(), kc) and torch.equal(vd.cpu(), vc)


@pytest.mark.parametrize("num_splits", [1, 2])
def test_gqa_decode_rising_scores_and_masked_tiles(zb, num_splits):
    """Scores that rise along the keys (the running max moves by more than 2^8 several times, so the tensor-memory
    accumulator is rescaled) and leading tiles whose keys are all masked."""
    gen = torch.Generator().manual_seed(21)
    B, Hq, Hkv, hd, slots, width = 3, 16, 4, 128, 3000, 900
    lens = [900, 700, 300]
    q, kc, vc, table, seq = _case(gen, B, Hq, Hkv, hd, lens, slots, width)
    qd = q.float().reshape(B, Hkv, Hq // Hkv, hd).mean(2)  # a direction shared by the group's heads
    qd = qd / qd.norm(dim=-1, keepdim=True)
    kf = kc.float()
    for b in range(B):
        idx = table[b, : lens[b]].long()
        ramp = torch.linspace(0.0, 60.0, lens[b])[:, None, None]
        kf[idx] = kf[idx] * 0.1 + ramp * qd[b][None]
    kc = kf.bfloat16()
    table[1, :260] = -1  # request 1: its first two 128-key tiles hold no key
    dev = torch.device("cuda")
    out = zb.ops.gqa_decode(q.to(dev), kc.to(dev), vc.to(dev), table.to(dev), seq.to(dev), num_splits=num_splits)
    ref = attention.decode_attention(q, kc, vc, table, seq)
    torch.testing.assert_close(out.float().cpu(), ref, atol=ATOL, rtol=RTOL)


@pytest.mark.parametrize("Hq,Hkv,num_splits", [(16, 4, 1), (16, 4, 3), (8, 8, 1)])
def test_gqa_decode_many_units_per_cta(zb, Hq, Hkv, num_splits):
    """More (request, KV head, split) units than SMs, so each persistent CTA walks several units of ragged
    lengths (some empty, some a single partial tile) back to back."""
    gen = torch.Generator().manual_seed(Hq + Hkv + num_splits)
    B, hd, width = 96, 128, 640
    lens = torch.randint(0, width + 1, (B,), generator=gen)
    lens[::7] = 0
    lens[1::11] = 1
    lens[2::13] = width
    lens = lens.tolist()
    q, kc, vc, table, seq = _case(gen, B, Hq, Hkv, hd, lens, 20000, width)
    dev = torch.device("cuda")
    out = zb.ops.gqa_decode(q.to(dev), kc.to(dev), vc.to(dev), table.to(dev), seq.to(dev), num_splits=num_splits)
    ref = attention.decode_attention(q, kc, vc, table, seq)
    torch.testing.assert_close(out.float().cpu(), ref, atol=ATOL, rtol=RTOL)
    assert all(out[b].float().abs().max().item() == 0.0 for b in range(B) if lens[b] == 0)

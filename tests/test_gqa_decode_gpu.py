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
                     None, 0, out.data_ptr(), 8 * 64, None, 0, torch.cuda.current_stream().cuda_stream)
    with pytest.raises(RuntimeError):  # head dim 96 is not built
        zb._lib.call("zb_gqa_decode", q.to(dev).data_ptr(), 8 * 96, kc.to(dev).data_ptr(), vc.to(dev).data_ptr(),
                     2 * 96, 128, table.to(dev).data_ptr(), 64, seq.to(dev).data_ptr(), 64, 2, 8, 2, 96, 0.125, 1, 64,
                     None, 0, out.data_ptr(), 8 * 96, None, 0, torch.cuda.current_stream().cuda_stream)


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


def test_gqa_prologue_matches_torch(zb):
    """zb_gqa_prologue_decode against the server's steps in torch (F.rms_norm in bf16, x |temp|, interleaved RoPE
    in fp32 as oracle/lm.py restates it, then the KV store): q and the stored k within bf16 rounding, v bit-exact,
    out-of-range slots untouched."""
    import torch.nn.functional as F
    from oracle import lm as olm

    gen = torch.Generator().manual_seed(17)
    N, Hq, Hkv, hd, slots = 40, 16, 4, 128, 500
    width = (Hq + 2 * Hkv) * hd + Hq  # q | k | v | gate columns, as the fused projection lays them out
    proj = torch.randn(N, width, generator=gen).bfloat16()
    temp = (torch.randn(Hq, generator=gen) * 2).bfloat16()
    positions = torch.randint(0, 4000, (N,), generator=gen, dtype=torch.int32)
    out_loc = torch.randperm(slots, generator=gen)[:N].to(torch.int32)
    out_loc[3], out_loc[7] = -1, slots + 9
    dev = torch.device("cuda")
    kc = torch.zeros(slots, Hkv, hd, dtype=torch.bfloat16, device=dev)
    vc = torch.zeros_like(kc)
    q = zb.ops.gqa_prologue_decode(proj.to(dev), temp.to(dev), positions.to(dev), kc, vc, out_loc.to(dev),
                                   heads=Hq, kv_heads=Hkv)
    qr = proj[:, : Hq * hd].view(N, Hq, hd)
    kr = proj[:, Hq * hd: (Hq + Hkv) * hd].view(N, Hkv, hd)
    vr = proj[:, (Hq + Hkv) * hd: (Hq + 2 * Hkv) * hd].reshape(N, Hkv, hd)
    qn = F.rms_norm(qr.to(dev), (hd,), eps=1e-6) * temp.abs().to(dev).view(1, Hq, 1)
    kn = F.rms_norm(kr.to(dev), (hd,), eps=1e-6)
    q_ref = olm.rope_interleaved(qn.cpu(), positions.long(), 10000.0)
    k_ref = olm.rope_interleaved(kn.cpu(), positions.long(), 10000.0)
    torch.testing.assert_close(q.float().cpu(), q_ref.float(), atol=3e-2, rtol=2e-2)
    ok = (out_loc >= 0) & (out_loc < slots)
    torch.testing.assert_close(kc.float().cpu()[out_loc[ok].long()], k_ref[ok].float(), atol=3e-2, rtol=2e-2)
    assert torch.equal(vc.cpu()[out_loc[ok].long()], vr[ok])
    untouched = torch.ones(slots, dtype=torch.bool)
    untouched[out_loc[ok].long()] = False
    assert kc.cpu()[untouched].eq(0).all() and vc.cpu()[untouched].eq(0).all()


@pytest.mark.parametrize("Hq,Hkv,hd,num_splits", [(16, 4, 128, 1), (16, 4, 128, 0), (8, 2, 64, 1), (8, 2, 32, 2)])
def test_gqa_decode_output_gate(zb, Hq, Hkv, hd, num_splits):
    """The output gate in the kernel's store (the attention layer's o * sigmoid(gater(x))) against the ungated output
    gated in torch at the same bf16 rounding points: >= 99.9 % identical, the rest one bf16 step apart (the
    sigmoid's last fp32 bit); the gate is read through a row stride (a column slice of the projection output)."""
    gen = torch.Generator().manual_seed(Hq + hd + num_splits)
    lens = [0, 1, 129, 700]
    q, kc, vc, table, seq = _case(gen, len(lens), Hq, Hkv, hd, lens, 2048, 800)
    dev = torch.device("cuda")
    proj = torch.randn(len(lens), 3 * Hq, generator=gen).bfloat16().to(dev)
    gate = proj[:, Hq:2 * Hq]
    args = (q.to(dev), kc.to(dev), vc.to(dev), table.to(dev), seq.to(dev))
    plain = zb.ops.gqa_decode(*args, num_splits=num_splits)
    gated = zb.ops.gqa_decode(*args, num_splits=num_splits, gate=gate)
    ref = plain * torch.sigmoid(gate).unsqueeze(-1)
    assert (gated == ref).float().mean().item() >= 0.999
    torch.testing.assert_close(gated.float(), ref.float(), atol=0, rtol=2 ** -7)

"""GPU: the decode prologue (zb_gdn_prologue_decode, one kernel with the conv-state history update) against the
general prologue (zb_gdn_prologue + its history kernel) on the same decode batch: q, k, v, g, beta and the new
conv state bit-identical, padding rows (slot -1, slot past the rows) untouched. The general prologue itself is
checked against the oracle through the GDN module and the cfg1 LM tests."""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("H,D", [(16, 128), (4, 64), (2, 32)])
def test_decode_prologue_matches_general(zb, H, D):
    gen = torch.Generator().manual_seed(H * 7 + D)
    N, rows = 37, 48
    inner = H * D
    dev = torch.device("cuda")
    mixed = (torch.randn(N, 4 * inner + 2 * H + 4, generator=gen)).bfloat16().to(dev)[:, : 4 * inner + 2 * H]
    conv_w = (0.3 * torch.randn(3 * inner, 1, 4, generator=gen)).bfloat16().to(dev)
    A_log = torch.randn(H, generator=gen).to(dev)
    dt_bias = torch.randn(H, generator=gen).to(dev)
    slots = torch.randperm(rows, generator=gen)[:N].to(torch.int64)
    slots[3], slots[11] = -1, rows + 5  # padding rows
    slots = slots.to(dev)
    state0 = torch.randn(rows, 3 * inner, 3, generator=gen).bfloat16().to(dev)
    cu = torch.arange(N + 1, dtype=torch.int32, device=dev)
    sot = torch.arange(N, dtype=torch.int32, device=dev)
    s_ref, s_dec = state0.clone(), state0.clone()
    ref = zb.ops.gdn_prologue(mixed, conv_w, A_log, dt_bias, cu, sot, slots, s_ref, heads=H, head_dim=D)
    got = zb.ops.gdn_prologue_decode(mixed, conv_w, A_log, dt_bias, slots, s_dec, heads=H, head_dim=D)
    torch.cuda.synchronize()
    for a, b, name in zip(got, ref, ("q", "k", "v", "g", "beta")):
        assert torch.equal(a, b), name
    assert torch.equal(s_dec, s_ref)
    touched = torch.zeros(rows, dtype=torch.bool)
    valid = slots.cpu()[(slots.cpu() >= 0) & (slots.cpu() < rows)]
    touched[valid] = True
    assert torch.equal(s_dec.cpu()[~touched], state0.cpu()[~touched])
    # the new history of a slot: old entries 1, 2 then the token's qkv input
    i = 0
    sl = int(slots[i])
    exp = torch.cat([state0[sl, :, 1:], mixed[i, : 3 * inner].unsqueeze(1)], 1)
    assert torch.equal(s_dec[sl], exp)

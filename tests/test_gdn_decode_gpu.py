"""GPU parity of the recurrent decode kernel (zb_gdn_decode_step) against the CPU oracle (lm.py:576-582).

Tolerances (north_star): fp32 recurrent state within 1e-3 relative (max-abs over max-abs), bf16 outputs within
2e-2 relative (Frobenius). Inputs are identical bf16 / fp32 tensors on both sides."""

from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

from conftest import max_rel_err, rel_err
from oracle import gdn as ogdn

pytestmark = pytest.mark.gpu

STATE_TOL = 1e-3
OUT_TOL = 2e-2


def make_inputs(B, H, dk, dv, seed, state_scale=0.1):
    """cfg2's distributions: q, k ~ N(0,1) then L2-normalised per head, v ~ N(0,1) (bf16),
    beta = sigmoid(N(0,1)), g = -softplus(N(0,1)), state ~ N(0, state_scale^2)."""
    gen = torch.Generator().manual_seed(seed)
    q = F.normalize(torch.randn(B, H, dk, generator=gen), dim=-1).bfloat16()
    k = F.normalize(torch.randn(B, H, dk, generator=gen), dim=-1).bfloat16()
    v = torch.randn(B, H, dv, generator=gen).bfloat16()
    beta = torch.sigmoid(torch.randn(B, H, generator=gen))
    g = -F.softplus(torch.randn(B, H, generator=gen))
    state = torch.randn(B, H, dv, dk, generator=gen) * state_scale
    return q, k, v, g, beta, state


@pytest.mark.parametrize("B,H,dk", [(1, 1, 128), (3, 16, 128), (64, 16, 128), (5, 4, 64)])
def test_single_step_matches_oracle(zb, B, H, dk):
    q, k, v, g, beta, state = make_inputs(B, H, dk, dk, seed=B * 100 + H)
    ref_state, ref_out = ogdn.recurrent_step(state, q, k, v, g, beta, dk ** -0.5)
    dev = torch.device("cuda")
    d_state = state.to(dev)
    out = zb.ops.gdn_decode_step(q.to(dev), k.to(dev), v.to(dev), g.to(dev), beta.to(dev), d_state)
    torch.cuda.synchronize()
    assert max_rel_err(d_state, ref_state) < STATE_TOL
    assert rel_err(out.float(), ref_out) < OUT_TOL


def test_many_steps_track_the_recurrence(zb):
    """64 sequential steps from a zero state: the error must not grow beyond the tolerances."""
    B, H, dk, T = 4, 8, 128, 64
    dev = torch.device("cuda")
    steps = [make_inputs(B, H, dk, dk, seed=1000 + t) for t in range(T)]
    ref_state = torch.zeros(B, H, dk, dk)
    d_state = torch.zeros(B, H, dk, dk, device=dev)
    for q, k, v, g, beta, _ in steps:
        ref_state, ref_out = ogdn.recurrent_step(ref_state, q, k, v, g, beta, dk ** -0.5)
        out = zb.ops.gdn_decode_step(q.to(dev), k.to(dev), v.to(dev), g.to(dev), beta.to(dev), d_state)
    torch.cuda.synchronize()
    assert max_rel_err(d_state, ref_state) < STATE_TOL
    assert rel_err(out.float(), ref_out) < OUT_TOL


def test_slots_and_padding_rows(zb):
    """Streams address state rows through ``slots``; a negative slot is a graph-padding row that outputs zeros
    and leaves every state row untouched."""
    B, H, dk = 4, 2, 128
    q, k, v, g, beta, _ = make_inputs(B, H, dk, dk, seed=7)
    cache = torch.randn(6, H, dk, dk) * 0.1
    slots = torch.tensor([5, 0, -1, 2])
    dev = torch.device("cuda")
    d_cache = cache.to(dev)
    out = zb.ops.gdn_decode_step(q.to(dev), k.to(dev), v.to(dev), g.to(dev), beta.to(dev), d_cache,
                                 slots=slots.to(dev))
    torch.cuda.synchronize()
    expect = cache.clone()
    for b, s in enumerate(slots.tolist()):
        if s < 0:
            assert torch.all(out[b].cpu() == 0)
            continue
        st, o = ogdn.recurrent_step(cache[s], q[b], k[b], v[b], g[b], beta[b], dk ** -0.5)
        expect[s] = st
        assert rel_err(out[b].float(), o) < OUT_TOL
    assert max_rel_err(d_cache, expect) < STATE_TOL
    for s in (1, 3, 4):  # untouched rows are bit-identical
        assert torch.equal(d_cache[s].cpu(), cache[s])


def test_strided_views_of_a_packed_projection(zb):
    """q, k, v may be column slices of one packed [B, 3*H*d] activation (row stride 3*H*d)."""
    B, H, dk = 3, 4, 128
    q, k, v, g, beta, state = make_inputs(B, H, dk, dk, seed=9)
    packed = torch.cat([q.reshape(B, -1), k.reshape(B, -1), v.reshape(B, -1)], -1).cuda()
    inner = H * dk
    qv = packed[:, :inner].view(B, H, dk)
    kv = packed[:, inner:2 * inner].view(B, H, dk)
    vv = packed[:, 2 * inner:].view(B, H, dk)
    ref_state, ref_out = ogdn.recurrent_step(state, q, k, v, g, beta, dk ** -0.5)
    d_state = state.cuda()
    out = zb.ops.gdn_decode_step(qv, kv, vv, g.cuda(), beta.cuda(), d_state)
    torch.cuda.synchronize()
    assert max_rel_err(d_state, ref_state) < STATE_TOL
    assert rel_err(out.float(), ref_out) < OUT_TOL


def test_reference_golden_recurrence(zb, golden):
    """Drive the kernel with the reference's own q/k/v/decay/beta from the golden GDN layer (4 heads of 128) and
    compare the state after the 15 tokens with the reference's state, inputs rounded to bf16 on both sides."""
    gd = golden("gdn_tiny.npz")
    q, k, v = (gd[n].bfloat16() for n in ("gdn_q", "gdn_k", "gdn_v"))
    g = torch.log(gd["gdn_decay"])
    beta = gd["gdn_beta"]
    T, H, dk = q.shape
    ref_state, ref_out = ogdn.recurrent_scan(torch.zeros(H, dk, dk), q, k, v, g, beta, dk ** -0.5)
    # the reference itself (fp32 inputs) agrees with the bf16-input oracle to well within tolerance
    assert max_rel_err(ref_state, gd["state_final"]) < 2e-2
    d_state = torch.zeros(1, H, dk, dk, device="cuda")
    outs = []
    for t in range(T):
        outs.append(zb.ops.gdn_decode_step(q[t:t + 1].cuda(), k[t:t + 1].cuda(), v[t:t + 1].cuda(),
                                           g[t:t + 1].cuda(), beta[t:t + 1].cuda(), d_state))
    torch.cuda.synchronize()
    assert max_rel_err(d_state[0], ref_state) < STATE_TOL
    assert rel_err(torch.cat(outs).float(), ref_out) < OUT_TOL

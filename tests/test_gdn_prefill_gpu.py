"""GPU parity of the chunked prefill (zb_gdn_chunk_prefill) against the per-token recurrence of the oracle
(lm.py:576-582): fp32 final state within 1e-3 relative (max-abs), bf16 outputs within 2e-2 relative."""

from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

from conftest import max_rel_err, rel_err
from oracle import gdn as ogdn

pytestmark = pytest.mark.gpu

STATE_TOL = 1e-3
OUT_TOL = 2e-2


def packed_inputs(lengths, H, d, seed, state_scale=0.0):
    gen = torch.Generator().manual_seed(seed)
    N = sum(lengths)
    q = F.normalize(torch.randn(N, H, d, generator=gen), dim=-1).bfloat16()
    k = F.normalize(torch.randn(N, H, d, generator=gen), dim=-1).bfloat16()
    v = torch.randn(N, H, d, generator=gen).bfloat16()
    beta = torch.sigmoid(torch.randn(N, H, generator=gen))
    g = -F.softplus(torch.randn(N, H, generator=gen))
    cu = torch.tensor([0] + list(torch.tensor(lengths).cumsum(0)), dtype=torch.int32)
    init = torch.randn(len(lengths), H, d, d, generator=gen) * state_scale
    return q, k, v, g, beta, cu, init


def reference(q, k, v, g, beta, cu, init, device="cpu"):
    """Per-sequence per-token recurrence (the oracle), vectorised over heads."""
    d = q.shape[-1]
    outs, finals = [], []
    for i in range(len(cu) - 1):
        a, b = int(cu[i]), int(cu[i + 1])
        st, o = ogdn.recurrent_scan(init[i].to(device), q[a:b].to(device), k[a:b].to(device), v[a:b].to(device),
                                    g[a:b].to(device), beta[a:b].to(device), d ** -0.5)
        outs.append(o.cpu())
        finals.append(st.cpu())
    return torch.cat(outs), torch.stack(finals)


@pytest.mark.parametrize("lengths,H,d", [([64], 2, 128), ([1, 63, 65, 130], 3, 128), ([200, 7], 4, 64),
                                         ([129], 16, 128)])
def test_chunked_prefill_matches_recurrence(zb, lengths, H, d):
    q, k, v, g, beta, cu, init = packed_inputs(lengths, H, d, seed=sum(lengths) + H)
    ref_out, ref_state = reference(q, k, v, g, beta, cu, init)
    out, state = zb.ops.gdn_chunk_prefill(q.cuda(), k.cuda(), v.cuda(), g.cuda(), beta.cuda(), cu.cuda())
    torch.cuda.synchronize()
    assert max_rel_err(state, ref_state) < STATE_TOL
    assert rel_err(out.float(), ref_out) < OUT_TOL


@pytest.mark.parametrize("regime", ["strong_decay", "mixed_sign"])
def test_decay_regimes(zb, regime):
    """Chunks outside the factored-decay fast path of the d=128 kernel: more than 80 of log decay inside a 16-token
    block (g about -6.5 per token), and a log decay that is positive for some tokens (G not monotone)."""
    lengths, H, d = [130, 64], 2, 128
    q, k, v, g, beta, cu, init = packed_inputs(lengths, H, d, seed=5, state_scale=0.3)
    gen = torch.Generator().manual_seed(6)
    if regime == "strong_decay":
        g = -8.0 * F.softplus(torch.randn(g.shape, generator=gen))
    else:
        g = 0.05 * torch.randn(g.shape, generator=gen)
    ref_out, ref_state = reference(q, k, v, g, beta, cu, init)
    out, state = zb.ops.gdn_chunk_prefill(q.cuda(), k.cuda(), v.cuda(), g.cuda(), beta.cuda(), cu.cuda(),
                                          initial_state=init.cuda())
    torch.cuda.synchronize()
    assert torch.isfinite(out.float()).all() and torch.isfinite(state).all()
    assert max_rel_err(state, ref_state) < STATE_TOL
    assert rel_err(out.float(), ref_out) < OUT_TOL


def test_initial_state_and_slots(zb):
    """A continuation from given states (the prefill of a request with cached rows), states addressed by slot."""
    lengths, H, d = [70, 33], 2, 128
    q, k, v, g, beta, cu, init = packed_inputs(lengths, H, d, seed=9, state_scale=0.3)
    ref_out, ref_state = reference(q, k, v, g, beta, cu, init)
    pool = torch.zeros(5, H, d, d)
    slots = torch.tensor([3, 1])
    pool[slots] = init
    d_pool = pool.cuda()
    out, _ = zb.ops.gdn_chunk_prefill(q.cuda(), k.cuda(), v.cuda(), g.cuda(), beta.cuda(), cu.cuda(),
                                      initial_state=d_pool, final_state=d_pool, state_slots=slots.cuda())
    torch.cuda.synchronize()
    assert max_rel_err(d_pool[slots].cpu(), ref_state) < STATE_TOL
    assert rel_err(out.float(), ref_out) < OUT_TOL
    assert torch.equal(d_pool[0].cpu(), pool[0])  # untouched rows


def test_prefill_then_decode_equals_longer_prefill(zb):
    """The reference's own invariant (model/tests/test_reference_lm.py:126-136): prefill(n) == prefill(n-k) plus k
    recurrent decode steps, here across the two CUDA kernels."""
    H, d, n, kk = 4, 128, 100, 5
    q, k, v, g, beta, cu, init = packed_inputs([n], H, d, seed=21)
    dev = torch.device("cuda")
    full_out, full_state = zb.ops.gdn_chunk_prefill(q.to(dev), k.to(dev), v.to(dev), g.to(dev), beta.to(dev),
                                                    cu.to(dev))
    part_cu = torch.tensor([0, n - kk], dtype=torch.int32, device=dev)
    m = n - kk
    part_out, state = zb.ops.gdn_chunk_prefill(q[:m].to(dev), k[:m].to(dev), v[:m].to(dev), g[:m].to(dev),
                                               beta[:m].to(dev), part_cu)
    outs = [part_out]
    for t in range(m, n):
        outs.append(zb.ops.gdn_decode_step(q[t:t + 1].to(dev), k[t:t + 1].to(dev), v[t:t + 1].to(dev),
                                           g[t:t + 1].to(dev), beta[t:t + 1].to(dev), state))
    torch.cuda.synchronize()
    assert max_rel_err(state, full_state) < STATE_TOL
    assert rel_err(torch.cat(outs).float(), full_out.float()) < OUT_TOL


def test_cfg3_full_size(zb):
    """cfg3: B=8 sequences of T=2048, 16 heads, dk=dv=128, zero initial state. The reference recurrence runs as a
    plain fp32 PyTorch computation on the device (the CPU would take minutes)."""
    B, T, H, d = 8, 2048, 16, 128
    q, k, v, g, beta, cu, init = packed_inputs([T] * B, H, d, seed=33)
    dev = torch.device("cuda")
    out, state = zb.ops.gdn_chunk_prefill(q.to(dev), k.to(dev), v.to(dev), g.to(dev), beta.to(dev), cu.to(dev))
    torch.cuda.synchronize()
    # the recurrence for all 8 sequences at once: [T, B, H, ...]
    qq, kk_, vv = (x.view(B, T, H, d).transpose(0, 1).to(dev) for x in (q, k, v))
    gg, bb = (x.view(B, T, H).transpose(0, 1).to(dev) for x in (g, beta))
    ref_state, ref_out = ogdn.recurrent_scan(torch.zeros(B, H, d, d, device=dev), qq, kk_, vv, gg, bb, d ** -0.5)
    assert max_rel_err(state, ref_state) < STATE_TOL
    assert rel_err(out.view(B, T, H, d).transpose(0, 1).float(), ref_out) < OUT_TOL

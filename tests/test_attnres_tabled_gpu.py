"""GPU parity of the Full AttnRes route over a logit table (zb_attnres_route_tabled) against the CPU oracle
(full_attnres_route, lm.py:384-389, with the reference Triton kernel's rounding points).

A forward's routes run in order; route r mixes bank rows [0, r) (logits read from the table, written by route r-1)
and its current source, and while it mixes writes route r+1's logits of rows [0, r] to the table. Every
output is compared with the oracle route over the same sources (2e-2 relative), and the recorded table entries with
the oracle's logits. Bit identity is required of >= 99 % of the elements of a whole schedule and >= 95 % of every
route: a logit summed in another fp32 order than the oracle's can put one softmax weight on the other side of a bf16
rounding boundary, which changes a good part of that token's row (the staged kernel's order does the same on the
same data)."""

from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

from conftest import rel_err
from oracle import attnres as oattn

pytestmark = pytest.mark.gpu

TOL = 2e-2
EPS = 1e-5


def make_schedule(R, T, D, seed):
    gen = torch.Generator().manual_seed(seed)
    bank = torch.stack([torch.randn(T, D, generator=gen) * (0.5 + s % 3) for s in range(R)]).bfloat16()
    queries = (0.2 * torch.randn(R, D, generator=gen)).bfloat16()
    norm_w = (1 + 0.1 * torch.randn(D, generator=gen)).bfloat16()
    return bank, queries, norm_w


def identical_fraction(a, b):
    return (a.cpu().view(torch.int16) == b.cpu().view(torch.int16)).float().mean().item()


def oracle_logits(rows, query):
    """[S, T] fp32 logits of bank rows for one query (the oracle's key * query sum)."""
    keys = F.rms_norm(rows, (rows.shape[-1],), eps=EPS)
    return (keys * query).sum(-1, dtype=torch.float32)


@pytest.mark.parametrize("R,T,D", [(1, 3, 256), (9, 33, 1024), (20, 17, 2048), (49, 64, 2048), (4, 4, 1536),
                                   (40, 6, 4096), (3, 2, 3072)])
def test_tabled_schedule_matches_oracle(zb, R, T, D):
    """Routes 0 .. R-1 in place over a growing bank (the current source is bank row r; the last route's is not
    kept), RMSNorm fused; the table fills as the routes run."""
    bank, queries, norm_w = make_schedule(R, T, D, seed=R * 7 + T + D)
    d_bank, d_q, d_w = bank.cuda(), queries.cuda(), norm_w.cuda()
    rows = (R + 3) // 4 * 4
    table = torch.full((R, T, rows), float("nan"), device="cuda")
    inv = torch.full((T, rows), float("nan"), device="cuda")
    same = []
    for r in range(R):
        out = zb.ops.attnres_route_tabled(d_bank, r, d_bank[r], d_q, r, table, inv, EPS, source_in_bank=r < R - 1,
                                          norm_weight=d_w, norm_eps=EPS)
        ref = oattn.weighted_rms_norm(oattn.full_attnres_route(bank[: r + 1], queries[r], EPS), norm_w, EPS)
        torch.cuda.synchronize()
        assert rel_err(out.float().cpu(), ref.float()) < TOL, r
        same.append(identical_fraction(out, ref))
        assert same[-1] > 0.95, r
    assert sum(same) / R > 0.99
    assert zb.ops.device_status() == 0
    # every recorded entry is the oracle's logit (up to a few keys that the kernel's inverse RMS rounds to the
    # neighbouring bf16 value, each moving the logit by about 2^-8 of one product: 1e-3 of the sum of |products|
    # still tells any other route's or source's logit apart); the entries no route records stay untouched
    tab = table.cpu()
    for r in range(1, R):
        ref = oracle_logits(bank[:r], queries[r]).T  # [T, r]
        scale = (F.rms_norm(bank[:r].float(), (D,), eps=EPS).abs() * queries[r].float().abs()).sum(-1).T
        assert ((tab[r, :, :r] - ref).abs() <= 1e-3 * scale).all(), r
        assert torch.isnan(tab[r, :, r:]).all(), r
    assert torch.isnan(tab[0]).all()
    rms = torch.rsqrt(bank[: R - 1].float().pow(2).mean(-1) + EPS).T  # [T, R-1]
    assert torch.allclose(inv[:, : R - 1].cpu(), rms, rtol=1e-5) and torch.isnan(inv[:, R - 1:].cpu()).all()


def test_tabled_rejects_wide_rows(zb):
    """Hidden sizes above 4096 are refused (the staged route serves them)."""
    d_q = torch.zeros(2, 8192, device="cuda", dtype=torch.bfloat16)
    src = torch.zeros(2, 8192, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(Exception, match="at most 4096"):
        zb.ops.attnres_route_tabled(None, 0, src, d_q, 0, torch.zeros(2, 2, 4, device="cuda"),
                                    torch.zeros(2, 4, device="cuda"), EPS)


def test_tabled_separate_source_append_and_mix(zb):
    """A current source outside the bank, appended to the next bank row by the route; un-normalised output, and
    mix_out beside a fused norm."""
    R, T, D = 7, 24, 2048
    bank, queries, norm_w = make_schedule(R, T, D, seed=3)
    d_q = queries.cuda()
    d_bank = torch.zeros_like(bank, device="cuda")
    table = torch.zeros((R, T, 8), device="cuda")
    inv = torch.zeros((T, 8), device="cuda")
    for r in range(R):
        src = bank[r].cuda()
        if r % 2:
            mix_out = torch.empty(T, D, device="cuda", dtype=torch.bfloat16)
            out = zb.ops.attnres_route_tabled(d_bank, r, src, d_q, r, table, inv, EPS, append_to=d_bank[r],
                                              norm_weight=norm_w.cuda(), norm_eps=EPS, mix_out=mix_out)
        else:
            mix_out = out = zb.ops.attnres_route_tabled(d_bank, r, src, d_q, r, table, inv, EPS,
                                                        append_to=d_bank[r])
        mix = oattn.full_attnres_route(bank[: r + 1], queries[r], EPS)
        torch.cuda.synchronize()
        assert torch.equal(d_bank[r].cpu(), bank[r]), r
        assert rel_err(mix_out.float().cpu(), mix.float()) < TOL and identical_fraction(mix_out, mix) > 0.95, r
        if r % 2:
            ref = oattn.weighted_rms_norm(mix, norm_w, EPS)
            assert rel_err(out.float().cpu(), ref.float()) < TOL and identical_fraction(out, ref) > 0.95, r
    assert zb.ops.device_status() == 0


def test_context_with_registered_queries(zb):
    """FusedBlockAttnResContext with the forward's queries registered: routes with appends (in place and from a
    separate source), a final route without append, two forwards; a query other than the registered one raises."""
    T, D, routes = 16, 1024, 9
    gen = torch.Generator().manual_seed(5)
    sources = [(torch.randn(T, D, generator=gen) * (0.5 + i % 3)).bfloat16() for i in range(routes)]
    queries = (0.2 * torch.randn(routes, D, generator=gen)).bfloat16()
    norm_w = (1 + 0.1 * torch.randn(D, generator=gen)).bfloat16()
    d_q = queries.cuda()
    ctx = zb.attnres.FusedBlockAttnResContext(routes - 1, sources[0].cuda())
    for trial in range(2):
        ctx.reset()
        ctx.register_queries(d_q, EPS)
        for i in range(routes):
            last = i == routes - 1
            src = sources[i].cuda()
            if i % 2 and not last:  # the producer writes straight into the next bank row
                ctx.next_row().copy_(src)
                src = ctx.next_row()
            out = ctx.route(src, d_q[i], EPS, not last, norm_weight=norm_w.cuda())
            ref = oattn.weighted_rms_norm(oattn.full_attnres_route(torch.stack(sources[: i + 1]), queries[i], EPS),
                                          norm_w, EPS)
            torch.cuda.synchronize()
            assert rel_err(out.float().cpu(), ref.float()) < TOL, (trial, i)
            assert identical_fraction(out, ref) > 0.99, (trial, i)
    assert ctx.completed_count == routes - 1
    ctx.reset()
    with pytest.raises(RuntimeError, match="registered"):
        ctx.route(sources[0].cuda(), d_q[1], EPS, True)
    with pytest.raises(RuntimeError, match="registered"):
        ctx.route(sources[0].cuda(), d_q[0].clone(), EPS, True)
    ctx.register_queries(None)
    out = ctx.route(sources[0].cuda(), d_q[0].clone(), EPS, True)  # unregistered: the staged route
    torch.cuda.synchronize()
    assert identical_fraction(out, sources[0]) == 1.0
    assert zb.ops.device_status() == 0

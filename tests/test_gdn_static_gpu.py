"""OriginalGDN's graph decode path (static mode: the engine's padded slot buffer, -1 padding rows, one CUDA graph
replayed per step; servers/sgl/src/zonos3_sgl/models/gdn.py:329-355 is the path it replaces) against the oracle layer
(oracle/gdn.gdn_layer restating lm.py:556-602) run per request in fp32 on the same bf16 weights.

The graph is captured before any request is loaded (as the engine captures at start-up); two requests are then
prefilled eagerly (ragged path) into slots 5 and 2 and decoded for 8 replays of a 4-row padded batch
[5, -1, 2, -1]. Bars: outputs within 2e-2 relative (bf16), fp32 states within 2e-2 of their max (bf16 inputs),
conv histories within 2e-2; the slots no request owns stay zero (padding rows touch no state)."""

from __future__ import annotations

import pytest
import torch

from conftest import max_rel_err, rel_err
from oracle import gdn as ogdn
from test_modules import fill_gdn, gdn_config

pytestmark = pytest.mark.gpu

TOL = 2e-2


@pytest.mark.parametrize("heads,head_dim,fused", [(4, 128, False), (16, 128, False), (4, 128, True),
                                                 (16, 128, True)])
def test_static_graph_decode_matches_oracle(zb, heads, head_dim, fused):
    """fused: the decode rows run the fused in_proj + prologue kernel (OriginalGDN.fused_in_proj)."""
    hidden, capacity, bs, steps = 256, 8, 4, 8
    dev = torch.device("cuda")
    layer = fill_gdn(zb.gdn.OriginalGDN(gdn_config(zb, hidden, heads, head_dim), 0), seed=7 + heads)
    layer.fused_in_proj = fused
    layer.to(dev, torch.bfloat16)
    layer.allocate_cache(capacity, dev, torch.bfloat16)
    w32 = {k: v.float().cpu() for k, v in layer.state_dict().items()}
    slots = torch.tensor([5, -1, 2, -1], dtype=torch.int64, device=dev)
    layer.enable_graph_decode(slots, zb.gdn.OriginalGDN.static_tables(dev, [bs]))
    layer.set_static_mode(True)
    Req = zb.core.Req
    decode_batch = zb.core.Batch(reqs=[Req(5, 1, 1, uid=0), Req(2, 1, 1, uid=1)], is_decode=True, padded_size=bs)
    x_buf = torch.zeros(bs, hidden, device=dev, dtype=torch.bfloat16)
    stream = torch.cuda.Stream(dev)
    stream.wait_stream(torch.cuda.current_stream())
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream), zb.core.forward_batch(decode_batch):
        layer.forward(x_buf)  # warm-up (touches slots 5 and 2, which the prefill below starts afresh)
        torch.cuda.synchronize()
        with torch.cuda.graph(graph, stream=stream):
            y_buf = layer.forward(x_buf)
    torch.cuda.current_stream().wait_stream(stream)

    lengths, owners = [10, 70], [5, 2]
    gen = torch.Generator().manual_seed(11)
    xs = [torch.randn(n + steps, hidden, generator=gen).bfloat16() for n in lengths]
    outs = [[], []]
    prefill = zb.core.Batch(reqs=[Req(s, n, 0, uid=i) for i, (s, n) in enumerate(zip(owners, lengths))],
                            is_decode=False)
    with zb.core.forward_batch(prefill):
        y = layer.forward(torch.cat([x[:n] for x, n in zip(xs, lengths)]).to(dev))
    for i, part in enumerate(y.split(lengths)):
        outs[i].append(part.float().cpu())
    for t in range(steps):
        rows = torch.randn(bs, hidden, generator=gen).bfloat16()  # padding rows carry noise
        rows[0], rows[2] = xs[0][lengths[0] + t], xs[1][lengths[1] + t]
        x_buf.copy_(rows)
        graph.replay()
        torch.cuda.synchronize()
        outs[0].append(y_buf[0:1].float().cpu())
        outs[1].append(y_buf[2:3].float().cpu())
    for i, (x, s) in enumerate(zip(xs, owners)):
        ref_y, conv, state = ogdn.gdn_layer(x.float(), w32, heads=heads, head_dim=head_dim)
        got = torch.cat(outs[i])
        assert rel_err(got, ref_y) < TOL, i
        assert rel_err(got[lengths[i]:], ref_y[lengths[i]:]) < TOL, f"decode rows of request {i}"
        assert max_rel_err(layer._recurrent_state[s].cpu(), state) < TOL, i
        assert rel_err(layer._conv_state[s].float().cpu(), conv) < TOL, i
    untouched = [s for s in range(capacity) if s not in owners]
    assert layer._recurrent_state[untouched].abs().max().item() == 0.0
    assert layer._conv_state[untouched].abs().max().item() == 0.0
    del graph


def test_static_padded_prefill_captured_and_replayed(zb):
    """The padded prefill of fresh requests (PrefillLayout whole = [1, 0, 2]: 128 + 64 + 192 rows, the reference's
    _forward_prefill_static layout, gdn.py:62-104, :357-393) captured once in a CUDA graph and replayed twice with
    other real lengths and other data, padding rows holding noise; every real output row, final state and conv
    history against the oracle run per request (oracle/gdn.gdn_layer), then one decode step per request continuing
    from the committed state."""
    hidden, heads, head_dim = 256, 4, 128
    dev = torch.device("cuda")
    layer = fill_gdn(zb.gdn.OriginalGDN(gdn_config(zb, hidden, heads, head_dim), 0), seed=21)
    layer.to(dev, torch.bfloat16)
    layer.allocate_cache(8, dev, torch.bfloat16)
    w32 = {k: v.float().cpu() for k, v in layer.state_dict().items()}
    whole = [1, 0, 2]
    layout = zb.gdn.PrefillLayout.build(whole, dev)
    starts = layout.starts.tolist()
    x_buf = torch.zeros(layout.rows, hidden, device=dev, dtype=torch.bfloat16)
    slots_buf = torch.tensor([5, 0, 3], dtype=torch.int64, device=dev)
    len_buf = torch.tensor([65, 1, 129], dtype=torch.int64, device=dev)
    Req = zb.core.Req
    inputs = zb.gdn.PrefillInputs(layout, slots_buf, len_buf)
    batch = zb.core.Batch(reqs=[Req(5, 128, 0, uid=0), Req(0, 64, 0, uid=1), Req(3, 192, 0, uid=2)], is_decode=False,
                          gdn_prefill=inputs)
    stream = torch.cuda.Stream(dev)
    stream.wait_stream(torch.cuda.current_stream())
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream), zb.core.forward_batch(batch):
        layer.forward(x_buf)
        torch.cuda.synchronize()
        with torch.cuda.graph(graph, stream=stream):
            y_buf = layer.forward(x_buf)
    torch.cuda.current_stream().wait_stream(stream)
    gen = torch.Generator().manual_seed(4)
    for lengths in ([70, 2, 150], [128, 64, 129]):
        xs = [torch.randn(n + 1, hidden, generator=gen).bfloat16() for n in lengths]  # the last row: a decode step
        rows = torch.randn(layout.rows, hidden, generator=gen).bfloat16()  # padding rows hold noise
        for s0, x, n in zip(starts, xs, lengths):
            rows[s0:s0 + n] = x[:n]
        x_buf.copy_(rows)
        len_buf.copy_(torch.tensor(lengths))
        graph.replay()
        torch.cuda.synchronize()
        layer.note_graph_forward([Req(s, n, 0, uid=i) for i, (s, n) in enumerate(zip([5, 0, 3], lengths))])
        reqs = [Req(s, 1, n, uid=i) for i, (s, n) in enumerate(zip([5, 0, 3], lengths))]
        with zb.core.forward_batch(zb.core.Batch(reqs=reqs, is_decode=True)):
            step = layer.forward(torch.stack([x[n] for x, n in zip(xs, lengths)]).to(dev))
        torch.cuda.synchronize()
        for i, (x, n, s0, slot) in enumerate(zip(xs, lengths, starts, [5, 0, 3])):
            ref_pre, conv, state = ogdn.gdn_layer(x[:n].float(), w32, heads=heads, head_dim=head_dim)
            assert rel_err(y_buf[s0:s0 + n].float().cpu(), ref_pre) < TOL, (lengths, i)
            ref_all, conv2, state2 = ogdn.gdn_layer(x.float(), w32, heads=heads, head_dim=head_dim)
            assert rel_err(step[i].float().cpu(), ref_all[n]) < TOL, (lengths, i)
            assert max_rel_err(layer._recurrent_state[slot].cpu(), state2) < TOL, (lengths, i)
            assert rel_err(layer._conv_state[slot].float().cpu(), conv2) < TOL, (lengths, i)
    del graph

"""Drop-in modules: checkpoint names, strict loading and weight-format conversion (CPU), and forward parity of
OriginalGDN / MoEFeedForward against the oracle's restatement of the reference layers (GPU)."""

from __future__ import annotations

import pytest
import torch

from conftest import max_rel_err, rel_err
from oracle import gdn as ogdn
from oracle import moe as omoe

TOL = 2e-2


def gdn_config(zb, hidden=256, heads=4, head_dim=128):
    return zb.config.ModelConfig(hidden_size=hidden, gdn_num_heads=heads, gdn_head_dim=head_dim)


def fill_gdn(layer, seed):
    gen = torch.Generator().manual_seed(seed)
    for name, t in layer.state_dict().items():
        noise = torch.randn(t.shape, generator=gen)
        if name == "out_weight":
            val = 1 + 0.1 * noise
        elif name in ("A_log", "dt_bias"):
            val = 0.5 * noise
        elif name == "conv.weight":
            val = 0.3 * noise
        else:
            val = 0.1 * noise
        obj, attr = layer, name.split(".")
        for a in attr[:-1]:
            obj = getattr(obj, a)
        setattr(obj, attr[-1], val.to(t.dtype))
    return layer


def test_gdn_checkpoint_names_and_strict_load(zb):
    layer = zb.gdn.OriginalGDN(gdn_config(zb), 0)
    assert sorted(layer.state_dict()) == sorted(
        ["in_proj.weight", "conv.weight", "out_weight", "A_log", "dt_bias", "wo.weight"])
    state = {k: torch.zeros_like(v) for k, v in layer.state_dict().items()}
    layer.load_state_dict(dict(state))
    with pytest.raises(RuntimeError):
        layer.load_state_dict({**state, "extra": torch.zeros(1)})
    with pytest.raises(ValueError):
        layer.load_state_dict({**state, "wo.weight": torch.zeros(3, 3)})


def test_moe_checkpoint_formats(zb):
    cfg = zb.config.ModelConfig(hidden_size=64, moe_n_experts=4, moe_topk=2, moe_intermediate_size=32, moe_alpha=0.5)
    ff = zb.moe.MoEFeedForward(cfg, 1)
    names = sorted(ff.state_dict())
    assert names == sorted(["router.router_linear.weight", "router.rmsnorm_eda.weight", "router.balancing_biases",
                            "experts.gate_up_proj", "experts.down_proj", "latent_down.weight", "latent_up.weight"])
    E, I, D = 4, 32, 32
    w1, w3, w2 = torch.randn(E, I, D), torch.randn(E, I, D), torch.randn(E, D, I)
    base = {k: torch.zeros_like(v) for k, v in ff.state_dict().items() if not k.startswith("experts.")}
    ff.load_state_dict({**base, "experts.w1.weight": w1, "experts.w3.weight": w3, "experts.w2.weight": w2})
    assert torch.equal(ff.experts.gate_up_proj, torch.cat([w1, w3], 1)) and torch.equal(ff.experts.down_proj, w2)
    inter = torch.stack([w1, w3], 2).flatten(1, 2)  # SonicMoE layout: gate / up rows interleaved
    ff.load_state_dict({**base, "experts.w13": inter, "experts.w2": w2})
    assert torch.equal(ff.experts.gate_up_proj, torch.cat([w1, w3], 1))


def make_batch(zb, reqs, decode):
    return zb.core.Batch(reqs=reqs, is_decode=decode)


@pytest.mark.gpu
@pytest.mark.parametrize("heads,head_dim", [(4, 128), (4, 64), (16, 128)])
def test_original_gdn_prefill_then_decode(zb, heads, head_dim):
    """Three requests prefilled together (ragged, one shorter than the conv window), then four decode steps; every
    output row and the final states against the oracle run per request in fp32 on the same bf16 weights."""
    hidden = 256
    cfg = gdn_config(zb, hidden, heads, head_dim)
    layer = fill_gdn(zb.gdn.OriginalGDN(cfg, 0), seed=heads + head_dim)
    layer.to("cuda", torch.bfloat16)
    layer.allocate_cache(8, "cuda", torch.bfloat16)
    w32 = {k: v.float().cpu() for k, v in layer.state_dict().items()}
    lengths, slots, steps = [70, 2, 130], [5, 0, 3], 4
    gen = torch.Generator().manual_seed(1)
    xs = [torch.randn(n + steps, hidden, generator=gen).bfloat16() for n in lengths]
    Req = zb.core.Req
    outs = [[] for _ in lengths]
    with zb.core.forward_batch(make_batch(zb, [Req(s, n, 0, uid=i) for i, (s, n) in enumerate(zip(slots, lengths))],
                                          False)):
        y = layer.forward(torch.cat([x[:n] for x, n in zip(xs, lengths)]).cuda())
    for i, part in enumerate(y.split(lengths)):
        outs[i].append(part)
    for t in range(steps):
        reqs = [Req(s, 1, n + t, uid=i) for i, (s, n) in enumerate(zip(slots, lengths))]
        with zb.core.forward_batch(make_batch(zb, reqs, True)):
            y = layer.forward(torch.stack([x[n + t] for x, n in zip(xs, lengths)]).cuda())
        for i in range(len(lengths)):
            outs[i].append(y[i:i + 1])
    torch.cuda.synchronize()
    for i, (x, s) in enumerate(zip(xs, slots)):
        ref_y, conv, state = ogdn.gdn_layer(x.float(), w32, heads=heads, head_dim=head_dim)
        got = torch.cat(outs[i]).float().cpu()
        assert rel_err(got, ref_y) < TOL, i
        assert max_rel_err(layer._recurrent_state[s].cpu(), state) < TOL, i
        assert rel_err(layer._conv_state[s].float().cpu(), conv) < TOL, i


@pytest.mark.gpu
def test_original_gdn_rejects_stale_state(zb):
    cfg = gdn_config(zb)
    layer = fill_gdn(zb.gdn.OriginalGDN(cfg, 0), seed=3).to("cuda", torch.bfloat16)
    layer.allocate_cache(2, "cuda", torch.bfloat16)
    Req = zb.core.Req
    with zb.core.forward_batch(make_batch(zb, [Req(0, 1, 5)], True)):
        with pytest.raises(RuntimeError, match="stale"):
            layer.forward(torch.zeros(1, 256, dtype=torch.bfloat16, device="cuda"))


@pytest.mark.gpu
@pytest.mark.parametrize("E,k,I,alpha", [(8, 2, 512, 1.0), (16, 2, 256, 0.5), (64, 8, 768, 1.0)])
def test_moe_feed_forward_matches_oracle(zb, E, k, I, alpha):
    hidden, T = 256 if E < 64 else 2048, 77
    cfg = zb.config.ModelConfig(hidden_size=hidden, moe_n_experts=E, moe_topk=k, moe_intermediate_size=I,
                                moe_alpha=alpha, norm_topk_prob=True)
    ff = zb.moe.MoEFeedForward(cfg, 1)
    gen = torch.Generator().manual_seed(E + k)
    for name, t in ff.state_dict().items():
        noise = torch.randn(t.shape, generator=gen)
        val = 1 + 0.1 * noise if "rmsnorm" in name else 0.05 * noise
        obj, attr = ff, name.split(".")
        for a in attr[:-1]:
            obj = getattr(obj, a)
        setattr(obj, attr[-1], val)
    ff.to("cuda", torch.bfloat16)
    x = torch.randn(T, hidden, generator=gen).bfloat16()
    logits_dev = torch.empty(T, E, device="cuda", dtype=torch.bfloat16)
    w, ids, _ = ff.router.forward(x.cuda(), logits=logits_dev)
    out, _ = ff.forward(x.cuda())
    torch.cuda.synchronize()
    f32 = {n: t.float().cpu() for n, t in ff.state_dict().items()}
    # selection on the kernel's own logits is bit-exact; weights as the training router computes them
    ref_ids, ref_w = omoe.route(logits_dev.cpu(), f32["router.balancing_biases"], k)
    assert torch.equal(ids.cpu(), ref_ids)
    torch.testing.assert_close(w.cpu(), ref_w, rtol=1e-5, atol=1e-6)
    # layer output: the oracle's expert loop (lm.py:618-639) on the same routing, renormalised like FusedMoE
    ref_w = ref_w / (ref_w.sum(-1, keepdim=True) + 1e-8)
    routed = torch.nn.functional.linear(x.float(), f32["latent_down.weight"]) if alpha < 1 else x.float()
    y = omoe.experts_fp32(routed, f32["experts.gate_up_proj"], f32["experts.down_proj"], ref_ids, ref_w)
    if alpha < 1:
        y = torch.nn.functional.linear(y, f32["latent_up.weight"])
    assert rel_err(out.float().cpu(), y) < TOL

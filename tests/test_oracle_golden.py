"""Pin the CPU oracle to the reference: the restatement must reproduce the golden vectors that the unmodified
reference (model/src/zonos3/reference/lm.py) produced in tests/golden/make_golden.py."""

from __future__ import annotations

import numpy as np
import torch

from oracle import attnres as oattn
from oracle import gdn as ogdn
from oracle import moe as omoe


def _gdn_weights(g):
    return {k[2:]: v for k, v in g.items() if k.startswith("w.")}


def test_gdn_layer_matches_reference_prefill_then_decode(golden):
    g = golden("gdn_tiny.npz")
    w = _gdn_weights(g)
    x = g["x"]
    cap: dict = {}
    y0, conv, state = ogdn.gdn_layer(x[:12], w, heads=4, head_dim=128, capture=cap)
    torch.testing.assert_close(state, g["state_prefill"], rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(conv, g["conv_state_prefill"], rtol=0, atol=0)
    for name in ("gdn_q", "gdn_k", "gdn_v", "gdn_decay", "gdn_beta", "gdn_recurrent", "gdn_gated"):
        torch.testing.assert_close(cap[name].float(), g[name][:12], rtol=1e-5, atol=1e-6, msg=name)
    ys = [y0]
    for row in range(12, 15):
        y, conv, state = ogdn.gdn_layer(x[row:row + 1], w, conv, state, heads=4, head_dim=128)
        ys.append(y)
    torch.testing.assert_close(torch.cat(ys), g["y"], rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(state, g["state_final"], rtol=1e-5, atol=1e-6)
    # single-row projections may take a different BLAS path than the generator run: allow 1 ulp
    torch.testing.assert_close(conv, g["conv_state_final"], rtol=1e-6, atol=1e-6)


def test_gdn_prefill_equals_prefill_plus_decode():
    """The reference's own invariant (model/tests/test_reference_lm.py:126-136) holds for the restated layer at a
    head width the reference does not express (dk = dv = 64)."""
    gen = torch.Generator().manual_seed(5)
    heads, hd, dim = 4, 64, 96
    inner = heads * hd
    w = {
        "in_proj.weight": 0.1 * torch.randn(4 * inner + 2 * heads, dim, generator=gen),
        "conv.weight": 0.3 * torch.randn(3 * inner, 1, 4, generator=gen),
        "out_weight": 1 + 0.1 * torch.randn(hd, generator=gen),
        "A_log": 0.5 * torch.randn(heads, generator=gen),
        "dt_bias": 0.5 * torch.randn(heads, generator=gen),
        "wo.weight": 0.1 * torch.randn(dim, inner, generator=gen),
    }
    x = torch.randn(20, dim, generator=gen)
    full, conv_f, state_f = ogdn.gdn_layer(x, w, heads=heads, head_dim=hd)
    part, conv, state = ogdn.gdn_layer(x[:13], w, heads=heads, head_dim=hd)
    outs = [part]
    for r in range(13, 20):
        y, conv, state = ogdn.gdn_layer(x[r:r + 1], w, conv, state, heads=heads, head_dim=hd)
        outs.append(y)
    torch.testing.assert_close(torch.cat(outs), full, rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(state, state_f, rtol=1e-5, atol=1e-6)


def test_attnres_route_matches_reference(golden):
    g = golden("attnres.npz")
    for tag, dtype in (("f32", torch.float32), ("bf16", torch.bfloat16), ("one", torch.bfloat16)):
        sources = g[f"{tag}_sources"].to(dtype)
        query = g[f"{tag}_query"].to(dtype)
        mixed = oattn.full_attnres_route(list(sources), query, 1e-5)
        torch.testing.assert_close(mixed.float(), g[f"{tag}_out"], rtol=0, atol=0, msg=tag)


def test_moe_layer_matches_reference(golden):
    g = golden("moe_tiny.npz")
    w = {k[2:]: v for k, v in g.items() if k.startswith("w.")}
    x = g["x"]
    latent_x = torch.nn.functional.linear(x, w["latent_down.weight"])
    logits = omoe.router_logits(x, w["router.rmsnorm_eda.weight"], w["router.router_linear.weight"], 1e-5)
    torch.testing.assert_close(logits, g["logits"], rtol=0, atol=0)
    ids, weights = omoe.route(logits, w["router.balancing_biases"], 2)
    assert torch.equal(ids.long(), g["topk"])
    out = omoe.experts_fp32(latent_x, w["experts.gate_up_proj"], w["experts.down_proj"], ids, weights)
    y = torch.nn.functional.linear(out, w["latent_up.weight"])
    torch.testing.assert_close(y, g["y"], rtol=1e-5, atol=1e-6)
    # the per-(token, rank) loop the reference runs, which the cfg4 CPU baseline times
    loop = omoe.experts_loop_fp32(latent_x, w["experts.gate_up_proj"], w["experts.down_proj"], ids, weights)
    torch.testing.assert_close(torch.nn.functional.linear(loop, w["latent_up.weight"]), g["y"], rtol=1e-5, atol=1e-6)


def test_topk_tie_rule_agrees_wherever_the_reference_is_deterministic(golden):
    """bf16 logits with zero biases tie often. Where the reference's top-k does not depend on a tie (the k+1 best
    scores of a row are distinct) the oracle's ids equal the reference's; elsewhere the sets agree whenever the
    boundary (k-th vs (k+1)-th score) is not tied."""
    g = golden("moe_ties.npz")
    scores, ref = g["scores"], g["topk"]
    k = ref.shape[1]
    ours = omoe.select_topk(scores, k).long()
    top = torch.sort(scores, dim=-1, descending=True).values[:, : k + 1]
    distinct = (top[:, 1:] < top[:, :-1]).all(-1)
    boundary_free = top[:, k - 1] > top[:, k]
    assert distinct.sum() > 0 and (~distinct).sum() > 0, "fixture should contain both kinds of rows"
    assert torch.equal(ours[distinct], ref[distinct])
    assert torch.equal(ours[boundary_free].sort(-1).values, ref[boundary_free].sort(-1).values)


def test_permutation_contract():
    ids = torch.tensor([[2, 3], [1, 2], [1, 3], [1, 2]])
    p = omoe.permutation(ids, 4, block=4)
    assert p["counts"].tolist() == [0, 3, 3, 2]
    assert p["offsets"].tolist() == [0, 0, 4, 8, 12]
    assert p["sorted_pairs"].tolist() == [2, 4, 6, -1, 0, 3, 7, -1, 1, 5, -1, -1]
    assert np.array_equal(p["sorted_pairs"][p["position"]], np.arange(8))


def test_whole_lm_matches_reference(golden):
    """The restated LM (oracle/lm.py) reproduces the reference Zonos3LM's logits for a prompt and two decode calls
    (a GDN layer, a global attention layer, dense FFN then MoE, Full AttnRes)."""
    from oracle import lm as olm

    g = golden("lm_tiny.npz")
    w = {k[2:]: v for k, v in g.items() if k.startswith("w.")}
    c = olm.LMConfig(dim=32, n_layers=2, gdn_period=2, gdn_heads=4, gdn_head_dim=128, n_heads=4, n_kv_heads=2,
                     head_dim=16, n_experts=4, topk=2, moe_hidden=32, moe_routed_dim=16, latent=True,
                     dense_first_layer=True, ffn_hidden=64, n_codebooks=10, codebook_size=16, text_rows=21)
    assert set(olm.weight_shapes(c)) <= set(w)
    for name, shape in olm.weight_shapes(c).items():
        assert tuple(w[name].shape) == shape, name
    ids = g["ids"].long()
    cache = olm.Cache()
    logits = torch.cat([olm.forward(c, w, ids[:12], cache), olm.forward(c, w, ids[12:13], cache),
                        olm.forward(c, w, ids[13:14], cache)])
    torch.testing.assert_close(logits, g["logits"], rtol=1e-4, atol=1e-5)

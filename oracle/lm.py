"""Whole-LM oracle (CPU, float32): a restatement of ``Zonos3LM.forward`` (model/src/zonos3/reference/lm.py:660-735)
with the architecture sizes as parameters, so it expresses both the reference's own model (layer 0 dense, GDN fixed
at 4 heads of 128, lm.py:28, :332) and the benchmark's config 1 (MoE in every layer, GDN 4 heads of 64).

Covered: summed multi-codebook + text embeddings, weightless embedding RMSNorm, the Full AttnRes schedule (a route
before every sublayer and a final one, lm.py:699-721), GDN layers (oracle.gdn.gdn_layer), global GQA attention
(lm.py:511-537, restated), dense FFN (lm.py:606-609), MoE (oracle.moe), output norm, multi-codebook head and
softcap. Left out (not on the hot path): speaker / condition rows, hidden steering, accents, alignment probes.

Weights use the checkpoint names of lm.py's module tree (``layers.{i}.attention.in_proj.weight`` ...).
Test infrastructure only (see ``oracle/__init__.py``).
"""

from __future__ import annotations

from dataclasses import dataclass, field

import torch
import torch.nn.functional as F

from . import attnres as oattn
from . import gdn as ogdn
from . import moe as omoe


@dataclass(frozen=True)
class LMConfig:
    dim: int = 256
    n_layers: int = 4
    gdn_period: int = 3  # layer uses GDN when (layer + 1) % gdn_period != 0, else global attention
    gdn_heads: int = 4
    gdn_head_dim: int = 64
    n_heads: int = 8
    n_kv_heads: int = 2
    head_dim: int = 32
    rope_theta: float = 10000.0
    norm_eps: float = 1e-5
    n_experts: int = 8
    topk: int = 2
    moe_hidden: int = 512
    moe_routed_dim: int = 256
    latent: bool = False  # latent_down / latent_up around the experts
    dense_first_layer: bool = False  # the reference makes layer 0 a dense FFN
    ffn_hidden: int = 512
    n_codebooks: int = 10
    codebook_size: int = 1024
    text_rows: int = 1025
    loss_softcap: float = 15.0

    @property
    def audio_vocab(self) -> int:
        return self.codebook_size + 2

    def uses_gdn(self, layer: int) -> bool:
        return (layer + 1) % self.gdn_period != 0

    def is_moe(self, layer: int) -> bool:
        return not (self.dense_first_layer and layer == 0)


@dataclass
class Cache:
    position: int = 0
    kv: dict = field(default_factory=dict)
    gdn_state: dict = field(default_factory=dict)
    conv_state: dict = field(default_factory=dict)


def rope_interleaved(x, positions, theta):
    """Interleaved-pair rotary embedding (lm.py:392-400)."""
    hd = x.shape[-1]
    freqs = theta ** (-torch.arange(0, hd, 2, dtype=torch.float32) / hd)
    ang = positions.float()[:, None] * freqs[None, :]
    cos, sin = ang.cos()[:, None, :], ang.sin()[:, None, :]
    pairs = x.float().reshape(*x.shape[:-1], hd // 2, 2)
    a, b = pairs[..., 0], pairs[..., 1]
    return torch.stack((a * cos - b * sin, a * sin + b * cos), -1).flatten(-2).to(x.dtype)


def rms(x, weight=None, eps=1e-5):
    return F.rms_norm(x, (x.shape[-1],), weight=weight, eps=eps)


def global_attention(c: LMConfig, w, p, x, layer, cache: Cache):
    """Gated GQA with q/k RMS (eps 1e-6), |temp| query scale, interleaved RoPE and a causal mask (lm.py:511-537)."""
    n, nh, nkv, hd = len(x), c.n_heads, c.n_kv_heads, c.head_dim
    gate = F.linear(x, w[p + "gater.weight"]).sigmoid()
    q = F.linear(x, w[p + "wq.weight"]).view(n, nh, hd)
    kv = F.linear(x, w[p + "wkv.weight"].reshape(2 * nkv * hd, c.dim))
    k, v = kv[:, : nkv * hd].reshape(n, nkv, hd), kv[:, nkv * hd:].reshape(n, nkv, hd)
    q = rms(q, eps=1e-6) * w[p + "temp"].abs().view(1, nh, 1)
    k = rms(k, eps=1e-6)
    pos = torch.arange(cache.position, cache.position + n)
    q, k = rope_interleaved(q, pos, c.rope_theta), rope_interleaved(k, pos, c.rope_theta)
    old_k, old_v = cache.kv.get(layer, (k[:0], v[:0]))
    k, v = torch.cat((old_k, k)), torch.cat((old_v, v))
    cache.kv[layer] = (k, v)
    rep = nh // nkv
    key = k.repeat_interleave(rep, 1).transpose(0, 1)
    value = v.repeat_interleave(rep, 1).transpose(0, 1)
    mask = torch.arange(len(k))[None, :] <= pos[:, None]
    out = F.scaled_dot_product_attention(q.transpose(0, 1), key, value, attn_mask=mask, scale=hd ** -0.5)
    return F.linear((out.transpose(0, 1) * gate.unsqueeze(-1)).reshape(n, nh * hd), w[p + "wo.weight"])


def feed_forward(c: LMConfig, w, p, x, layer, capture=None):
    if not c.is_moe(layer):  # dense SwiGLU with the FIRST half multiplied by SiLU(second half) (lm.py:606-609)
        hidden = c.ffn_hidden
        flat = F.linear(x, w[p + "w_in.weight"].reshape(2 * hidden, -1))
        return F.linear(flat[:, :hidden] * F.silu(flat[:, hidden:]), w[p + "w_out.weight"])
    logits = omoe.router_logits(x, w[p + "router.rmsnorm_eda.weight"], w[p + "router.router_linear.weight"], c.norm_eps)
    if capture is not None:
        capture[f"router_logits_{layer}"] = logits
    ids, weights = omoe.route(logits, w[p + "router.balancing_biases"], c.topk)
    routed = F.linear(x, w[p + "latent_down.weight"]) if c.latent else x
    out = omoe.experts_fp32(routed, w[p + "experts.gate_up_proj"], w[p + "experts.down_proj"], ids, weights)
    return F.linear(out, w[p + "latent_up.weight"]) if c.latent else out


def forward(c: LMConfig, w: dict, ids: torch.Tensor, cache: Cache, capture: dict | None = None) -> torch.Tensor:
    """Logits [rows, n_codebooks, audio_vocab] (softcapped) of ids [rows, n_codebooks + 1] continuing ``cache``."""
    x = sum(F.embedding(ids[:, cb], w[f"multi_embedder.embedders.{cb}.weight"]) for cb in range(c.n_codebooks + 1))
    x = rms(x, eps=c.norm_eps)
    sources = [x]
    queries = w["block_attnres_queries"]
    for layer in range(c.n_layers):
        p = f"layers.{layer}."
        h = rms(oattn.full_attnres_route(sources, queries[2 * layer], c.norm_eps), w[p + "attention_norm.weight"],
                c.norm_eps)
        if c.uses_gdn(layer):
            gw = {k[len(p + "attention."):]: v for k, v in w.items() if k.startswith(p + "attention.")}
            h, cache.conv_state[layer], cache.gdn_state[layer] = ogdn.gdn_layer(
                h, gw, cache.conv_state.get(layer), cache.gdn_state.get(layer), heads=c.gdn_heads,
                head_dim=c.gdn_head_dim)
        else:
            h = global_attention(c, w, p + "attention.", h, layer, cache)
        sources.append(h)
        h = rms(oattn.full_attnres_route(sources, queries[2 * layer + 1], c.norm_eps), w[p + "ffn_norm.weight"],
                c.norm_eps)
        sources.append(feed_forward(c, w, p + "feed_forward.", h, layer, capture))
    h = rms(oattn.full_attnres_route(sources, queries[-1], c.norm_eps), w["out_norm.weight"], c.norm_eps)
    logits = F.linear(h, w["multi_output.weight"]).view(len(ids), c.n_codebooks, c.audio_vocab)
    cache.position += len(ids)
    return c.loss_softcap * torch.tanh(logits / c.loss_softcap)


def weight_shapes(c: LMConfig) -> dict:
    """Checkpoint name -> shape of every weight the forward reads."""
    inner = c.gdn_heads * c.gdn_head_dim
    s = {f"multi_embedder.embedders.{cb}.weight": (c.audio_vocab, c.dim) for cb in range(c.n_codebooks)}
    s[f"multi_embedder.embedders.{c.n_codebooks}.weight"] = (c.text_rows, c.dim)
    for layer in range(c.n_layers):
        p = f"layers.{layer}."
        s[p + "attention_norm.weight"] = (c.dim,)
        s[p + "ffn_norm.weight"] = (c.dim,)
        a = p + "attention."
        if c.uses_gdn(layer):
            s.update({a + "in_proj.weight": (4 * inner + 2 * c.gdn_heads, c.dim),
                      a + "conv.weight": (3 * inner, 1, 4), a + "out_weight": (c.gdn_head_dim,),
                      a + "A_log": (c.gdn_heads,), a + "dt_bias": (c.gdn_heads,), a + "wo.weight": (c.dim, inner)})
        else:
            s.update({a + "wq.weight": (c.n_heads * c.head_dim, c.dim), a + "wkv.weight": (2, c.n_kv_heads * c.head_dim, c.dim),
                      a + "wo.weight": (c.dim, c.n_heads * c.head_dim), a + "temp": (1, c.n_heads, 1),
                      a + "gater.weight": (c.n_heads, c.dim)})
        f = p + "feed_forward."
        if c.is_moe(layer):
            s.update({f + "experts.gate_up_proj": (c.n_experts, 2 * c.moe_hidden, c.moe_routed_dim),
                      f + "experts.down_proj": (c.n_experts, c.moe_routed_dim, c.moe_hidden),
                      f + "router.router_linear.weight": (c.n_experts, c.dim), f + "router.rmsnorm_eda.weight": (c.dim,),
                      f + "router.balancing_biases": (c.n_experts,)})
            if c.latent:
                s.update({f + "latent_down.weight": (c.moe_routed_dim, c.dim),
                          f + "latent_up.weight": (c.dim, c.moe_routed_dim)})
        else:
            s.update({f + "w_in.weight": (2, c.ffn_hidden, c.dim), f + "w_out.weight": (c.dim, c.ffn_hidden)})
    s["out_norm.weight"] = (c.dim,)
    s["multi_output.weight"] = (c.n_codebooks * c.audio_vocab, c.dim)
    s["block_attnres_queries"] = (2 * c.n_layers + 1, c.dim)
    return s


def random_weights(c: LMConfig, seed: int = 0, std: float = 0.02) -> dict:
    """Seeded random init: matrices N(0, std^2); norm weights 1; GDN A_log = dt_bias = 0 (decay = exp(-softplus(a)),
    the operator configs' g = -softplus(N(0,1)) when a ~ N(0,1)); balancing biases 0; |temp| = 1."""
    gen = torch.Generator().manual_seed(seed)
    w = {}
    for name, shape in weight_shapes(c).items():
        if name.endswith(("norm.weight", "rmsnorm_eda.weight", "out_weight")):
            w[name] = torch.ones(shape)
        elif name.endswith(("A_log", "dt_bias", "balancing_biases")):
            w[name] = torch.zeros(shape)
        elif name.endswith("temp"):
            w[name] = torch.ones(shape)
        elif name.endswith("conv.weight"):
            w[name] = 0.3 * torch.randn(shape, generator=gen)
        else:
            w[name] = std * torch.randn(shape, generator=gen)
    return w

"""The benchmark's config 1 end to end: a tiny random-init hybrid LM (hidden 256; layers [GDN, GDN, GQA, GDN]; GDN 4 heads
of 64; MoE 8 experts top-2, SwiGLU 512, in every layer; Full AttnRes; vocab 1024) run on the B200 path (the
drop-in OriginalGDN and MoEFeedForward modules, the AttnRes route kernel with the norms fused, the KV store and
the decode attention of the GQA layer, bf16) against the
fp32 oracle LM (oracle/lm.py, pinned to the reference Zonos3LM): a 64-token prompt then greedy decode steps.

Bars: teacher-forced (both models fed the oracle's tokens) logits cosine >= 0.999 at every step; the greedy
argmax agrees on >= 97% of (step, codebook) slots. The first step where free-running greedy sequences diverge
is reported in the assertion context, not required to be absent (bf16 vs fp32 ties flip argmax)."""

from __future__ import annotations

import warnings

import pytest
import torch
import torch.nn.functional as F

from oracle import lm as olm

pytestmark = pytest.mark.gpu

PROMPT, STEPS = 64, 256


class _W:
    def __init__(self, t):
        self.weight = t


class GQA:
    """The reference's gated GQA with KV cache (lm.py:511-537) in plain torch: not on the north_star path."""

    def __init__(self, c, w, p, dev, zb=None, max_tokens=1024):
        self.c, self.zb, self.max_tokens = c, zb, max_tokens
        g = lambda n: w[p + n].to(dev, torch.bfloat16)  # noqa: E731
        self.wq, self.wkv, self.wo, self.gater = g("wq.weight"), g("wkv.weight"), g("wo.weight"), g("gater.weight")
        self.temp = w[p + "temp"].to(dev, torch.float32)
        self.k = self.v = None
        self.kc = self.vc = None  # slot-indexed cache (slot = position) filled through zb.ops.kv_store
        self.position = 0

    def forward(self, x):
        c, n = self.c, len(x)
        nh, nkv, hd = c.n_heads, c.n_kv_heads, c.head_dim
        gate = F.linear(x, self.gater).sigmoid()
        q = F.linear(x, self.wq).view(n, nh, hd)
        kv = F.linear(x, self.wkv.reshape(2 * nkv * hd, c.dim))
        k, v = kv[:, : nkv * hd].reshape(n, nkv, hd), kv[:, nkv * hd:].reshape(n, nkv, hd)
        q = (F.rms_norm(q.float(), (hd,), eps=1e-6) * self.temp.abs().view(1, nh, 1)).to(x.dtype)
        k = F.rms_norm(k.float(), (hd,), eps=1e-6).to(x.dtype)
        pos = torch.arange(self.position, self.position + n, device=x.device)
        freqs = c.rope_theta ** (-torch.arange(0, hd, 2, dtype=torch.float32, device=x.device) / hd)
        ang = pos.float()[:, None] * freqs[None, :]
        cos, sin = ang.cos()[:, None, :], ang.sin()[:, None, :]

        def rope(t):
            pr = t.float().reshape(*t.shape[:-1], hd // 2, 2)
            a, b = pr[..., 0], pr[..., 1]
            return torch.stack((a * cos - b * sin, a * sin + b * cos), -1).flatten(-2).to(t.dtype)

        q, k = rope(q), rope(k)
        if self.zb is not None:  # the B200 KV store and, for a decode row, the B200 decode attention
            if self.kc is None:
                self.kc = torch.zeros(self.max_tokens, nkv, hd, device=x.device, dtype=x.dtype)
                self.vc = torch.zeros_like(self.kc)
            slots = torch.arange(self.position, self.position + n, device=x.device, dtype=torch.int32)
            self.zb.ops.kv_store(self.kc, self.vc, slots, k, v)
            if n == 1:
                table = torch.arange(self.max_tokens, device=x.device, dtype=torch.int32)[None]
                seq = torch.tensor([self.position + 1], device=x.device, dtype=torch.int32)
                out = self.zb.ops.gqa_decode(q, self.kc, self.vc, table, seq, softmax_scale=hd ** -0.5)
                self.position += n
                return F.linear((out * gate.unsqueeze(-1)).reshape(n, nh * hd), self.wo)
            k, v = self.kc[: self.position + n], self.vc[: self.position + n]
            self.k, self.v = k, v
        else:
            self.k = k if self.k is None else torch.cat((self.k, k))
            self.v = v if self.v is None else torch.cat((self.v, v))
        rep = nh // nkv
        key = self.k.repeat_interleave(rep, 1).transpose(0, 1)
        value = self.v.repeat_interleave(rep, 1).transpose(0, 1)
        mask = torch.arange(len(self.k), device=x.device)[None, :] <= pos[:, None]
        out = F.scaled_dot_product_attention(q.transpose(0, 1), key, value, attn_mask=mask, scale=hd ** -0.5)
        self.position += n
        return F.linear((out.transpose(0, 1) * gate.unsqueeze(-1)).reshape(n, nh * hd), self.wo)


class Layer:
    pass


class B200LM:
    def __init__(self, zb, c: olm.LMConfig, w: dict):
        dev = torch.device("cuda")
        self.zb, self.c, self.dev = zb, c, dev
        bf = lambda t: t.to(dev, torch.bfloat16)  # noqa: E731
        self.emb = [bf(w[f"multi_embedder.embedders.{cb}.weight"]) for cb in range(c.n_codebooks + 1)]
        self.queries = bf(w["block_attnres_queries"])
        self.out_norm = bf(w["out_norm.weight"])
        self.head = bf(w["multi_output.weight"])
        mcfg = zb.config.ModelConfig(hidden_size=c.dim, gdn_num_heads=c.gdn_heads, gdn_head_dim=c.gdn_head_dim,
                                     moe_n_experts=c.n_experts, moe_topk=c.topk, moe_intermediate_size=c.moe_hidden,
                                     moe_alpha=1.0, norm_topk_prob=False, use_training_router_weights=True,
                                     rms_norm_eps=c.norm_eps)
        self.layers = []
        for i in range(c.n_layers):
            p = f"layers.{i}."
            layer = Layer()
            layer.attention_norm, layer.ffn_norm = _W(bf(w[p + "attention_norm.weight"])), _W(bf(w[p + "ffn_norm.weight"]))
            if c.uses_gdn(i):
                gdn = zb.gdn.OriginalGDN(mcfg, i)
                gdn.load_state_dict({k[len(p + "attention."):]: v for k, v in w.items() if k.startswith(p + "attention.")})
                gdn.to(dev, torch.bfloat16)
                gdn.allocate_cache(1, dev, torch.bfloat16)
                layer.attention = gdn
            else:
                layer.attention = GQA(c, w, p + "attention.", dev, zb)
            ff = zb.moe.MoEFeedForward(mcfg, i)
            ff.load_state_dict({k[len(p + "feed_forward."):]: v for k, v in w.items()
                                if k.startswith(p + "feed_forward.")})
            ff.to(dev, torch.bfloat16)
            layer.feed_forward, layer.is_moe = ff, True
            self.layers.append(layer)
        self.states = {}
        self.position = 0

    def forward(self, ids):
        zb, c = self.zb, self.c
        n = len(ids)
        ids = ids.to(self.dev)
        x = sum(F.embedding(ids[:, cb], self.emb[cb]) for cb in range(c.n_codebooks + 1))
        x = F.rms_norm(x.float(), (c.dim,), eps=c.norm_eps).to(torch.bfloat16)
        if n not in self.states:
            self.states[n] = zb.attnres.FusedBlockAttnResContext(2 * c.n_layers, x)
        batch = zb.core.Batch(reqs=[zb.core.Req(0, n, self.position)], is_decode=self.position > 0 and n == 1)
        with zb.core.forward_batch(batch):
            h = zb.attnres.forward_layers_full(self.layers, x, self.queries, c.norm_eps, self.states[n], self.out_norm)
        self.position += n
        logits = F.linear(h, self.head).float().view(n, c.n_codebooks, c.audio_vocab)
        return c.loss_softcap * torch.tanh(logits / c.loss_softcap)


def test_cfg1_tiny_lm_prompt_and_greedy_decode(zb, record_property):
    c = olm.LMConfig()  # cfg1 shapes
    w = olm.random_weights(c, seed=0)
    gen = torch.Generator().manual_seed(0)
    prompt = torch.cat([torch.randint(0, c.codebook_size, (PROMPT, c.n_codebooks), generator=gen),
                        torch.randint(0, c.text_rows, (PROMPT, 1), generator=gen)], 1)
    ours = B200LM(zb, c, w)
    cache = olm.Cache()
    ref_logits = olm.forward(c, w, prompt, cache)[-1:]
    got_logits = ours.forward(prompt)[-1:].cpu()
    cosines, agree, first_divergence = [], [], None
    free_ref, free_ours = [], []
    for step in range(STEPS):
        cos = F.cosine_similarity(got_logits.flatten(), ref_logits.flatten(), dim=0).item()
        cosines.append(cos)
        tok_ref, tok_ours = ref_logits.argmax(-1), got_logits.argmax(-1)
        agree.append((tok_ref == tok_ours).float().mean().item())
        if first_divergence is None and not torch.equal(tok_ref, tok_ours):
            first_divergence = step
        free_ref.append(tok_ref)
        free_ours.append(tok_ours)
        # teacher forcing: both continue from the oracle's greedy tokens (text row: padding id)
        nxt = torch.cat([tok_ref, torch.full((1, 1), c.text_rows - 1)], 1)
        ref_logits = olm.forward(c, w, nxt, cache)
        got_logits = ours.forward(nxt).cpu()
    msg = f"min cosine {min(cosines):.5f}, argmax agreement {sum(agree) / len(agree):.4f}, " \
          f"first greedy divergence at step {first_divergence}"
    print(f"cfg1: {msg}")
    # kept in the run's record: the junit property and a warning in pytest's summary
    record_property("cfg1_min_cosine", min(cosines))
    record_property("cfg1_first_greedy_divergence", first_divergence)
    warnings.warn(f"cfg1 tiny LM: {msg}")
    assert min(cosines) >= 0.999, msg
    assert sum(agree) / len(agree) >= 0.97, msg
    assert zb.ops.device_status() == 0

"""Generate the golden fixtures of ``tests/golden/`` by running the UNMODIFIED reference oracle
(``zonos3.reference.lm`` from the reference checkout's ``model/src``) on seeded inputs.

    python tests/golden/make_golden.py /path/to/reference

Each fixture stores the inputs, the layer weights and the reference's outputs, so the tests never need the
reference at run time. What each file pins:

* ``gdn_tiny.npz``   — ``Zonos3LM._gdn`` (lm.py:556-602) on a 12-row prefill followed by three 1-row decode calls:
  conv, q, k, v, decay, beta, recurrent output, gated output, layer output, and the GDN / conv states after
  the prefill and after the last decode call (float32 model, 4 heads of 128).
* ``attnres.npz``    — ``full_attnres_route`` (lm.py:384-389) on float32 and bf16 banks, including the
  production width D=2048 and a one-source bank.
* ``moe_tiny.npz``   — ``Zonos3LM._feed_forward`` (lm.py:604-639) of a MoE layer (float32): router logits, the
  ``torch.topk`` indices the reference computed, and the layer output.
* ``moe_ties.npz``   — the same layer cast to bf16 with zero balancing biases, where bf16 logits tie often:
  the reference's ``torch.topk`` indices, to measure where its tie order is arbitrary.
* ``lm_tiny.npz``    — ``Zonos3LM.forward`` (lm.py:660-735) of a whole 2-layer model (GDN layer + global attention
  layer, dense FFN then MoE, Full AttnRes, dim 32): every weight, a 12-row prompt and two 1-row decode calls, and
  the softcapped logits of all three calls.

* ``sampler.npz``    — ``sample_tts`` (model/src/zonos3/tts/sampler.py:159-372): seeded logits with masks, stop
  bias and repetition penalty, and the ids the reference drew (greedy and seeded multinomial) for four settings.

``python tests/golden/make_golden.py /path/to/reference [fixture ...]`` regenerates only the named fixtures.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent

CONFIG = {
    "n_layers": 2,
    "dim": 64,
    "head_dim": 16,
    "n_heads": 4,
    "n_kv_heads": 2,
    "norm_eps": 1e-5,
    "rope_theta": 10000.0,
    "max_seqlen": 256,
    "loss_softcap": 15.0,
    "ffn_dim_multiplier": 2.0,
    "multiple_of": 32,
    "moe_ffn_dim_multiplier": 1.0,
    "moe_multiple_of": 32,
    "moe_alpha": 0.5,
    "moe_n_experts": 4,
    "n_codebooks": 10,
    "codebook_size": 16,
    "eoa_id": 16,
    "audio_pad_id": 17,
    "text_vocab": 20,
    "speaker_embedding_dim": 8,
    "attention_pattern": "gdn1_global1",
    "residual_type": "full_attnres",
    "use_xsa": False,
    "speaker_enabled": True,
    "condition_tokens_enabled": True,
    "moe_router_type": "linear",
    "moe_router_use_eda": False,
    "moe_balancing_strategy": "quantile",
    "moe_router_topk": 2,
    "moe_start_from_layer": 1,
    "moe_end_from_layer": 0,
    "condition_count": 1,
    "condition_n_buckets": 4,
    "condition_names": ["loudness"],
}


def build_model(lm, seed, **overrides):
    model = lm.Zonos3LM(lm.Zonos3LMConfig.from_params({"model": {**CONFIG, **overrides}}))
    gen = torch.Generator().manual_seed(seed)
    for name, param in model.named_parameters():
        noise = torch.randn(param.shape, generator=gen)
        if name.endswith(("norm.weight", "rmsnorm_eda.weight", "out_weight")):
            param.data = 1.0 + 0.1 * noise
        elif name.endswith("balancing_biases"):
            param.data = 0.1 * noise
        elif name.endswith(("A_log", "dt_bias")):
            param.data = 0.5 * noise
        else:
            param.data = 0.1 * noise
    return model.eval()


def weights_of(module, prefix=""):
    return {prefix + name: p.detach().float().numpy().copy() for name, p in module.named_parameters()}


def gdn_fixture(lm):
    model = build_model(lm, seed=11)
    gen = torch.Generator().manual_seed(12)
    x = torch.randn(15, CONFIG["dim"], generator=gen)
    cache = lm.LMCache()
    rows = {}
    outputs = []
    out = {}
    for call, (lo, hi) in enumerate(((0, 12), (12, 13), (13, 14), (14, 15))):
        model._capture = {}
        y = model._gdn(x[lo:hi], 0, cache)
        outputs.append(y)
        cap = model._capture
        model._capture = None
        for name in ("gdn_conv", "gdn_q", "gdn_k", "gdn_v", "gdn_decay", "gdn_beta", "gdn_recurrent", "gdn_gated"):
            rows.setdefault(name, []).append(cap[f"{name}_0"])
        if call in (0, 3):
            tag = "prefill" if call == 0 else "final"
            out[f"state_{tag}"] = cap["gdn_state_0"]
            out[f"conv_state_{tag}"] = cap["gdn_conv_state_0"]
    out.update({name: np.concatenate(v) for name, v in rows.items()})
    out["y"] = torch.cat(outputs).numpy()
    out["x"] = x.numpy()
    out.update(weights_of(model.layers[0].attention, "w."))
    np.savez_compressed(HERE / "gdn_tiny.npz", **out)


def attnres_fixture(lm):
    out = {}
    cases = (("f32", torch.float32, 5, 7, 64), ("bf16", torch.bfloat16, 9, 4, 2048), ("one", torch.bfloat16, 1, 3, 256))
    for tag, dtype, S, T, D in cases:
        gen = torch.Generator().manual_seed(20 + S)
        sources = [(torch.randn(T, D, generator=gen) * (1 + s)).to(dtype) for s in range(S)]
        query = (0.02 * torch.randn(D, generator=gen) * 20).to(dtype)
        mixed = lm.full_attnres_route(sources, query, 1e-5)
        out[f"{tag}_sources"] = torch.stack(sources).float().numpy()
        out[f"{tag}_query"] = query.float().numpy()
        out[f"{tag}_out"] = mixed.float().numpy()
    np.savez_compressed(HERE / "attnres.npz", **out)


class TopkRecorder:
    def __init__(self):
        self.calls = []
        self._topk = torch.topk

    def __enter__(self):
        def topk(input, k, *args, **kwargs):
            result = self._topk(input, k, *args, **kwargs)
            self.calls.append((input.detach().clone(), result.indices.clone()))
            return result

        torch.topk = topk
        return self

    def __exit__(self, *exc):
        torch.topk = self._topk


def moe_fixture(lm):
    model = build_model(lm, seed=31, moe_n_experts=16, moe_alpha=1.0)
    gen = torch.Generator().manual_seed(32)
    x = torch.randn(24, CONFIG["dim"], generator=gen)
    model._capture = {}
    with TopkRecorder() as rec:
        y = model._feed_forward(x, 1)
    cap = model._capture
    model._capture = None
    (scores, indices), = rec.calls
    out = {"x": x.numpy(), "y": y.numpy(), "logits": cap["router_logits_1"], "scores": scores.numpy(),
           "topk": indices.numpy()}
    out.update(weights_of(model.layers[1].feed_forward, "w."))
    np.savez_compressed(HERE / "moe_tiny.npz", **out)

    tied = build_model(lm, seed=33, moe_n_experts=16, moe_alpha=1.0)
    tied.layers[1].feed_forward.router.balancing_biases.data.zero_()
    tied.cast(torch.bfloat16)
    x = torch.randn(256, CONFIG["dim"], generator=gen).bfloat16()
    with TopkRecorder() as rec:
        tied._feed_forward(x, 1)
    (scores, indices), = rec.calls
    np.savez_compressed(HERE / "moe_ties.npz", scores=scores.numpy(), topk=indices.numpy())


def lm_fixture(lm):
    model = build_model(lm, seed=41, dim=32)
    gen = torch.Generator().manual_seed(42)
    rows = 14
    ids = torch.full((rows, CONFIG["n_codebooks"] + 1), CONFIG["codebook_size"] + 1, dtype=torch.long)
    ids[:, -1] = torch.randint(4, CONFIG["text_vocab"], (rows,), generator=gen)
    ids[8:, :-1] = torch.randint(0, CONFIG["codebook_size"], (rows - 8, CONFIG["n_codebooks"]), generator=gen)
    cache = lm.LMCache()
    logits = [model(ids[:12], cache).logits, model(ids[12:13], cache).logits, model(ids[13:14], cache).logits]
    out = {"ids": ids.numpy(), "logits": torch.cat(logits).numpy()}
    out.update({"w." + k: v.detach().float().numpy().copy() for k, v in model.state_dict().items()})
    np.savez_compressed(HERE / "lm_tiny.npz", **out)


SAMPLER_CASES = [  # (temperatures, top_ks, top_ps, min_ps)
    ([0.0, 0.0, 0.0], [0, 0, 0], [1.0, 1.0, 1.0], [0.0, 0.0, 0.0]),
    ([0.7, 1.0, 1.3], [20, 30, 40], [0.9, 0.8, 0.5], [0.0, 0.05, 0.0]),
    ([1.0, 1.0, 1.0], [0, 0, 0], [0.95, 0.95, 0.95], [0.0, 0.0, 0.0]),
    ([0.5, 0.5, 0.5], [5, 5, 5], [1.0, 1.0, 1.0], [0.1, 0.1, 0.1]),
]


def sampler_fixture(_lm):
    """``sample_tts`` (model/src/zonos3/tts/sampler.py:159-372) on seeded fp32 logits [3, 4, 70] (codebook 64, EOA 64,
    padding 65, span-end 66) with a stop-id mix, a repetition window, per-codebook sizes, a blocked stop and a stop
    bias: the ids of each case with per-request generators seeded 100 + b."""
    from zonos3.tts import sampler as ref

    g = torch.Generator().manual_seed(0)
    B, C, V = 3, 4, 70
    logits = torch.randn(B, C, V, generator=g) * 3
    stop = torch.tensor([64, 64, 66])
    rep = torch.randint(0, V, (B, C, 5), generator=g)
    pen = torch.tensor([1.0, 1.3, 2.0])
    sizes = [64, 60, 64, 50]
    blocked = torch.zeros(B, C, dtype=torch.bool)
    blocked[1, 2] = True
    bias = torch.tensor([0.0, 2.5, -1.0])
    out = {"logits": logits.numpy(), "stop": stop.numpy(), "rep": rep.numpy(), "pen": pen.numpy(),
           "sizes": np.array(sizes), "blocked": blocked.numpy(), "bias": bias.numpy()}
    for n, (temps, tk, tp, mp) in enumerate(SAMPLER_CASES):
        gens = [torch.Generator().manual_seed(100 + i) for i in range(B)]
        ids = ref.sample_tts(logits.clone(), torch.tensor(temps, dtype=torch.float32), torch.tensor(tk),
                             torch.tensor(tp), torch.tensor(mp), codebook_size=64, audio_pad_id=65,
                             stop_token_ids=stop, repetition_token_ids=rep, repetition_penalties=pen,
                             codebook_sizes=sizes, text_vocab=7, generators=gens, stop_blocked=blocked,
                             stop_bias=bias)
        out[f"case{n}"] = np.array([temps, tk, tp, mp], dtype=np.float64)
        out[f"ids{n}"] = ids.numpy()
    np.savez_compressed(HERE / "sampler.npz", **out)


FIXTURES = {"gdn": "gdn_fixture", "attnres": "attnres_fixture", "moe": "moe_fixture", "lm": "lm_fixture",
            "sampler": "sampler_fixture"}


def main(reference: str, which: list[str]) -> None:
    sys.path.insert(0, str(Path(reference) / "model" / "src"))
    import zonos3.reference.lm as lm

    torch.set_num_threads(1)
    for name in which or list(FIXTURES):
        globals()[FIXTURES[name]](lm)
    for f in sorted(HERE.glob("*.npz")):
        print(f.name, f.stat().st_size)


if __name__ == "__main__":
    if len(sys.argv) < 2:
        sys.exit("usage: python tests/golden/make_golden.py /path/to/reference [fixture ...]")
    main(sys.argv[1], sys.argv[2:])

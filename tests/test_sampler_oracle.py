"""CPU: the sampler oracle (oracle/sampler.py) against ids the unmodified reference's sample_tts drew
(tests/golden/sampler.npz, made by tests/golden/make_golden.py): greedy ids equal the oracle's argmax, and drawing
from the oracle's distributions with the reference's seeded generators (over each row's vocabulary width, as the
reference does) reproduces the reference's sampled ids exactly."""

from __future__ import annotations

import torch

from oracle import sampler as osam


def test_oracle_reproduces_reference_ids(golden):
    g = golden("sampler.npz")
    logits = g["logits"]
    B, C, V = logits.shape
    stop = g["stop"]
    args = dict(codebook_size=64, audio_pad_id=65, stop_token_ids=stop, codebook_sizes=g["sizes"].tolist(),
                stop_blocked=g["blocked"], stop_bias=g["bias"], repetition_token_ids=g["rep"],
                repetition_penalties=g["pen"])
    widths = [max(int(s), 65) + 1 for s in stop]
    n = 0
    while f"case{n}" in g:
        temps, tk, tp, mp = g[f"case{n}"]
        probs, greedy = osam.final_probs(logits, temps.tolist(), int(min(tk)), float(max(tp)), float(max(mp)), **args)
        if (temps <= 0).all():
            ids = greedy
        else:
            gens = [torch.Generator().manual_seed(100 + i) for i in range(B)]
            ids = torch.cat([torch.multinomial(probs[i * C:(i + 1) * C, :widths[i]].contiguous(), 1, generator=gens[i])
                             for i in range(B)]).view(B, C)
        ref = g[f"ids{n}"]
        assert torch.equal(ids.long(), ref[:, :C].long()), n
        assert (ref[:, C] == 7).all()
        n += 1
    assert n == 4

"""GPU: the TTS sampler kernel (zb_sample_tts) through the C ABI.

* the final distribution of every (request, codebook) row (probs_out) against the oracle (oracle/sampler.py, pinned
  to the reference's sample_tts) within 1e-5, for masks, stop bias, blocked stops, per-codebook sizes, repetition
  penalty, temperature, top-k, top-p and min-p, on fp32 and bf16 logits of the production vocabulary (4098);
* greedy ids equal to the ids the reference drew (tests/golden/sampler.npz) and to the oracle's argmax;
* sampled ids: never an id of zero probability, and the frequencies of 24,000 draws within 5 sigma of the oracle's
  probabilities (the draw uses its own Philox stream, so ids match the reference in distribution only);
* rows with more ties at the k-th value than the sorted top-k path holds, and a codebook with fewer finite logits
  than k: their distributions against the oracle as well."""

from __future__ import annotations

import pytest
import torch

from oracle import sampler as osam

pytestmark = pytest.mark.gpu

CB, PAD, V = 4096, 4097, 4098


def _inputs(gen, B, C, V=V, scale=3.0):
    logits = torch.randn(B, C, V, generator=gen) * scale
    stop = torch.full((B,), CB, dtype=torch.int32)
    rep = torch.randint(0, V, (B, C, 16), generator=gen, dtype=torch.int32)
    rep[:, :, -1] = -1  # an unused slot of the window
    pen = torch.linspace(1.0, 1.8, B)
    sizes = [CB] * (C - 1) + [CB - 96]
    blocked = torch.zeros(B, C, dtype=torch.bool)
    blocked[0, 1] = True
    bias = torch.linspace(-1.0, 1.5, B)
    return logits, dict(codebook_size=CB, audio_pad_id=PAD, stop_token_ids=stop, codebook_sizes=sizes,
                        stop_blocked=blocked, stop_bias=bias, repetition_token_ids=rep, repetition_penalties=pen)


def _run(zb, logits, temps, tk, tp, mp, args, dtype=torch.float32, seed=0, offset=0):
    dev = torch.device("cuda")
    B, C, Vv = logits.shape
    probs = torch.empty(B * C, Vv, device=dev, dtype=torch.float32)
    out = zb.ops.sample_tts(logits.to(dev, dtype), temps, [tk] * B, [tp] * B, [mp] * B,
                            codebook_size=args["codebook_size"], audio_pad_id=args["audio_pad_id"],
                            stop_token_ids=args["stop_token_ids"], repetition_token_ids=args["repetition_token_ids"],
                            repetition_penalties=args["repetition_penalties"], codebook_sizes=args["codebook_sizes"],
                            stop_blocked=args["stop_blocked"], stop_bias=args["stop_bias"], text_vocab=11,
                            seed=seed, offset=offset, probs_out=probs)
    return out.cpu(), probs.cpu()


@pytest.mark.parametrize("temps,tk,tp,mp", [(0.8, 0, 1.0, 0.0), (1.0, 50, 1.0, 0.0), (0.7, 0, 0.9, 0.0),
                                            (1.2, 200, 0.8, 0.02), (0.5, 0, 1.0, 0.05), (1.0, 1, 1.0, 0.0)])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_distribution_matches_oracle(zb, temps, tk, tp, mp, dtype):
    gen = torch.Generator().manual_seed(int(temps * 10) + tk)
    B, C = 4, 10
    logits, args = _inputs(gen, B, C)
    logits = logits.to(dtype).float()  # the oracle sees the values the kernel reads
    tlist = [temps] * B
    out, probs = _run(zb, logits, tlist, tk, tp, mp, args, dtype=dtype)
    ref, _ = osam.final_probs(logits, tlist, tk, tp, mp, **args)
    torch.testing.assert_close(probs, ref, atol=1e-5, rtol=1e-4)
    ids = out[:, :C].reshape(-1)
    assert (ref[torch.arange(B * C), ids.long()] > 0).all()  # every draw has probability
    assert (out[:, C] == 11).all()


def test_greedy_matches_reference_ids(zb, golden):
    g = golden("sampler.npz")
    logits = g["logits"]
    B, C, Vv = logits.shape
    args = dict(codebook_size=64, audio_pad_id=65, stop_token_ids=g["stop"].int(), codebook_sizes=g["sizes"].tolist(),
                stop_blocked=g["blocked"], stop_bias=g["bias"].float(), repetition_token_ids=g["rep"].int(),
                repetition_penalties=g["pen"].float())
    out, probs = _run(zb, logits, [0.0] * B, 0, 1.0, 0.0, args)
    ref = g["ids0"]
    assert torch.equal(out[:, :C].long(), ref[:, :C].long())
    assert torch.equal(out[:, C].long(), torch.full((B,), 11))
    # the sampled cases: the kernel's distributions equal the oracle's, whose draws reproduce the reference ids
    n = 1
    while f"case{n}" in g:
        temps, tk, tp, mp = g[f"case{n}"].tolist()
        _, probs = _run(zb, logits, temps, int(min(tk)), float(max(tp)), float(max(mp)), args)
        ref_p, _ = osam.final_probs(logits, temps, int(min(tk)), float(max(tp)), float(max(mp)), **args)
        torch.testing.assert_close(probs, ref_p, atol=1e-5, rtol=1e-4)
        n += 1


def test_greedy_production_vocab(zb):
    gen = torch.Generator().manual_seed(9)
    logits, args = _inputs(gen, 16, 10)
    out, _ = _run(zb, logits, [0.0] * 16, 0, 1.0, 0.0, args)
    _, ref = osam.final_probs(logits, [0.0] * 16, 0, 1.0, 0.0, **args)
    assert torch.equal(out[:, :10].long(), ref.long())


def test_draw_frequencies(zb):
    """2,000 identical rows x 12 offsets: the empirical frequencies of a 70-id row against the oracle."""
    gen = torch.Generator().manual_seed(4)
    base = torch.randn(1, 1, 70, generator=gen) * 1.5
    B = 2000
    logits = base.expand(B, 1, 70).contiguous()
    args = dict(codebook_size=64, audio_pad_id=65, stop_token_ids=torch.full((B,), 64, dtype=torch.int32),
                codebook_sizes=None, stop_blocked=None, stop_bias=None, repetition_token_ids=None,
                repetition_penalties=None)
    counts = torch.zeros(70)
    for off in range(12):
        out, _ = _run(zb, logits, [0.9] * B, 40, 0.95, 0.0, args, seed=1234, offset=off)
        counts += torch.bincount(out[:, 0].long(), minlength=70).float()
    n = counts.sum()
    ref, _ = osam.final_probs(base, [0.9], 40, 0.95, 0.0, **{**args, "stop_token_ids": torch.tensor([64])})
    p = ref[0]
    assert counts[p == 0].sum() == 0
    sigma = (p * (1 - p) / n).sqrt()
    assert ((counts / n - p).abs() <= 5 * sigma + 1e-4).all()


def test_tiny_top_p_keeps_the_top_id(zb):
    gen = torch.Generator().manual_seed(6)
    logits, args = _inputs(gen, 3, 10)
    out, _ = _run(zb, logits, [1.0] * 3, 0, 1e-6, 0.0, args)
    _, greedy = osam.final_probs(logits, [0.0] * 3, 0, 1.0, 0.0, **args)
    assert torch.equal(out[:, :10].long(), greedy.long())


def test_rejects_bad_arguments(zb):
    dev = torch.device("cuda")
    logits = torch.zeros(1, 1, 20000, device=dev)
    with pytest.raises(ValueError):
        zb.ops.sample_tts(logits, [1.0], [0], [1.0], [0.0], codebook_size=16000, audio_pad_id=16001,
                          stop_token_ids=[16000])
    with pytest.raises(ValueError):
        zb.ops.sample_tts(logits[:, :, :100], [1.0], [0], [1.0], [0.0], codebook_size=100, audio_pad_id=101,
                          stop_token_ids=[100])


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_fused_softcap_matches_torch(zb, dtype):
    """softcap = 15 on the raw head output: the same distribution as torch's soft cap (evaluated on the GPU in the
    head's dtype, as compute_logits does) followed by the oracle; greedy ids identical."""
    gen = torch.Generator().manual_seed(13)
    logits, args = _inputs(gen, 4, 10, scale=20.0)
    dev = torch.device("cuda")
    raw = logits.to(dev, dtype)
    capped = (15.0 * torch.tanh(raw / 15.0)).float().cpu()  # the reference's softcap in the head's dtype
    kw = dict(codebook_size=CB, audio_pad_id=PAD, stop_token_ids=args["stop_token_ids"],
              repetition_token_ids=args["repetition_token_ids"], repetition_penalties=args["repetition_penalties"],
              codebook_sizes=args["codebook_sizes"], stop_blocked=args["stop_blocked"], stop_bias=args["stop_bias"])
    probs = torch.empty(40, V, device=dev)
    zb.ops.sample_tts(raw, [0.9] * 4, [0] * 4, [0.9] * 4, [0.0] * 4, softcap=15.0, probs_out=probs, **kw)
    ref, _ = osam.final_probs(capped, [0.9] * 4, 0, 0.9, 0.0, **args)
    torch.testing.assert_close(probs.cpu(), ref, atol=1e-5, rtol=1e-4)
    ids = zb.ops.sample_tts(raw, [0.0] * 4, [0] * 4, [1.0] * 4, [0.0] * 4, softcap=15.0, **kw)
    _, greedy = osam.final_probs(capped, [0.0] * 4, 0, 1.0, 0.0, **args)
    assert torch.equal(ids[:, :10].cpu().long(), greedy.long())


def test_tied_rows_and_short_codebooks(zb):
    """Top-k 50 with 300 ids tied at the largest logit (every tie survives the top-k), and a codebook whose size
    leaves fewer finite logits than k (the k-th value is -inf, so every id survives the top-k and the mass decides);
    beside ordinary rows. Every row's distribution against the oracle."""
    gen = torch.Generator().manual_seed(12)
    B, C = 3, 10
    logits, args = _inputs(gen, B, C)
    logits[0, 2, 100:400] = 20.0  # 300 ids tied at the top
    args["codebook_sizes"] = [CB] * 4 + [20] + [CB] * (C - 5)  # codebook 4: 20 finite ids (+ the stop id)
    args["repetition_token_ids"] = None
    args["repetition_penalties"] = None
    out, probs = _run(zb, logits, [0.9] * B, 50, 0.95, 0.0, args)
    ref, _ = osam.final_probs(logits, [0.9] * B, 50, 0.95, 0.0, **args)
    torch.testing.assert_close(probs, ref, atol=1e-5, rtol=1e-4)
    ids = out[:, :C].reshape(-1)
    assert (ids >= 0).all()
    assert (ref[torch.arange(B * C), ids.long()] > 0).all()

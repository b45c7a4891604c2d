"""Sampler oracle (CPU, float32): the deterministic part of sample_tts (model/src/zonos3/tts/sampler.py:159-372)
restated — invalid-id masks and stop bias (:238-253), repetition penalty (apply_repetition_penalty, :83-108), the
greedy path (:288-289), temperature, top-k, softmax, top-p (apply_top_p, :59-69), min-p (apply_min_p, :72-80) and
the empty-row fallback (:308-313) — returning the final per-row distribution and the greedy ids. The multinomial
draw itself is left to the caller (torch.multinomial with the reference's generators reproduces the reference's
ids from these probabilities). Test infrastructure only (see ``oracle/__init__.py``).
"""

from __future__ import annotations

import torch


def masked_logits(logits, *, codebook_size, audio_pad_id, stop_token_ids, codebook_sizes=None, stop_blocked=None,
                  stop_bias=None, repetition_token_ids=None, repetition_penalties=None):
    """Logits [B, C, V] (float32) after the invalid-id masks, the stop bias and the repetition penalty."""
    B, C, V = logits.shape
    x = logits.float().clone()
    ids = torch.arange(V).view(1, 1, V)
    stop = torch.as_tensor(stop_token_ids).long().view(B, 1, 1)
    invalid = (ids == audio_pad_id) | ((ids >= codebook_size) & (ids != stop))
    if codebook_sizes is not None:
        limits = torch.as_tensor(codebook_sizes).view(1, C, 1)
        invalid = invalid | ((ids >= limits) & (ids < codebook_size))
    if stop_blocked is not None:
        invalid = invalid | ((ids == stop) & torch.as_tensor(stop_blocked).bool().view(B, C, 1))
    x = x.masked_fill(invalid, float("-inf"))
    if stop_bias is not None:
        x = x + (ids == stop) * torch.as_tensor(stop_bias).float().view(B, 1, 1)
    if repetition_token_ids is not None and repetition_penalties is not None and repetition_token_ids.numel():
        rep = torch.as_tensor(repetition_token_ids)
        valid = (rep >= 0) & (rep < V)
        counts = torch.zeros(B, C, V, dtype=torch.int32)
        counts.scatter_add_(-1, rep.clamp(0, V - 1).long(), valid.to(torch.int32))
        pen = torch.as_tensor(repetition_penalties).float().view(B, 1, 1).clamp(min=1.0)
        x = torch.where(counts > 0, torch.where(x > 0, x / pen, x * pen), x)
    return x


def final_probs(logits, temperatures, top_k, top_p, min_p, **mask_args):
    """(probs [B*C, V], greedy ids [B, C]) of sample_tts for batch-level top_k / top_p / min_p. Greedy rows (every
    temperature <= 0) get a one-hot distribution. Top-p follows the reference's sorted-cumsum rule with a stable
    sort: equal probabilities are ranked by index, as torch's CUDA sort of the production vocabulary (a stable
    radix sort above 4096 entries) ranks them."""
    x = masked_logits(logits, **mask_args)
    B, C, V = x.shape
    temps = torch.as_tensor(temperatures).float()
    if bool((temps <= 0).all()):
        ids = x.argmax(-1)
        return torch.nn.functional.one_hot(ids.view(-1), V).float(), ids
    flat = (x / temps.view(B, 1, 1).clamp(min=1e-8)).view(B * C, V)
    if 0 < top_k < V:
        kth = torch.topk(flat, top_k, dim=-1).values[..., -1:]
        flat = flat.masked_fill(flat < kth, float("-inf"))
    probs = torch.softmax(flat, -1)
    if 0.0 < top_p < 1.0:  # sorted cumulative mass before each id (= the mass strictly above it when distinct)
        srt, idx = torch.sort(probs, dim=-1, descending=True, stable=True)  # CUDA's sort of V > 4096 is stable
        srt = srt.masked_fill(torch.cumsum(srt, -1) - srt > top_p, 0.0)
        probs = probs.scatter(-1, idx, srt)
        probs = probs / probs.sum(-1, keepdim=True).clamp(min=1e-8)
    if min_p > 0.0:
        probs = probs.masked_fill(probs < min_p * probs.max(-1, keepdim=True).values, 0.0)
        probs = probs / probs.sum(-1, keepdim=True).clamp(min=1e-8)
    empty = probs.sum(-1) <= 0
    greedy = flat.argmax(-1)
    probs = torch.where(empty[:, None], torch.nn.functional.one_hot(greedy, V).float(), probs)
    return probs, greedy.view(B, C)

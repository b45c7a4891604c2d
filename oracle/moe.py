"""MoE oracle (CPU; the expert functions also run unchanged on CUDA tensors as a plain fp32 PyTorch reference
for sizes the CPU cannot finish quickly, with TF32 off): router, top-k selection, token permutation and the routed SwiGLU experts.

Restates ``Zonos3LM._feed_forward`` (model/src/zonos3/reference/lm.py:604-639), the serving router
(servers/sgl/src/zonos3_sgl/models/zonos3.py:746-828) and FusedMoE's renormalisation
(servers/sgl/src/zonos3_sgl/layers/moe/fused_moe/layer.py:159-161).

Tie rule. ``torch.topk`` leaves the order of equal scores unspecified (on CPU it differs even between k and k+1),
and the reference's CPU oracle and CUDA server disagree there. This oracle and the CUDA router therefore use one
total order: descending score, then ascending expert index. ``tests/test_oracle_golden.py`` checks that it gives
the reference's own ``torch.topk`` result on every row where the reference's answer does not depend on a tie.

Permutation contract. The (token, slot) pairs, flattened as p = token * k + slot, are stably sorted by expert:
pairs of one expert keep ascending p. Every expert's segment can be padded to a multiple of ``block`` rows.

Test infrastructure only (see ``oracle/__init__.py``).
"""

from __future__ import annotations

import numpy as np
import torch
import torch.nn.functional as F


def select_topk(scores, k):
    """Indices [T, k] of the k largest scores per row, ties broken by lower index (stable descending sort)."""
    return torch.sort(scores, dim=-1, descending=True, stable=True).indices[..., :k]


def router_logits(x, norm_weight, w_router, eps):
    """logits = router_linear(rmsnorm_eda(x)) in x's dtype (lm.py:610-611; zonos3.py:815-822)."""
    return F.linear(F.rms_norm(x, (x.shape[-1],), weight=norm_weight, eps=eps), w_router)


def route(logits, bias, k, *, weights="selected_softmax", renormalize=False):
    """Top-k ids (int32) and fp32 weights from router logits (lm.py:613-617; zonos3.py:746-766, 822-828).

    ``weights="selected_softmax"``: softmax over the selected logits (lm.py:617, and the server with
    ZONOS3_USE_TRAINING_ROUTER_WEIGHTS=1, zonos3.py:822-827). ``weights="full_softmax"``: the selected entries of the
    softmax over all experts (zonos3.py:821, :765). ``renormalize``: w / (sum(w) + 1e-8) (layer.py:159-161).
    """
    scores = logits.float() - bias.float()
    ids = select_topk(scores, k)
    if weights == "selected_softmax":
        w = logits.float().gather(-1, ids).softmax(-1)
    elif weights == "full_softmax":
        w = torch.softmax(logits.float(), dim=-1).gather(-1, ids)
    else:
        raise ValueError(weights)
    if renormalize:
        w = w / (w.sum(-1, keepdim=True) + 1e-8)
    return ids.to(torch.int32), w


def permutation(ids, num_experts, block=1):
    """Stable counting sort of the flattened (token, slot) pairs by expert (numpy, int64).

    Returns dict(counts [E], offsets [E+1] (padded segment starts), sorted_pairs [offsets[E]] (-1 = padding),
    position [T*k] (row of each pair in the sorted order)).
    """
    flat = np.asarray(ids, dtype=np.int64).reshape(-1)
    counts = np.bincount(flat, minlength=num_experts)[:num_experts]
    padded = (counts + block - 1) // block * block
    offsets = np.zeros(num_experts + 1, dtype=np.int64)
    offsets[1:] = np.cumsum(padded)
    order = np.argsort(flat, kind="stable")
    sorted_pairs = np.full(int(offsets[-1]), -1, dtype=np.int64)
    position = np.empty(flat.size, dtype=np.int64)
    start = 0
    for e in range(num_experts):
        n = int(counts[e])
        seg = order[start:start + n]
        sorted_pairs[offsets[e]:offsets[e] + n] = seg
        position[seg] = offsets[e] + np.arange(n)
        start += n
    return {"counts": counts, "offsets": offsets, "sorted_pairs": sorted_pairs, "position": position}


def experts_fp32(x, gate_up, down, ids, weights):
    """The reference's expert loop in float32 (lm.py:618-639): per (token, rank), gate_up = W13[e] x with the gate
    in the first half, h = SiLU(gate) * up, y = W2[e] h, out += (y * w).to(x.dtype). Vectorised per expert; the
    accumulation over ranks keeps rank order."""
    T, k = ids.shape
    half = gate_up.shape[1] // 2
    terms = torch.zeros(T, k, down.shape[1], dtype=torch.float32, device=x.device)
    for e in torch.unique(ids).tolist():
        tok, rank = torch.nonzero(ids == e, as_tuple=True)
        gu = F.linear(x[tok].float(), gate_up[e].float())
        h = F.silu(gu[:, :half]) * gu[:, half:]
        terms[tok, rank] = F.linear(h, down[e].float()) * weights[tok, rank].float()[:, None]
    out = torch.zeros(T, down.shape[1], dtype=x.dtype, device=x.device)
    for rank in range(k):
        out += terms[:, rank].to(x.dtype)
    return out


def experts_loop_fp32(x, gate_up, down, ids, weights):
    """The reference's expert loop as written (lm.py:622-637): for every token and every rank, gate_up = W13[e] x,
    h = SiLU(first half) * second half, y = W2[e] h, out[token] += (y * w).to(x.dtype). One matrix-vector product
    pair per (token, rank): the CPU path the reference runs, timed as the cfg4 CPU baseline."""
    half = gate_up.shape[1] // 2
    out = torch.zeros(x.shape[0], down.shape[1], dtype=x.dtype)
    for token in range(x.shape[0]):
        for rank in range(ids.shape[1]):
            e = int(ids[token, rank])
            gu = F.linear(x[token], gate_up[e])
            h = F.silu(gu[:half]) * gu[half:]
            out[token] += (F.linear(h, down[e]).float() * weights[token, rank]).to(x.dtype)
    return out


def experts_bf16(x, gate_up, down, ids, weights):
    """The server's bf16 rounding points (fused_moe_impl.py:218-289): GEMM1 output rounded to bf16, SiLU(gate)*up
    rounded (silu_and_mul), GEMM2 output times the routing weight rounded per (token, slot), then the k slots
    summed in float32 and rounded once. GEMM accumulation is float32."""
    T, k = ids.shape
    half = gate_up.shape[1] // 2
    terms = torch.zeros(T, k, down.shape[1], dtype=torch.bfloat16, device=x.device)
    for e in torch.unique(ids).tolist():
        tok, rank = torch.nonzero(ids == e, as_tuple=True)
        gu = F.linear(x[tok].float(), gate_up[e].float()).bfloat16().float()
        h = (F.silu(gu[:, :half]) * gu[:, half:]).bfloat16().float()
        y = F.linear(h, down[e].float()) * weights[tok, rank].float()[:, None]
        terms[tok, rank] = y.bfloat16()
    return terms.float().sum(1).bfloat16()

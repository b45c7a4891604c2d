"""Full AttnRes oracle (CPU): the route over every bank source so far.

Restates ``full_attnres_route`` (model/src/zonos3/reference/lm.py:384-389, identical to
servers/sgl/src/zonos3_sgl/models/zonos3.py:99-113). With bf16 sources its rounding points are the ones the
reference's fused Triton kernel keeps on purpose (training_attnres_kernels.py:1297-1341): the RMS-normalised key
and the key*query product are rounded to the source dtype, logits are summed in float32, the softmax runs in
float32, each weight and each weighted term is rounded to the source dtype, and the terms are summed in float32.

Test infrastructure only (see ``oracle/__init__.py``).
"""

from __future__ import annotations

import torch
import torch.nn.functional as F


def full_attnres_route(sources, query, eps):
    """sources: list of [T, D] tensors (or a [S, T, D] tensor); query [D]. Returns the [T, D] mix."""
    bank = torch.stack(list(sources)) if not isinstance(sources, torch.Tensor) else sources
    keys = F.rms_norm(bank, (bank.shape[-1],), eps=eps)
    logits = (keys * query).sum(-1, dtype=torch.float32)
    weights = logits.softmax(0).to(bank.dtype)
    return (bank * weights.unsqueeze(-1)).sum(0)


def route_weights(sources, query, eps):
    """The [S, T] softmax weights (rounded to the source dtype) of the same route, for diagnostics."""
    bank = torch.stack(list(sources)) if not isinstance(sources, torch.Tensor) else sources
    keys = F.rms_norm(bank, (bank.shape[-1],), eps=eps)
    return (keys * query).sum(-1, dtype=torch.float32).softmax(0).to(bank.dtype)


def weighted_rms_norm(x, weight, eps):
    """RMSNorm with a weight (the attention_norm / ffn_norm / out_norm after each route, lm.py:469-470)."""
    return F.rms_norm(x, (x.shape[-1],), weight=weight, eps=eps)

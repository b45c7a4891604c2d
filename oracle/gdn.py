"""Gated-DeltaNet oracle (CPU, float32): a restatement of ``Zonos3LM._gdn``
(model/src/zonos3/reference/lm.py:556-602) with the head count and head width as parameters (the reference fixes
4 heads of 128, lm.py:28), plus the bare recurrence the CUDA decode / prefill kernels implement.

Test infrastructure only (see ``oracle/__init__.py``).
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

L2_EPS = 1e-6  # q/k normalisation, lm.py:570-571
NORM_EPS = 1e-5  # FLA rms_norm_gated's fixed eps, lm.py:585-586


def recurrent_step(state, q, k, v, g, beta, scale):
    """One token of the gated delta rule, vectorised over leading dims (lm.py:576-582).

    state [..., H, dv, dk] (V-first); q, k [..., H, dk]; v [..., H, dv]; g, beta [..., H] with decay = exp(g).
    Returns (new state, output [..., H, dv]) in float32.
    """
    state, q, k, v = state.float(), q.float(), k.float(), v.float()
    decayed = state * torch.exp(g.float())[..., None, None]
    prediction = (decayed * k[..., None, :]).sum(-1)
    delta = beta.float()[..., None] * (v - prediction)
    updated = decayed + delta[..., :, None] * k[..., None, :]
    output = (updated * (q * scale)[..., None, :]).sum(-1)
    return updated, output


def recurrent_scan(state, q, k, v, g, beta, scale):
    """Tokens along dim 0: q, k [T, ..., H, dk] etc. Returns (final state, outputs [T, ..., H, dv])."""
    outputs = []
    for t in range(q.shape[0]):
        state, o = recurrent_step(state, q[t], k[t], v[t], g[t], beta[t], scale)
        outputs.append(o)
    return state, torch.stack(outputs)


def log_decay(a, A_log, dt_bias):
    """g = -exp(A_log) * softplus(a + dt_bias), the logarithm of the reference's decay (lm.py:572)."""
    return -A_log.float().exp() * F.softplus(a.float() + dt_bias.float())


def l2_normalise(x):
    """x * rsqrt(sum(x^2) + 1e-6) over the last dim, in float32 (lm.py:570-571)."""
    x = x.float()
    return x * torch.rsqrt(x.square().sum(-1, keepdim=True) + L2_EPS)


def causal_conv_silu(qkv, history, weight):
    """Depthwise causal conv + SiLU over rows of ``qkv`` [N, C] continuing ``history`` [C, K-1]
    (lm.py:563-568; weight [C, 1, K], weight[..., 0] multiplies the oldest row).
    Returns (activations [N, C] in qkv's dtype, new history [C, K-1])."""
    channels, width = weight.shape[0], weight.shape[-1]
    sequence = torch.cat((history, qkv.T), -1)
    conv = F.conv1d(sequence.unsqueeze(0), weight, groups=channels).squeeze(0).T
    return F.silu(conv), sequence[:, -(width - 1):].clone()


def gated_rms_norm(o, z, weight):
    """Per-head RMSNorm(o; weight, eps 1e-5) * SiLU(z), rounded to o's dtype (lm.py:585-587).
    o [N, H, dv] in the activation dtype; z [N, H*dv]."""
    normalized = F.rms_norm(o, (o.shape[-1],), weight=weight, eps=NORM_EPS)
    n, heads, width = o.shape
    return (normalized.float() * F.silu(z.reshape(n, heads, width).float())).to(o.dtype).reshape(n, heads * width)


def gdn_layer(x, weights, conv_state=None, state=None, *, heads, head_dim, capture=None):
    """The GDN mixer over rows ``x`` [N, D] of ONE sequence continuing (conv_state, state).

    ``weights`` holds the checkpoint names of one layer's ``attention.*`` (lm.py:270-279): ``in_proj.weight``
    [4*inner + 2*heads, D], ``conv.weight`` [3*inner, 1, K], ``out_weight`` [head_dim], ``A_log`` [heads],
    ``dt_bias`` [heads], ``wo.weight`` [D, inner]. Returns (y [N, D], conv_state [3*inner, K-1], state
    [heads, head_dim, head_dim] float32). ``capture`` receives the intermediates under the reference's names.
    """
    inner = heads * head_dim
    channels = 3 * inner
    width = weights["conv.weight"].shape[-1]
    projection = F.linear(x, weights["in_proj.weight"])
    qkv, z, a, b = projection.split((channels, inner, heads, heads), -1)
    if conv_state is None:
        conv_state = torch.zeros(channels, width - 1, dtype=x.dtype)
    conv, conv_state = causal_conv_silu(qkv, conv_state, weights["conv.weight"])
    q, k, v = (part.reshape(len(x), heads, head_dim).float() for part in conv.split(inner, -1))
    q, k = l2_normalise(q), l2_normalise(k)
    g = log_decay(a, weights["A_log"], weights["dt_bias"])
    beta = b.float().sigmoid()
    if state is None:
        state = torch.zeros(heads, head_dim, head_dim, dtype=torch.float32)
    state, outputs = recurrent_scan(state, q, k, v, g, beta, head_dim ** -0.5)
    recurrent = outputs.to(x.dtype)
    gated = gated_rms_norm(recurrent, z, weights["out_weight"])
    if capture is not None:
        capture.update(gdn_conv=conv, gdn_q=q, gdn_k=k, gdn_v=v, gdn_decay=torch.exp(g), gdn_beta=beta,
                       gdn_recurrent=recurrent, gdn_gated=gated, gdn_state=state, gdn_conv_state=conv_state)
    return F.linear(gated, weights["wo.weight"]), conv_state, state

"""The decode step's dense projections on tcgen05 (``zb_proj_gemm``) and the DeltaNet in_proj GEMM fused with its
decode prologue (``zb_gdn_in_proj_decode``).

proj_gemm against the fp32 product x.float() @ w.float().T (TF32 off) over the tilings (column tile 64 / 128 / 256,
1 to 4 K slices), ragged token counts (1, 37, 256, 300: one and two 256-token tiles) and a column count that is not a
multiple of the tile; bar: every element within one bf16 rounding of the fp32 product (2^-8 relative) plus 1e-5 of
the output's largest magnitude for the fp32 summation order. Split-K runs are checked to leave the workspace's ticket
counters at zero and to repeat bit for bit.

The fused in_proj + prologue against the unfused kernels on the same bf16 mixed rows, computed here as the fp32
product rounded once to bf16 (what the fused epilogue rounds): q / k / v, z, g, beta and the shifted conv history;
padding slots (-1) must leave the history untouched. A product whose fp32 sum order differs can round across a bf16
boundary, and the conv then sees a one-step different input, so the bars are: >= 99 % of q / k / v elements and of
the history bit-identical; q / k / v within 1 % of their head's largest magnitude; z and the history (rounded
products themselves) within one bf16 step; >= 99.5 % of g / beta within 1e-5 relative and all within 5 % (an a / b
input one bf16 step apart). Reference: OriginalGDN in_proj + _run_packed prologue
(servers/sgl/src/zonos3_sgl/models/gdn.py:399-434).
"""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


def _ref(x, w):
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        return x.float() @ w.float().t()
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


def _check_close(got, ref, rel=2.0 ** -8):
    """Within `rel` of |ref| (2^-8: one bf16 rounding of an fp32 value; 2^-7: two bf16 roundings of fp32 values
    that differ only in summation order) plus 1e-5 of the largest |ref| for that order."""
    err = (got.float() - ref).abs()
    bar = ref.abs() * rel + 1e-5 * ref.abs().max()
    assert bool((err <= bar).all()), f"max excess {(err - bar).max().item():.3e}"


@pytest.mark.parametrize("T,K,N,block_n,splits", [
    (256, 2048, 2048, 64, 2), (256, 2048, 2048, 128, 1), (256, 2048, 2048, 256, 4), (256, 1024, 3088, 0, 0),
    (37, 512, 1000, 256, 1), (1, 384, 520, 64, 3), (300, 512, 2056, 128, 2), (256, 512, 40984, 0, 0),
])
def test_proj_gemm_matches_fp32(zb, T, K, N, block_n, splits):
    gen = torch.Generator(device="cuda").manual_seed(T * 7 + N)
    x = torch.randn(T, K, device="cuda", generator=gen).bfloat16()
    w = (torch.randn(N, K, device="cuda", generator=gen) * K ** -0.5).bfloat16()
    y = zb.ops.proj_gemm(x, w, block_n=block_n, splits=splits)
    torch.cuda.synchronize()
    _check_close(y, _ref(x, w))
    y2 = zb.ops.proj_gemm(x, w, block_n=block_n, splits=splits)
    torch.cuda.synchronize()
    assert torch.equal(y, y2), "split-K partials must be summed in a fixed order"
    if block_n and splits > 1:  # the workspace starts with one ticket counter per (token tile, column tile, CTA)
        ws = zb.ops._PROJ_WS[torch.device("cuda", torch.cuda.current_device())]
        tickets = ((T + 255) // 256) * ((N + block_n - 1) // block_n) * 2
        assert int(ws[:4 * tickets].view(torch.int32).abs().sum().item()) == 0, "ticket counters must return to zero"


def test_proj_gemm_row_strides(zb):
    """x and out as column slices of wider buffers (row strides > K, N)."""
    T, K, N = 64, 256, 384
    gen = torch.Generator(device="cuda").manual_seed(3)
    xb = torch.randn(T, K + 64, device="cuda", generator=gen).bfloat16()
    w = (torch.randn(N, K, device="cuda", generator=gen) * K ** -0.5).bfloat16()
    ob = torch.full((T, N + 16), 7.0, device="cuda", dtype=torch.bfloat16)
    zb.ops.proj_gemm(xb[:, :K], w, out=ob[:, :N])
    torch.cuda.synchronize()
    _check_close(ob[:, :N], _ref(xb[:, :K], w))
    assert bool((ob[:, N:] == 7.0).all()), "columns past N must not be written"


def test_proj_gemm_rejects_bad_shapes(zb):
    x = torch.zeros(4, 100, device="cuda", dtype=torch.bfloat16)
    w = torch.zeros(64, 100, device="cuda", dtype=torch.bfloat16)
    with pytest.raises((ValueError, RuntimeError)):
        zb.ops.proj_gemm(x, w)  # K not a multiple of 128


@pytest.mark.parametrize("T,K,H,D,splits", [(256, 2048, 16, 128, 1), (256, 2048, 16, 128, 2), (37, 512, 4, 64, 0),
                                            (300, 256, 4, 128, 2)])
def test_gdn_in_proj_decode_matches_unfused(zb, T, K, H, D, splits):
    ops = zb.ops
    inner = H * D
    N = 4 * inner + 2 * H
    dev = torch.device("cuda")
    gen = torch.Generator(device="cuda").manual_seed(T + H)
    x = torch.randn(T, K, device=dev, generator=gen).bfloat16()
    w = (torch.randn(N, K, device=dev, generator=gen) * K ** -0.5).bfloat16()
    conv_w = (torch.randn(3 * inner, 1, 4, device=dev, generator=gen) * 0.5).bfloat16()
    A_log = torch.randn(H, device=dev, generator=gen) * 0.5
    dt_bias = torch.randn(H, device=dev, generator=gen) * 0.5
    rows = T + 8
    conv0 = torch.randn(rows, 3 * inner, 3, device=dev, generator=gen).bfloat16()
    slots = torch.randperm(rows, device=dev, generator=gen)[:T].to(torch.int64)
    slots[::5] = -1  # padding rows
    # unfused: the bf16 mixed rows the fused epilogue rounds, then the decode prologue kernel
    mixed = _ref(x, w).bfloat16()
    conv_ref = conv0.clone()
    q0, k0, v0, g0, b0 = ops.gdn_prologue_decode(mixed, conv_w, A_log, dt_bias, slots, conv_ref, heads=H, head_dim=D)
    conv_got = conv0.clone()
    q, k, v, z, g, beta = ops.gdn_in_proj_decode(x, w, conv_w, A_log, dt_bias, slots, conv_got, heads=H, head_dim=D,
                                                 splits=splits)
    torch.cuda.synchronize()
    for name, got, ref in (("q", q, q0), ("k", k, k0), ("v", v, v0)):
        same = (got == ref).float().mean().item()
        assert same >= 0.99, f"{name}: only {same:.4f} bit-identical"
        head_max = ref.float().abs().amax(dim=-1, keepdim=True).clamp(min=1e-6)
        assert ((got.float() - ref.float()).abs() / head_max).max().item() <= 1e-2, name
    same = (conv_got == conv_ref).float().mean().item()
    assert same >= 0.99, f"conv_state: only {same:.4f} bit-identical"
    _check_close(conv_got, conv_ref.float(), rel=2.0 ** -7)
    _check_close(z, mixed[:, 3 * inner:4 * inner].float(), rel=2.0 ** -7)
    for name, got, ref in (("g", g, g0), ("beta", beta, b0)):
        rel = (got - ref).abs() / ref.abs().clamp(min=1e-6)
        assert (rel <= 1e-5).float().mean().item() >= 0.995, name
        assert rel.max().item() <= 0.05, name  # an a / b input one bf16 step apart (up to 0.03 at |a| ~ 4)
    untouched = torch.ones(rows, dtype=torch.bool, device=dev)
    untouched[slots[slots >= 0]] = False
    assert torch.equal(conv_got[untouched], conv0[untouched]), "rows no token owns must not change"

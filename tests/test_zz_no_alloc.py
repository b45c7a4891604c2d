"""The allocation-free MoE down projection + combine (zb_moe_down_combine_noalloc), called through the C ABI.

Some callers of these kernels cannot call cudaMalloc: a serving runtime that reserves its device memory at
start-up and forbids allocation afterwards, or a C / Go / Java binding that has no device allocator and only
passes the tensors it owns. This entry point serves them by keeping its intermediate rows in a static 8 MiB
device array instead of a caller buffer. The test checks it against the allocating pair of entry points
(zb_moe_gemm_down + zb_moe_combine) on two calls in a row (the second with different routing, so rows left from
the first call must not leak in), and that a call beyond the array's size is refused.

The file is named to be collected last, so a run that stops at the first failure has run every other test."""

from __future__ import annotations

import ctypes

import pytest
import torch

from conftest import rel_err

pytestmark = pytest.mark.gpu

TOL = 2e-2
SCRATCH_ELEMS = 4 << 20


def _case(zb, T, k, E, D, I, seed):
    gen = torch.Generator().manual_seed(seed)
    dev = torch.device("cuda")
    ids = torch.stack([torch.randperm(E, generator=gen)[:k] for _ in range(T)]).int().to(dev)
    w = torch.softmax(torch.randn(T, k, generator=gen), -1).to(dev)
    x = torch.randn(T, D, generator=gen).bfloat16().to(dev)
    gate_up = (0.02 * torch.randn(E, 2 * I, D, generator=gen)).bfloat16().to(dev)
    down = (0.02 * torch.randn(E, D, I, generator=gen)).bfloat16().to(dev)
    ws = zb.ops.MoEWorkspace(T, k, E, D, I, dev)
    perm = zb.ops.moe_permute(ids, E, capacity=ws.capacity, out=ws.perm)
    zb.ops.moe_gather(x, perm["sorted_pairs"], k, ws.x_perm)
    zb.ops.moe_gemm_swiglu(ws.x_perm, gate_up, perm["offsets"], ws.h)
    return ws, down, w


def _noalloc(zb, ws, down, w, T, k, out):
    E, D, I = down.shape
    lib = zb._lib.load()
    return lib.zb_moe_down_combine_noalloc(
        ws.h.data_ptr(), ws.capacity, down.data_ptr(), E, D, I, ws.perm["offsets"].data_ptr(),
        ws.perm["sorted_pairs"].data_ptr(), w.data_ptr(), T, k, out.data_ptr(), out.stride(0),
        torch.cuda.current_stream().cuda_stream)


def test_noalloc_matches_the_allocating_entry_points_twice(zb):
    for T, k, E, D, I, seed in ((96, 8, 64, 2048, 768, 1), (40, 4, 16, 1024, 256, 2)):
        ws, down, w = _case(zb, T, k, E, D, I, seed)
        ref = torch.empty(T, D, device="cuda", dtype=torch.bfloat16)
        zb.ops.moe_gemm_down(ws.h, down, ws.perm["offsets"], ws.perm["sorted_pairs"], w, ws.y)
        zb.ops.moe_combine(ws.y, k, ref)
        out = torch.full((T, D), 3.0, device="cuda", dtype=torch.bfloat16)
        status = _noalloc(zb, ws, down, w, T, k, out)
        assert status == 0, zb._lib.last_error()
        torch.cuda.synchronize()
        assert rel_err(out.float(), ref.float()) < TOL


def test_noalloc_refuses_sizes_beyond_its_scratch(zb):
    ws, down, w = _case(zb, 8, 2, 8, 256, 128, 3)
    E, D, I = down.shape
    T, k = SCRATCH_ELEMS // (2 * D) + 1, 2  # one token more than the array holds
    out = torch.empty(1, D, device="cuda", dtype=torch.bfloat16)
    lib = zb._lib.load()
    status = lib.zb_moe_down_combine_noalloc(
        ws.h.data_ptr(), ws.capacity, down.data_ptr(), E, D, I, ws.perm["offsets"].data_ptr(),
        ws.perm["sorted_pairs"].data_ptr(), w.data_ptr(), T, k, out.data_ptr(), D,
        torch.cuda.current_stream().cuda_stream)
    assert status == 3 and "static scratch" in zb._lib.last_error()

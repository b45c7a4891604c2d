"""The allocation-free MoE down projection + combine (zb_moe_down_combine_noalloc), called through the C ABI.

Some callers of these kernels cannot call cudaMalloc: a serving runtime that reserves its device memory at
start-up and forbids allocation afterwards, or a C / Go / Java binding that has no device allocator and only
passes the tensors it owns. This entry point serves them by keeping its intermediate rows in a static 8 MiB
device array instead of a caller buffer. The test checks it against the allocating pair of entry points
(zb_moe_gemm_down + zb_moe_combine, their buffer zero-filled) and against the oracle's expert loop with the
server's rounding points, on two calls in a row. The second call routes fewer tokens and gives some (token, slot)
pairs an invalid expert id: the permutation skips those pairs, so their rows are written by no GEMM, and only the
clearing of the array keeps the first call's rows out of the result. A call beyond the array's size is refused.

The file is named to be collected last, so a run that stops at the first failure has run every other test."""

from __future__ import annotations

import pytest
import torch

from conftest import rel_err
from oracle import moe as omoe

pytestmark = pytest.mark.gpu

TOL = 2e-2
SCRATCH_ELEMS = 4 << 20


def _case(zb, T, k, E, D, I, seed, invalid=0):
    """Routed inputs of the down projection: ids (the first ``invalid`` tokens get ids -1 and E in two slots),
    weights, x, weights of the experts, and the permutation / gather / GEMM1 results in a workspace."""
    gen = torch.Generator().manual_seed(seed)
    dev = torch.device("cuda")
    ids = torch.stack([torch.randperm(E, generator=gen)[:k] for _ in range(T)]).int()
    ids[:invalid, 0] = -1
    ids[:invalid, k - 1] = E
    w = torch.softmax(torch.randn(T, k, generator=gen), -1)
    x = torch.randn(T, D, generator=gen).bfloat16()
    gate_up = (0.02 * torch.randn(E, 2 * I, D, generator=gen)).bfloat16()
    down = (0.02 * torch.randn(E, D, I, generator=gen)).bfloat16()
    ws = zb.ops.MoEWorkspace(T, k, E, D, I, dev)
    perm = zb.ops.moe_permute(ids.to(dev), E, capacity=ws.capacity, out=ws.perm)
    zb.ops.moe_gather(x.to(dev), perm["sorted_pairs"], k, ws.x_perm)
    zb.ops.moe_gemm_swiglu(ws.x_perm, gate_up.to(dev), perm["offsets"], ws.h, counts=perm["counts"])
    return ws, dict(ids=ids, w=w, x=x, gate_up=gate_up, down=down)


def _noalloc(zb, ws, down, w, T, k, out, counts=True):
    E, D, I = down.shape
    lib = zb._lib.load()
    return lib.zb_moe_down_combine_noalloc(
        ws.h.data_ptr(), ws.capacity, down.data_ptr(), E, D, I, ws.perm["offsets"].data_ptr(),
        ws.perm["counts"].data_ptr() if counts else None, ws.perm["sorted_pairs"].data_ptr(), w.data_ptr(), T, k,
        out.data_ptr(), out.stride(0), torch.cuda.current_stream().cuda_stream)


def _oracle(case, E):
    """The oracle's expert loop with the server's rounding points (oracle/moe.experts_bf16); a pair with an
    invalid expert id contributes zero."""
    ids, w = case["ids"].long(), case["w"]
    valid = (ids >= 0) & (ids < E)
    return omoe.experts_bf16(case["x"], case["gate_up"], case["down"], ids.clamp(0, E - 1), w * valid)


def test_noalloc_matches_the_allocating_entry_points_twice(zb):
    dev = torch.device("cuda")
    # the second call routes fewer tokens, some through invalid ids: its cleared rows must not keep the first's
    for T, k, E, D, I, seed, invalid, counts in ((96, 8, 64, 2048, 768, 1, 0, True),
                                                 (40, 4, 16, 1024, 256, 2, 9, False)):
        ws, case = _case(zb, T, k, E, D, I, seed, invalid)
        down, w = case["down"].to(dev), case["w"].to(dev)
        ref = torch.empty(T, D, device=dev, dtype=torch.bfloat16)
        ws.y.zero_()
        zb.ops.moe_gemm_down(ws.h, down, ws.perm["offsets"], ws.perm["sorted_pairs"], w, ws.y,
                             counts=ws.perm["counts"])
        zb.ops.moe_combine(ws.y, k, ref)
        out = torch.full((T, D), 3.0, device=dev, dtype=torch.bfloat16)
        status = _noalloc(zb, ws, down, w, T, k, out, counts)
        assert status == 0, zb._lib.last_error()
        torch.cuda.synchronize()
        assert rel_err(out.float(), ref.float()) < TOL
        oracle = _oracle(case, E)
        assert rel_err(out.float().cpu(), oracle.float()) < TOL
        if invalid:
            # tokens with invalid slots sum only their valid slots, exactly as the allocating pair does
            assert torch.equal(out[:invalid], ref[:invalid])


def test_noalloc_refuses_sizes_beyond_its_scratch(zb):
    ws, case = _case(zb, 8, 2, 8, 256, 128, 3)
    down, w = case["down"].cuda(), case["w"].cuda()
    E, D, I = down.shape
    T, k = SCRATCH_ELEMS // (2 * D) + 1, 2  # one token more than the array holds
    out = torch.empty(1, D, device="cuda", dtype=torch.bfloat16)
    lib = zb._lib.load()
    status = lib.zb_moe_down_combine_noalloc(
        ws.h.data_ptr(), ws.capacity, down.data_ptr(), E, D, I, ws.perm["offsets"].data_ptr(), None,
        ws.perm["sorted_pairs"].data_ptr(), w.data_ptr(), T, k, out.data_ptr(), D,
        torch.cuda.current_stream().cuda_stream)
    assert status == 3 and "static scratch" in zb._lib.last_error()

"""The C-ABI library loads on a machine without a GPU, exports every entry point ``include/zonos3_b200.h``
declares, and rejects bad arguments before touching the device (no compute call is made here)."""

from __future__ import annotations

import ctypes
import re

import pytest

from conftest import ROOT

HEADER = ROOT / "include" / "zonos3_b200.h"


def declared_symbols() -> list[str]:
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(zb_\w+)\s*\(", text)))


def test_header_declares_the_abi():
    names = declared_symbols()
    assert "zb_last_error" in names and "zb_gdn_decode_step" in names


def test_library_exports_every_declared_symbol(zb):
    lib = zb._lib.load()
    missing = [n for n in declared_symbols() if not hasattr(lib, n)]
    assert not missing, f"library lacks {missing}"
    assert set(declared_symbols()) <= set(zb._lib.SIGNATURES), "every declared symbol has a ctypes signature"


def test_invalid_arguments_are_rejected_before_launch(zb):
    lib = zb._lib.load()
    fake = ctypes.c_void_p(256)  # never dereferenced: the checks fail first
    # unsupported head width -> status 3
    status = lib.zb_gdn_decode_step(fake, fake, fake, 0, 0, 0, fake, fake, 0, fake, None, 1, fake, 0,
                                    1, 1, 96, 96, 1.0, None)
    assert status == 3 and "dk=96" in zb._lib.last_error()
    # misaligned state -> status 1
    status = lib.zb_gdn_decode_step(fake, fake, fake, 128, 128, 128, fake, fake, 1, ctypes.c_void_p(260), None, 1,
                                    fake, 128, 1, 1, 128, 128, 1.0, None)
    assert status == 1 and "aligned" in zb._lib.last_error()
    # vocoder tail: an even mixer, a ring that is not a power of two, a push with no frames -> status 1
    P, N = fake, None
    head = [P, 0, P, 0, 0, 1, 4, 736, 2208, 184, P, P, P, P, 4.6, P]
    state = [P, P, 0, P, P]
    status = lib.zb_istft_head_push(*head, 126, *state, 4096, 0, 0, 0, 0, P, 1 << 20, P, N)
    assert status == 1 and "odd" in zb._lib.last_error()
    status = lib.zb_istft_head_push(*head, 127, *state, 4000, 0, 0, 0, 0, P, 1 << 20, P, N)
    assert status == 1 and "power of two" in zb._lib.last_error()
    status = lib.zb_istft_head_push(*[h if i != 6 else 0 for i, h in enumerate(head)], 127, *state, 4096, 0, 0, 0, 0,
                                    P, 1 << 20, P, N)
    assert status == 1 and "push at least one" in zb._lib.last_error()
    status = lib.zb_resample_push(P, 0, 10, 1, 10, P, 1024, 0, P, 736, 735, 17, 0, 1, 736, P, N, 0, N)
    assert status == 1 and "blocks" in zb._lib.last_error()  # more outputs than one block holds
    with pytest.raises(ValueError):
        zb._lib.check(1, "probe")
    with pytest.raises(RuntimeError):
        zb._lib.check(2, "probe")


def test_vocoder_streams_refuse_cpu_devices(zb):
    with pytest.raises(ValueError, match="CUDA"):
        zb.vocoder.IstftHeadStream((736, 2208), 184, [[0.0] * 736, [0.0] * 2208], [[1.0], [0.0]], 4.6, "cpu")
    with pytest.raises(ValueError, match="CUDA"):
        zb.vocoder.ResamplerStream([[1.0]], 1, 1, 0, "cpu")


def test_ops_refuse_cpu_tensors(zb):
    import torch

    q = torch.zeros(1, 1, 128, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA"):
        zb.ops.gdn_decode_step(q, q, q, torch.zeros(1, 1), torch.zeros(1, 1), torch.zeros(1, 1, 128, 128))

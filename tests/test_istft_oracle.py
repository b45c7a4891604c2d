"""The vocoder DSP-tail oracle against the reference's golden stream outputs (tests/golden/istft_stream.npz, made by
tests/golden/make_istft_golden.py from model/src/zonos3/codec/stream_host.py) and torchaudio's resampling kernel."""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

from oracle import istft

GOLDEN = Path(__file__).resolve().parent / "golden" / "istft_stream.npz"


@pytest.fixture(scope="module")
def golden():
    return dict(np.load(GOLDEN))


def f32_close(got, want):
    """Float32 outputs of a float64 computation summed in another order: within 4 float32 ulps of the signal's peak
    (the reference's host and device streams agree to the same float32 rounding)."""
    got, want = np.asarray(got, np.float64), np.asarray(want, np.float64)
    assert got.shape == want.shape
    if want.size == 0:
        return
    bar = 4 * np.spacing(np.float32(np.abs(want).max()))
    err = np.abs(got - want).max()
    assert err <= bar, f"max error {err:.3g} above {bar:.3g}"


def test_kernel_restatement_matches_torchaudio(golden):
    kernel, width, orig, new = istft.sinc_resample_kernel(44160, 44100, 16, 0.99)
    assert (orig, new, width) == tuple(golden["resampler"])
    assert kernel.shape == (735, 2 * 17 + 736) and kernel.dtype == np.float32
    rows = kernel[golden["ta_row_index"]]
    np.testing.assert_allclose(rows, golden["ta_rows"], rtol=0, atol=2 * np.spacing(np.float32(1)))
    np.testing.assert_allclose(kernel.astype(np.float64).sum(1), golden["ta_row_sums"], rtol=0, atol=1e-6)


def test_stream_outputs_match_the_reference(golden):
    chunks = golden["chunks"]
    n = len(chunks)
    kernel, width, orig, new = istft.sinc_resample_kernel(44160, 44100, 16, 0.99)
    head, res = istft.stream_outputs(
        [golden[f"y0_{c}"] for c in range(n)], [golden[f"y1_{c}"] for c in range(n)], (736, 2208), 184,
        [golden["window0"], golden["window1"]], golden["mixer"], float(golden["max_log_mag"]), kernel, orig, new,
        width)
    for c in range(n):
        f32_close(head[c], golden[f"head_{c}"])
        f32_close(res[c], golden[f"res_{c}"])
    f32_close(head[n], golden["head_flush"])
    f32_close(res[n], golden["res_flush"])


def test_emission_schedule():
    """Emission bounds: nothing until the longest branch's centre padding and the mixer's right taps are final."""
    assert istft.istft_emitted(6, (736, 2208), 184, 127) == 0
    assert istft.istft_emitted(10, (736, 2208), 184, 127) == 10 * 184 - 1104 - 63
    assert istft.istft_emitted(10, (736, 2208), 184, 127, flushed=True) == 1840
    assert istft.istft_emitted(0, (736, 2208), 184, 127, flushed=True) == 0
    assert istft.resample_emitted(752, 736, 735, 17, 770) == 0
    assert istft.resample_emitted(753, 736, 735, 17, 770) == 735
    assert istft.resample_emitted(1840, 736, 735, 17, 770, flushed=True) == -(-735 * 1840 // 736)

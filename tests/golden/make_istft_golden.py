"""Golden vectors of the codec's streaming iSTFT head + resampler (tests/golden/istft_stream.npz), from the
reference's own NumPy streams (model/src/zonos3/codec/stream_host.py: IstftHeadStream, ResamplerStream) imported from
the reference checkout, and torchaudio's resampling kernel. Run from the repository root with the reference's
`model/src` on the path:

    PYTHONPATH=<reference>/model/src python tests/golden/make_istft_golden.py

Configuration: the MR-iSTFT head's two branches (n_fft 736 and 2208, hop 184, periodic Hann windows in float32 as the
model registers them, a 127-tap FIR mixer over the two branches, log-magnitude clamp ln 100) and the 44160 -> 44100 Hz
resampler (torchaudio `Resample(44160, 44100, lowpass_filter_width=16, rolloff=0.99)`: 736 -> 735 phases, width 17).
Inputs are seeded: log-magnitudes N(-3, 1.5) (a few above the clamp), phases U(-pi, pi), a mixer of N(0, 0.05) plus a
unit centre tap on branch 0, all float32. Chunks of 3, 1, 0, 2, 4 and 8 head frames are pushed (the empty push returns
nothing), then the streams are flushed; every call's output is recorded, the iSTFT output going through the resampler
as the codec does (model/src/zonos3/codec/istft_head_a_20261002/stream.py:205-215).

The streams run with the resampling kernel of `oracle.istft.sinc_resample_kernel`, so the vectors are reproducible from
the stored inputs; a few rows of torchaudio's own kernel (and each row's sum) are stored to pin that restatement."""

from __future__ import annotations

import math
import sys
from pathlib import Path

import numpy as np
import torch
import torchaudio
from zonos3.codec.stream_host import IstftHeadStream, ResamplerStream

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
from oracle.istft import sinc_resample_kernel  # noqa: E402

N_FFTS, HOP, TAPS = (736, 2208), 184, 127
CHUNKS = (3, 1, 0, 2, 4, 8)
KERNEL_ROWS = (0, 1, 2, 367, 733, 734)


def main() -> None:
    rng = np.random.default_rng(2026)
    windows = [torch.hann_window(n, periodic=True).numpy() for n in N_FFTS]
    mixer = rng.normal(0, 0.05, (2, TAPS)).astype(np.float32)
    mixer[0, TAPS // 2] += 1.0
    ta = torchaudio.transforms.Resample(44160, 44100, lowpass_filter_width=16, rolloff=0.99)
    ta_kernel = ta.kernel[:, 0].numpy()
    kernel, width, orig, new = sinc_resample_kernel(44160, 44100, 16, 0.99)
    assert (width, orig, new) == (ta.width, 736, 735) and kernel.shape == ta_kernel.shape
    head = IstftHeadStream(N_FFTS, HOP, windows, mixer, math.log(100.0))
    res = ResamplerStream(kernel, orig, new, width)
    arrays = {"window0": windows[0], "window1": windows[1], "mixer": mixer, "chunks": np.array(CHUNKS),
              "max_log_mag": np.float64(math.log(100.0)), "resampler": np.array([orig, new, width]),
              "ta_rows": ta_kernel[list(KERNEL_ROWS)], "ta_row_index": np.array(KERNEL_ROWS),
              "ta_row_sums": ta_kernel.astype(np.float64).sum(1)}
    for c, cols in enumerate(CHUNKS):
        for i, n in enumerate(N_FFTS):
            bins = n // 2 + 1
            y = np.concatenate([rng.normal(-3.0, 1.5, (cols, bins)), rng.uniform(-np.pi, np.pi, (cols, bins))], 1)
            arrays[f"y{i}_{c}"] = y.astype(np.float32)
        out = head.push(arrays[f"y0_{c}"], arrays[f"y1_{c}"])
        arrays[f"head_{c}"] = out
        arrays[f"res_{c}"] = res.push(out)
    tail = head.flush()
    arrays["head_flush"] = tail
    arrays["res_flush"] = np.concatenate([res.push(tail), res.flush()])
    path = Path(__file__).resolve().parent / "istft_stream.npz"
    np.savez_compressed(path, **arrays)
    print(path, {k: v.shape for k, v in arrays.items() if k.startswith(("head", "res_"))})


if __name__ == "__main__":
    main()

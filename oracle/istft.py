"""Vocoder DSP-tail oracle (CPU, float64 NumPy): the codec's streaming two-branch iSTFT head with its FIR mixer, and the
44160 -> 44100 Hz sinc resampler behind it (model/src/zonos3/codec/stream_host.py, IstftHeadStream :16-127 and
ResamplerStream :122-171; their torch twins in stream_device.py follow the same steps).

Restated as whole-signal decodes plus the streams' emission schedules rather than incremental buffers: a stream that
has been fed F head frames has emitted exactly the first ``istft_emitted(F)`` samples of the whole-signal decode of
those frames, and the resampler likewise. Sums run in another order than the reference's running buffers, so the
outputs agree with it to float32 rounding (the reference's own device twin makes the same statement of itself).
Test infrastructure only (see ``oracle/__init__.py``).
"""

from __future__ import annotations

import math

import numpy as np


def branch_frames(y, n: int, window, max_log_mag: float) -> np.ndarray:
    """Head frames y [cols, n + 2] (log-magnitude for n//2 + 1 bins, then phase) -> windowed real frames [cols, n].

    The magnitude is exp(min(log-magnitude, max_log_mag)); the imaginary parts of the DC and Nyquist bins are zeroed;
    frames are the inverse real DFT of length n (1/n scaling) times the window (stream_host.py:55-63)."""
    y = np.asarray(y, np.float64)
    bins = n // 2 + 1
    mag = np.exp(np.minimum(y[:, :bins], max_log_mag))
    spec = mag * np.cos(y[:, bins:]) + 1j * (mag * np.sin(y[:, bins:]))
    spec[:, 0] = spec[:, 0].real
    spec[:, -1] = spec[:, -1].real
    return np.fft.irfft(spec, n, axis=-1) * np.asarray(window, np.float64)


def branch_signal(y, n: int, hop: int, window, max_log_mag: float) -> np.ndarray:
    """The centred iSTFT of one branch: frames overlap-added every hop samples, divided by the overlap-added squared
    window, with the first n//2 samples (the centre padding) dropped -> [(cols - 1) * hop + n - n//2]
    (stream_host.py:64-79 and the finalize step :104-113)."""
    frames = branch_frames(y, n, window, max_log_mag)
    cols = frames.shape[0]
    span = (cols - 1) * hop + n
    ola = np.zeros(span)
    env = np.zeros(span)
    w2 = np.asarray(window, np.float64) ** 2
    for c in range(cols):
        ola[c * hop: c * hop + n] += frames[c]
        env[c * hop: c * hop + n] += w2
    return ola[n // 2:] / env[n // 2:]


def mixer_output(signals, mixer, total: int) -> np.ndarray:
    """The FIR mixer over the two branch signals: y[m] = sum_c sum_k mixer[c][k] * s_c[m + k - h] for m < total,
    h = (K - 1) // 2, with zeros outside each signal's [0, total) (the h leading zeros of the mixer input and the
    zeros appended at flush, stream_host.py:31, :95-100 and :115-127)."""
    mixer = np.asarray(mixer, np.float64)
    K = mixer.shape[1]
    h = (K - 1) // 2
    y = np.zeros(total)
    for c, s in enumerate(signals):
        padded = np.zeros(total + 2 * h)
        take = min(total, len(s))
        padded[h: h + take] = s[:take]
        y += np.correlate(padded, mixer[c], "valid")[:total]
    return y


def istft_emitted(frames: int, n_ffts, hop: int, K: int, flushed: bool = False) -> int:
    """Samples a head stream has emitted after `frames` head frames: every mixer output whose taps are final,
    i.e. frames * hop - max(n // 2) - (K - 1) // 2 (from the finalize and mix-emit bounds, stream_host.py:81-83 and
    :117-121), or all frames * hop once flushed (:88-101)."""
    if flushed:
        return frames * hop if frames else 0
    return max(0, frames * hop - max(n // 2 for n in n_ffts) - (K - 1) // 2)


def istft_decode(ys0, ys1, n_ffts, hop: int, windows, mixer, max_log_mag: float) -> np.ndarray:
    """Whole-signal decode of F head frames (both branches [F, n_i + 2]) -> float64 [F * hop]."""
    frames = np.asarray(ys0).shape[0]
    sigs = [branch_signal(y, n, hop, w, max_log_mag) for y, n, w in zip((ys0, ys1), n_ffts, windows)]
    return mixer_output(sigs, mixer, frames * hop)


def resample(x, kernel, orig: int, new: int, width: int, count: int) -> np.ndarray:
    """The first `count` outputs of the polyphase sinc resampler: out[b * new + i] = sum_k kernel[i][k] *
    x[b * orig + k - width], x zero outside [0, len(x)) (stream_host.py:122-171)."""
    kernel = np.asarray(kernel, np.float64)
    x = np.asarray(x, np.float64)
    kl = kernel.shape[1]
    blocks = -(-count // new)
    lo = -width
    hi = (blocks - 1) * orig - width + kl
    seg = np.zeros(max(0, hi - lo))
    a, b = max(lo, 0), min(hi, len(x))
    if b > a:
        seg[a - lo: b - lo] = x[a:b]
    out = np.array([kernel @ seg[blk * orig: blk * orig + kl] for blk in range(blocks)]).reshape(-1)
    return out[:count]


def resample_emitted(n_in: int, orig: int, new: int, width: int, kl: int, flushed: bool = False) -> int:
    """Samples a resampler stream has emitted after n_in input samples: whole blocks whose window lies inside the
    input (stream_host.py:150-152), or ceil(new * n_in / orig) once flushed (:147-149)."""
    if flushed:
        return -(-new * n_in // orig)
    reach = n_in + width - kl
    return (reach // orig + 1) * new if reach >= 0 else 0


def sinc_resample_kernel(orig_freq: int, new_freq: int, lowpass_filter_width: int = 16, rolloff: float = 0.99):
    """The Hann-windowed sinc kernel of torchaudio's `Resample` (torchaudio 2.11, `_get_sinc_resample_kernel` with
    resampling_method "sinc_interp_hann" and the default float32 output), as the codec builds it for
    44160 -> 44100 Hz with lowpass_filter_width 16 and rolloff 0.99 (model/src/zonos3/codec/hybrid10_dual_encoding/
    base_model.py:209) and hands to the stream (istft_head_a_20261002/stream.py:183-185).

    Returns (kernel float32 [new, 2 * width + orig], width, orig, new) for the gcd-reduced rates. The published steps:
    base = min(orig, new) * rolloff; width = ceil(L * orig / base); for output phase i and tap k the time is
    t = (-i / new) + (k - width) / orig (the first term evaluated in float32, as torchaudio's integer arange divided in
    the default dtype), scaled by base and clamped to [-L, L]; the window is cos(t * pi / (2 L))^2 and the tap
    sinc(pi t) * window * base / orig."""
    g = math.gcd(int(orig_freq), int(new_freq))
    orig, new = int(orig_freq) // g, int(new_freq) // g
    L = lowpass_filter_width
    base = min(orig, new) * rolloff
    width = math.ceil(L * orig / base)
    idx = np.arange(-width, width + orig, dtype=np.float64)[None, :] / orig
    phase = (np.arange(0, -new, -1).astype(np.float32) / np.float32(new)).astype(np.float64)[:, None]
    t = (phase + idx) * base
    t = np.clip(t, -L, L)
    window = np.cos(t * math.pi / L / 2) ** 2
    t = t * math.pi
    with np.errstate(invalid="ignore", divide="ignore"):
        taps = np.where(t == 0, 1.0, np.sin(t) / t)
    taps = taps * window * (base / orig)
    return taps.astype(np.float32), width, orig, new


def stream_outputs(chunks0, chunks1, n_ffts, hop, windows, mixer, max_log_mag, kernel, orig, new, width):
    """What the reference's chained head + resampler streams return for a sequence of pushes and a final flush
    (istft_head_a_20261002/stream.py:205-215: head.push then resampler.push per chunk; at the end
    resampler.push(head.flush()) + resampler.flush()). Returns ([head outputs per push] + [head flush],
    [resampler outputs per push] + [resampler flush + tail]), float32 like the reference."""
    K = np.asarray(mixer).shape[1]
    kl = np.asarray(kernel).shape[1]
    ys0 = np.concatenate([np.asarray(c, np.float64) for c in chunks0])
    ys1 = np.concatenate([np.asarray(c, np.float64) for c in chunks1])
    full = istft_decode(ys0, ys1, n_ffts, hop, windows, mixer, max_log_mag).astype(np.float32)
    counts, f = [], 0
    for c in chunks0:
        f += len(c)
        counts.append(istft_emitted(f, n_ffts, hop, K))
    counts.append(istft_emitted(f, n_ffts, hop, K, flushed=True))
    head, prev = [], 0
    for n in counts:
        head.append(full[prev:max(prev, n)])
        prev = max(prev, n)
    res_full = resample(full, kernel, orig, new, width, resample_emitted(len(full), orig, new, width, kl, True))
    res, prev, n_in = [], 0, 0
    for i, h in enumerate(head):
        n_in += len(h)
        n = resample_emitted(n_in, orig, new, width, kl, flushed=i == len(head) - 1)
        res.append(res_full[prev:max(prev, n)].astype(np.float32))
        prev = max(prev, n)
    return head, res

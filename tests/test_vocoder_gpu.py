"""The codec's streaming DSP tail on the GPU (zonos3_mini_b200.vocoder: zb_istft_head_push, zb_resample_push) against
the reference's golden stream outputs and the float64 oracle (oracle/istft.py).

Bar: float32 outputs of float64 arithmetic summed in another order than the reference's, so within 4 float32 ulps of
each output's peak (the reference's host and device streams agree to the same float32 rounding)."""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import istft

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden" / "istft_stream.npz"
N_FFTS, HOP = (736, 2208), 184


@pytest.fixture(scope="module")
def voc(zb):
    return zb.vocoder


@pytest.fixture(scope="module")
def stream_golden():
    return dict(np.load(GOLDEN))


@pytest.fixture(scope="module")
def codec(stream_golden):
    golden = stream_golden
    kernel, width, orig, new = istft.sinc_resample_kernel(44160, 44100, 16, 0.99)
    return dict(windows=[golden["window0"], golden["window1"]], mixer=golden["mixer"],
                max_log_mag=float(golden["max_log_mag"]), kernel=kernel, orig=orig, new=new, width=width)


def close(got, want, ulps=4):
    got = got.detach().cpu().numpy().astype(np.float64) if isinstance(got, torch.Tensor) else np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    assert got.shape == want.shape, (got.shape, want.shape)
    if want.size == 0:
        return
    bar = ulps * np.spacing(np.float32(np.abs(want).max()))
    err = np.abs(got - want).max()
    assert err <= bar, f"max error {err:.3g} above {bar:.3g} ({ulps} float32 ulps of the peak)"


def frames(rng, cols, n_ffts=N_FFTS, streams=None):
    lead = () if streams is None else (streams,)
    out = []
    for n in n_ffts:
        bins = n // 2 + 1
        lm = rng.normal(-3.0, 1.5, lead + (cols, bins))
        ph = rng.uniform(-np.pi, np.pi, lead + (cols, bins))
        out.append(np.concatenate([lm, ph], -1).astype(np.float32))
    return out


def make(voc, codec, **kw):
    dev = torch.device("cuda:0")
    head_kw = {k: kw[k] for k in ("streams", "max_cols") if k in kw}
    res_kw = {k: kw[k] for k in ("streams", "max_push") if k in kw}
    head = voc.IstftHeadStream(kw.get("n_ffts", N_FFTS), kw.get("hop", HOP), kw.get("windows", codec["windows"]),
                               kw.get("mixer", codec["mixer"]), kw.get("max_log_mag", codec["max_log_mag"]), dev,
                               **head_kw)
    res = voc.ResamplerStream(kw.get("kernel", codec["kernel"]), kw.get("orig", codec["orig"]), kw.get("new", codec["new"]),
                              kw.get("width", codec["width"]), dev, **res_kw)
    return head, res


def run_chain(head, res, chunks0, chunks1):
    heads, ress = [], []
    for y0, y1 in zip(chunks0, chunks1):
        h = head.push(torch.as_tensor(y0).cuda(), torch.as_tensor(y1).cuda())
        heads.append(h)
        ress.append(res.push(h))
    tail = head.flush()
    heads.append(tail)
    ress.append(torch.cat([res.push(tail), res.flush()], dim=-1))
    torch.cuda.synchronize()
    return heads, ress


def test_twiddles(voc):
    for n in (10, 736, 2208):
        tw = voc.IstftHeadStream((n, n), n // 2 if n > 10 else 5, [np.hanning(n)] * 2, np.ones((2, 1)), 1.0,
                                 "cuda:0").twiddles[0].cpu().numpy()
        e = (np.arange(n) + n // 2) % n - n // 2  # angles reduced to [-pi, pi) before NumPy rounds them
        want = np.exp(2j * np.pi * e / n)
        assert np.abs(tw[:, 0] + 1j * tw[:, 1] - want).max() < 1e-15  # a few ulps of 1 (NumPy rounds too)


def test_golden_stream(voc, stream_golden, codec):
    """The reference's own stream outputs for pushes of 3, 1, 0, 2, 4 and 8 frames and the flush."""
    golden = stream_golden
    head, res = make(voc, codec)
    n = len(golden["chunks"])
    heads, ress = run_chain(head, res, [golden[f"y0_{c}"] for c in range(n)], [golden[f"y1_{c}"] for c in range(n)])
    for c in range(n):
        close(heads[c], golden[f"head_{c}"])
        close(ress[c], golden[f"res_{c}"])
    close(heads[n], golden["head_flush"])
    close(ress[n], golden["res_flush"])


def test_stream_tail_chains_as_the_codec_does(voc, stream_golden, codec):
    """StreamTail (head then resampler per push; head flush through the resampler, then its flush) on the golden
    pushes: the reference's resampler outputs."""
    golden = stream_golden
    tail = voc.StreamTail(*make(voc, codec))
    n = len(golden["chunks"])
    for c in range(n):
        close(tail.push(torch.as_tensor(golden[f"y0_{c}"]).cuda(), torch.as_tensor(golden[f"y1_{c}"]).cuda()),
              golden[f"res_{c}"])
    close(tail.flush(), golden["res_flush"])
    with pytest.raises(ValueError, match="share"):
        voc.StreamTail(make(voc, codec, streams=2)[0], make(voc, codec)[1])


@pytest.mark.parametrize("max_cols,max_push", [(64, 1 << 16), (5, 700)])
def test_long_stream_matches_oracle(voc, codec, max_cols, max_push):
    """Two seconds of frames in uneven chunks; small max_cols / max_push split pushes and wrap the rings many times."""
    rng = np.random.default_rng(7)
    sizes = [1, 7, 13, 0, 39, 2, 100, 64, 65, 189]
    chunks = [frames(rng, c) for c in sizes]
    head, res = make(voc, codec, max_cols=max_cols, max_push=max_push)
    heads, ress = run_chain(head, res, [c[0] for c in chunks], [c[1] for c in chunks])
    want_h, want_r = istft.stream_outputs([c[0] for c in chunks], [c[1] for c in chunks], N_FFTS, HOP,
                                          codec["windows"], codec["mixer"], codec["max_log_mag"], codec["kernel"],
                                          codec["orig"], codec["new"], codec["width"])
    assert len(heads) == len(want_h)
    for got, want in zip(heads, want_h):
        close(got, want)
    for got, want in zip(ress, want_r):
        close(got, want)


def test_lockstep_streams_and_fork(voc, codec):
    """Several streams in one call, each equal to its own single-stream decode; a copy() continues independently."""
    rng = np.random.default_rng(11)
    S = 5
    sizes = [4, 9, 3]
    chunks = [frames(rng, c, streams=S) for c in sizes]
    head, res = make(voc, codec, streams=S, max_cols=8)
    for y0, y1 in chunks[:2]:
        res.push(head.push(torch.as_tensor(y0).cuda(), torch.as_tensor(y1).cuda()))
    twin_h, twin_r = head.copy(), res.copy()
    alt = frames(rng, 6, streams=S)
    a = [twin_r.push(twin_h.push(torch.as_tensor(alt[0]).cuda(), torch.as_tensor(alt[1]).cuda()))]
    b = [res.push(head.push(torch.as_tensor(chunks[2][0]).cuda(), torch.as_tensor(chunks[2][1]).cuda()))]
    a.append(torch.cat([twin_r.push(twin_h.flush()), twin_r.flush()], 1))
    b.append(torch.cat([res.push(head.flush()), res.flush()], 1))
    torch.cuda.synchronize()
    for s in range(S):
        for branch, tail in ((a, alt), (b, chunks[2])):
            c0 = [chunks[0][0][s], chunks[1][0][s], tail[0][s]]
            c1 = [chunks[0][1][s], chunks[1][1][s], tail[1][s]]
            _, want_r = istft.stream_outputs(c0, c1, N_FFTS, HOP, codec["windows"], codec["mixer"],
                                             codec["max_log_mag"], codec["kernel"], codec["orig"], codec["new"],
                                             codec["width"])
            got = torch.cat([branch[0][s], branch[1][s]]).cpu().numpy()
            close(got, np.concatenate(want_r[2:]))


def test_float64_inputs_and_generic_radices(voc):
    """Other sizes: n_fft 20 and 60 (half lengths 10 = 2 * 5 and 30 = 2 * 3 * 5), hop 10, a 5-tap mixer, a 3 -> 2
    resampler; float64 frames and float64 resampler input."""
    rng = np.random.default_rng(3)
    n_ffts, hop = (20, 60), 10
    windows = [0.5 - 0.5 * np.cos(2 * np.pi * np.arange(n) / n) for n in n_ffts]
    mixer = rng.normal(0, 0.3, (2, 5))
    kernel = rng.normal(0, 0.2, (2, 2 * 4 + 3))
    dev = torch.device("cuda:0")
    sizes = [2, 1, 5, 3]
    chunks = [[c.astype(np.float64) for c in frames(rng, k, n_ffts)] for k in sizes]
    head = voc.IstftHeadStream(n_ffts, hop, windows, mixer, 0.5, dev, max_cols=2)
    res = voc.ResamplerStream(kernel, 3, 2, 4, dev, max_push=7)
    heads, ress = [], []
    for y0, y1 in chunks:
        h = head.push(torch.as_tensor(y0).cuda(), torch.as_tensor(y1).cuda())
        heads.append(h)
        ress.append(res.push(h.double()))
    tail = head.flush()
    heads.append(tail)
    ress.append(torch.cat([res.push(tail.double()), res.flush()]))
    want_h, want_r = istft.stream_outputs([c[0] for c in chunks], [c[1] for c in chunks], n_ffts, hop, windows, mixer,
                                          0.5, kernel, 3, 2, 4)
    for got, want in zip(heads, want_h):
        close(got, want)
    for got, want in zip(ress, want_r):
        close(got, want)


@pytest.mark.parametrize("n_ffts,hop,taps", [((1024, 8192), 512, 31), ((96, 288), 48, 9)])
def test_other_sizes_and_both_overlap_add_paths(voc, n_ffts, hop, taps):
    """Sizes beyond the codec's: n_fft 8192 (the largest the kernels take: half length 4096 = 4^6, 131 KB of shared
    memory per frame CTA) with 1024, and 96 / 288 (half lengths 48 = 4^2 * 3 and 144 = 4^2 * 9 -> 3 * 3: radix 3 twice);
    pushes of 3 and 40 frames (the second through the grouped overlap-add) and the flush, against the oracle."""
    rng = np.random.default_rng(13)
    windows = [0.5 - 0.5 * np.cos(2 * np.pi * np.arange(n) / n) for n in n_ffts]
    mixer = rng.normal(0, 0.1, (2, taps))
    mixer[0, taps // 2] += 1.0
    kernel = rng.normal(0, 0.2, (2, 2 * 4 + 3))
    dev = torch.device("cuda:0")
    chunks = [frames(rng, k, n_ffts, streams=3) for k in (3, 40)]
    head = voc.IstftHeadStream(n_ffts, hop, windows, mixer, 1.5, dev, streams=3)
    res = voc.ResamplerStream(kernel, 3, 2, 4, dev, streams=3)
    outs = [res.push(head.push(torch.as_tensor(y0).cuda(), torch.as_tensor(y1).cuda())) for y0, y1 in chunks]
    outs.append(torch.cat([res.push(head.flush()), res.flush()], 1))
    torch.cuda.synchronize()
    for s_ in range(3):
        _, want_r = istft.stream_outputs([c[0][s_] for c in chunks], [c[1][s_] for c in chunks], n_ffts, hop,
                                         windows, mixer, 1.5, kernel, 3, 2, 4)
        for got, want in zip(outs, want_r):
            close(got[s_], want)


def test_stream_errors(voc, codec):
    head, res = make(voc, codec)
    assert head.flush().numel() == 0  # nothing pushed: nothing to flush
    with pytest.raises(ValueError, match="branch 0 has shape"):
        head.push(torch.zeros(2, 10, device="cuda"), torch.zeros(2, 2210, device="cuda"))
    with pytest.raises(ValueError, match="branch 1 has shape"):
        head.push(torch.zeros(2, 738, device="cuda"), torch.zeros(3, 2210, device="cuda"))
    with pytest.raises(ValueError, match="mixer kernel must be odd"):
        type(head)(N_FFTS, HOP, codec["windows"], np.zeros((2, 4)), 1.0, "cuda:0")
    with pytest.raises(ValueError, match="window of"):
        type(head)(N_FFTS, HOP, [codec["windows"][0][:-1], codec["windows"][1]], codec["mixer"], 1.0, "cuda:0")
    with pytest.raises(ValueError, match="kernel shape"):
        type(res)(np.zeros((735, 10)), 736, 735, 17, "cuda:0")
    head2, _ = make(voc, codec)
    rng = np.random.default_rng(0)
    y0, y1 = frames(rng, 2)
    assert head2.push(torch.as_tensor(y0).cuda(), torch.as_tensor(y1).cuda()).numel() == 0
    assert head2.flush().numel() == 2 * HOP
    with pytest.raises(RuntimeError, match="push after flush"):
        head2.push(torch.as_tensor(y0).cuda(), torch.as_tensor(y1).cuda())
    assert head2.flush().numel() == 0


def test_many_streams_property(voc, codec):
    """256 lock-step streams, one second (240 frames) each in pushes of 4 frames: a sample of streams against the
    oracle, and every stream's output length equal to the reference's schedule."""
    rng = np.random.default_rng(5)
    S, total, step = 256, 240, 4
    ys = frames(rng, total, streams=S)
    head, res = make(voc, codec, streams=S, max_cols=step)
    y0 = torch.as_tensor(ys[0]).cuda()
    y1 = torch.as_tensor(ys[1]).cuda()
    outs = []
    for c0 in range(0, total, step):
        outs.append(res.push(head.push(y0[:, c0:c0 + step], y1[:, c0:c0 + step])))
    outs.append(torch.cat([res.push(head.flush()), res.flush()], 1))
    got = torch.cat(outs, 1).cpu().numpy()
    assert got.shape == (S, -(-735 * total * HOP // 736))
    assert np.isfinite(got).all()
    for s in (0, 1, 127, 255):
        full = istft.istft_decode(ys[0][s], ys[1][s], N_FFTS, HOP, codec["windows"], codec["mixer"],
                                  codec["max_log_mag"]).astype(np.float32)
        want = istft.resample(full, codec["kernel"], codec["orig"], codec["new"], codec["width"], got.shape[1])
        close(got[s], want)

"""The codec's streaming DSP tail on the GPU: the two-branch iSTFT head with its FIR mixer, and the 44160 -> 44100 Hz
sinc resampler (the reference's model/src/zonos3/codec/stream_device.py: IstftHeadStream :15-146 and
ResamplerStream :149-197, torch twins of the NumPy ports in stream_host.py).

Same constructor arguments, ``push``/``flush``/``copy`` methods, error messages and float64 arithmetic as the
reference's classes; the work runs in the library's kernels (``zb_istft_head_push``, ``zb_resample_push``) over state
that stays on the device (overlap-add carries, mixer-input and resampler-input rings). ``streams=S`` runs S streams in
lock step: ``push`` then takes [S, cols, n + 2] frames (or [S, samples]) and returns [S, samples]; the default S = 1
takes and returns the reference's shapes. Positions and lengths are host integers, as in the reference's device twin,
so nothing synchronises with the device except the caller's copy of the output.
"""

from __future__ import annotations

import torch

from . import _lib


def _next_pow2(x: int) -> int:
    return 1 << max(0, int(x) - 1).bit_length()


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _f64(t, device) -> torch.Tensor:
    return torch.as_tensor(t).to(device=device, dtype=torch.float64).contiguous()


def _frames_input(y, device):
    """Head frames as float32 or float64 device rows (other float types widen to float32 exactly)."""
    y = torch.as_tensor(y)
    if y.dtype not in (torch.float32, torch.float64):
        y = y.float()
    y = y.to(device)
    if y.ndim != 3 or y.stride(2) != 1 or y.stride(1) != y.shape[2]:  # rows of a stream must be contiguous
        y = y.contiguous()
    return y


class IstftHeadStream:
    """Two-branch centered iSTFT (shared hop) followed by the linear FIR mixer, fed head frames incrementally."""

    def __init__(self, n_ffts, hop, windows, mixer, max_log_mag, device, *, streams: int = 1, max_cols: int = 64):
        self.n_ffts = [int(n) for n in n_ffts]
        self.hop = int(hop)
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise ValueError("istft: the B200 head stream runs on a CUDA device")
        self.windows = [_f64(w, self.device) for w in windows]
        self.mixer = _f64(mixer, self.device)
        if self.mixer.ndim != 2 or self.mixer.shape[0] != 2 or self.mixer.shape[1] % 2 != 1:
            raise ValueError("istft: mixer kernel must be odd")
        if len(self.n_ffts) != 2 or len(self.windows) != 2:
            raise ValueError("istft: the head has two branches")
        for n, w in zip(self.n_ffts, self.windows):
            if len(w) != n or n % self.hop:
                raise ValueError(f"istft: window of {len(w)} taps for n_fft {n}, hop {self.hop}")
            if n % 2 or n // self.hop < 2:
                raise ValueError(f"istft: n_fft {n} must be even and at least two hops")
        self.max_log_mag = float(max_log_mag)
        self.K = self.mixer.shape[1]
        self.h = (self.K - 1) // 2
        self.streams = int(streams)
        self.max_cols = int(max_cols)  # longer pushes run as several calls of at most max_cols frames
        if self.streams < 1 or self.max_cols < 1:
            raise ValueError("istft: streams and max_cols must be positive")
        self.ring_size = _next_pow2(self.max_cols * self.hop + 2 * self.K + max(self.n_ffts))
        f64 = dict(dtype=torch.float64, device=self.device)
        self.twiddles = []
        with torch.cuda.device(self.device):
            for n in self.n_ffts:
                tw = torch.empty(n, 2, **f64)
                _lib.call("zb_istft_twiddles", n, tw.data_ptr(), _stream(self.device))
                self.twiddles.append(tw)
        self.carry = [torch.zeros(2, self.streams, n - self.hop, **f64) for n in self.n_ffts]
        self.rings = [torch.zeros(self.streams, self.ring_size, **f64) for _ in range(2)]
        self.scratch = torch.empty(self.streams * self.max_cols * sum(self.n_ffts), **f64)
        self.parity = 0
        self.mix_next = 0
        self.frames = 0
        self.done = False

    def copy(self) -> "IstftHeadStream":
        """An independent twin: the carries and rings are copied; constants and the frame scratch are shared (so the
        twins run on one CUDA stream, as the reference's run on one device)."""
        twin = object.__new__(IstftHeadStream)
        twin.__dict__.update(self.__dict__)
        twin.carry = [t.clone() for t in self.carry]
        twin.rings = [t.clone() for t in self.rings]
        return twin

    def _empty(self) -> torch.Tensor:
        shape = (0,) if self.streams == 1 else (self.streams, 0)
        return torch.zeros(shape, dtype=torch.float32, device=self.device)

    def _emitted(self, frames: int) -> int:
        """Mixer outputs whose taps are all final after `frames` frames (stream_host.py:117-121)."""
        return max(self.mix_next, frames * self.hop - max(self.n_ffts) // 2 - self.h)

    def _call(self, ys, y_f64: int, cols: int, mix_to: int, flush: int, out) -> None:
        (y0, s0), (y1, s1) = ((None, 0), (None, 0)) if ys is None else [(y.data_ptr(), y.stride(0)) for y in ys]
        _lib.call(
            "zb_istft_head_push", y0, s0, y1, s1, y_f64, self.streams, cols, self.n_ffts[0], self.n_ffts[1], self.hop,
            self.windows[0].data_ptr(), self.windows[1].data_ptr(), self.twiddles[0].data_ptr(),
            self.twiddles[1].data_ptr(), self.max_log_mag, self.mixer.data_ptr(), self.K, self.carry[0].data_ptr(),
            self.carry[1].data_ptr(), self.parity, self.rings[0].data_ptr(), self.rings[1].data_ptr(), self.ring_size,
            self.frames, self.mix_next, mix_to, flush, self.scratch.data_ptr(), self.scratch.numel(),
            out.data_ptr() if out is not None else None, _stream(self.device))

    def push(self, y0, y1) -> torch.Tensor:
        """y_i [cols, n_i + 2] (or [streams, cols, n_i + 2]): log-magnitude for n_i//2+1 bins, then phase. Returns the
        44160 Hz samples now final."""
        if self.done:
            raise RuntimeError("istft: push after flush")
        ys = []
        cols = None
        for i, y in enumerate((y0, y1)):
            n = self.n_ffts[i]
            y = _frames_input(y, self.device)
            if self.streams == 1 and y.ndim == 2:
                y = y.unsqueeze(0)
            if (y.ndim != 3 or y.shape[0] != self.streams or y.shape[2] != n + 2
                    or (cols is not None and y.shape[1] != cols)):
                lead = "" if self.streams == 1 else f"{self.streams}, "
                raise ValueError(f"istft: branch {i} has shape {tuple(y.shape)}, expected [{lead}cols, {n + 2}]")
            cols = y.shape[1]
            ys.append(y)
        if cols == 0:
            return self._empty()
        if ys[0].dtype != ys[1].dtype:
            ys = [y.double() for y in ys]
        y_f64 = int(ys[0].dtype == torch.float64)
        outs = []
        with torch.cuda.device(self.device):
            for c0 in range(0, cols, self.max_cols):
                c = min(self.max_cols, cols - c0)
                parts = [y[:, c0:c0 + c] for y in ys]  # frame rows stay contiguous; streams keep their stride
                mix_to = self._emitted(self.frames + c)
                out = torch.empty(self.streams, mix_to - self.mix_next, dtype=torch.float32, device=self.device)
                self._call(parts, y_f64, c, mix_to, 0, out)
                self.frames += c
                self.parity ^= 1
                self.mix_next = mix_to
                outs.append(out)
        out = torch.cat(outs, dim=1)
        return out[0] if self.streams == 1 else out

    def flush(self) -> torch.Tensor:
        """End of stream: every sample m < frames*hop is final; the mixer sees h zeros after the last sample."""
        if self.done or self.frames == 0:
            return self._empty()
        self.done = True
        mix_to = self.frames * self.hop
        out = torch.empty(self.streams, mix_to - self.mix_next, dtype=torch.float32, device=self.device)
        with torch.cuda.device(self.device):
            self._call(None, 0, 0, mix_to, 1, out)
        self.mix_next = mix_to
        return out[0] if self.streams == 1 else out


class ResamplerStream:
    """Streaming torchaudio sinc resampler: out[n*new + i] = sum_k kernel[i][k] * x[n*orig + k - width]."""

    def __init__(self, kernel, orig, new, width, device, *, streams: int = 1, max_push: int = 1 << 16):
        self.orig, self.new, self.width = int(orig), int(new), int(width)
        self.kl = 2 * self.width + self.orig
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise ValueError("resampler: the B200 resampler stream runs on a CUDA device")
        self.kernel = _f64(kernel, self.device)
        if tuple(self.kernel.shape) != (self.new, self.kl):
            raise ValueError(f"resampler: kernel shape {tuple(self.kernel.shape)}, expected {(self.new, self.kl)}")
        self.kernel_t = self.kernel.t().contiguous()  # [kl, new]: one coalesced row per tap
        self.streams = int(streams)
        self.max_push = int(max_push)
        if self.streams < 1 or self.max_push < 1:
            raise ValueError("resampler: streams and max_push must be positive")
        self.ring_size = _next_pow2(self.max_push + self.kl + 2 * self.orig)
        self.ring = torch.zeros(self.streams, self.ring_size, dtype=torch.float64, device=self.device)
        self.n_in = 0  # samples pushed
        self.next_block = 0
        self._ws = None

    def copy(self) -> "ResamplerStream":
        """An independent twin (the input ring is copied; the kernel is shared)."""
        twin = object.__new__(ResamplerStream)
        twin.__dict__.update(self.__dict__)
        twin.ring = self.ring.clone()
        twin._ws = None
        return twin

    def _workspace(self, elems: int) -> torch.Tensor | None:
        """Float64 scratch for the tap-split of a call with few (stream, block) pairs; calls too large for the
        cached buffer (above 2^22 elements) run unsplit, where the tiles alone fill the GPU."""
        if elems > 1 << 22:
            return None
        if self._ws is None or self._ws.numel() < elems:
            self._ws = torch.empty(elems, dtype=torch.float64, device=self.device)
        return self._ws

    def _out(self, count: int) -> torch.Tensor:
        return torch.empty(self.streams, count, dtype=torch.float32, device=self.device)

    def _run(self, x, count: int, flush: bool) -> torch.Tensor:
        O, N, W, KL = self.orig, self.new, self.width, self.kl
        n_in = self.n_in + count
        if flush:
            total = -(-N * n_in // O)
            end = -(-total // N)
        else:
            reach = n_in + W - KL
            end = reach // O + 1 if reach >= 0 else 0
        end = max(end, self.next_block)
        out_count = (end - self.next_block) * N
        if flush and end > self.next_block:
            out_count = total - self.next_block * N
        out = self._out(out_count)
        x_ptr, x_f64, x_stride = (None, 0, 0) if x is None else (x.data_ptr(), int(x.dtype == torch.float64), x.stride(0))
        ws = self._workspace(8 * self.streams * (end - self.next_block) * N) if out_count else None
        _lib.call("zb_resample_push", x_ptr, x_f64, x_stride, self.streams, count, self.ring.data_ptr(),
                  self.ring_size, self.n_in, self.kernel_t.data_ptr(), O, N, W, self.next_block, end, out_count,
                  out.data_ptr() if out_count else None, ws.data_ptr() if ws is not None else None,
                  ws.numel() if ws is not None else 0, _stream(self.device))
        self.n_in = n_in
        self.next_block = end
        return out

    def push(self, x) -> torch.Tensor:
        x = torch.as_tensor(x)
        if x.dtype not in (torch.float32, torch.float64):
            x = x.float()
        x = x.to(self.device)
        x = x.reshape(1, -1) if self.streams == 1 else x
        if x.ndim != 2 or x.shape[0] != self.streams:
            raise ValueError(f"resampler: input of shape {tuple(x.shape)} for {self.streams} streams")
        x = x.contiguous()
        outs = []
        with torch.cuda.device(self.device):
            for c0 in range(0, max(1, x.shape[1]), self.max_push):
                part = x[:, c0:c0 + self.max_push]
                outs.append(self._run(part if part.shape[1] else None, part.shape[1], False))
        out = torch.cat(outs, dim=1)
        return out[0] if self.streams == 1 else out

    def flush(self) -> torch.Tensor:
        with torch.cuda.device(self.device):
            out = self._run(None, 0, True)
        return out[0] if self.streams == 1 else out


class StreamTail:
    """The head stream and the resampler chained as the codec's decode loop chains them
    (model/src/zonos3/codec/istft_head_a_20261002/stream.py:205-215 per chunk, :211-214 at the end): each push returns
    the 44.1 kHz samples now final, `flush()` the rest."""

    def __init__(self, head: IstftHeadStream, resampler: ResamplerStream):
        if head.streams != resampler.streams or head.device != resampler.device:
            raise ValueError("stream tail: the head and the resampler must share their device and stream count")
        self.head, self.resampler = head, resampler

    def push(self, y0, y1) -> torch.Tensor:
        return self.resampler.push(self.head.push(y0, y1))

    def flush(self) -> torch.Tensor:
        return torch.cat([self.resampler.push(self.head.flush()), self.resampler.flush()], dim=-1)

    def copy(self) -> "StreamTail":
        return StreamTail(self.head.copy(), self.resampler.copy())

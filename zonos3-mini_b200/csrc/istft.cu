// The codec's streaming DSP tail on the device: the two-branch centred iSTFT head with its FIR mixer, and the
// polyphase sinc resampler behind it (model/src/zonos3/codec/stream_host.py: IstftHeadStream :16-127,
// ResamplerStream :122-171; the reference's torch twins in stream_device.py run the same float64 steps with
// torch.fft.irfft, F.fold and F.conv1d). Arithmetic is float64 like the reference's; outputs are float32.
//
// Streams advance in lock step: one call pushes `cols` head frames for each of `streams` streams (the reference's
// class is the streams == 1 case). Positions and lengths are host integers, as in the reference's device twin.
//
//   istft_frames_kernel   one CTA per (frame, branch): magnitude/phase -> spectrum in shared memory, the length-n
//                         inverse real DFT as a length-n/2 complex inverse DFT (even/odd samples as real/imaginary
//                         parts) by a mixed-radix Stockham pass per factor of n/2, times the window -> frame scratch.
//   istft_ola_kernel      one thread per overlap-add position of a branch: the carried partial sums of earlier
//                         pushes plus this push's frames; positions below frames * hop are final and go, divided by
//                         the overlap-added squared window and without the n/2 centre padding, into the branch's
//                         mixer-input ring; the rest become the next carry.
//   istft_mix_kernel      one thread per emitted sample: the K-tap correlation over both branches' rings.
//   resample_append_kernel / resample_kernel   the resampler's input ring, then out[b*new + i] =
//                         sum_k kernel[i][k] * x[b*orig + k - width], a CTA holding the input windows of 8 (stream,
//                         block) pairs in shared memory and one output phase per thread (kernel stored transposed).
#include <algorithm>
#include <vector>

#include "common.cuh"

namespace {

constexpr int kMaxStages = 24;
constexpr int kFrameThreads = 256;
constexpr int kMaxN = 8192;  // (n + 1) complex float64 values of shared memory per frame CTA

struct FrameBranch {
  const void* y;           // [frames, n + 2] float32 or float64: log-magnitude for n/2 + 1 bins, then phase
  const double* window;    // [n]
  const double2* twiddle;  // [n]: e^{2 pi i e / n}
  double* out;             // [frames, n] windowed frames
  int n;
  int nstages;
  int radix[kMaxStages];
};

struct FrameParams {
  FrameBranch br[2];
  int frames;
  int y_f64;
  double max_log_mag;
};

__device__ __forceinline__ double2 cmul(double2 a, double2 b) {
  return make_double2(a.x * b.x - a.y * b.y, a.x * b.y + a.y * b.x);
}

__device__ __forceinline__ double2 cmad(double2 acc, double2 a, double2 b) {
  acc.x = fma(a.x, b.x, fma(-a.y, b.y, acc.x));
  acc.y = fma(a.x, b.y, fma(a.y, b.x, acc.y));
  return acc;
}

// Windowed inverse real DFT of one head frame of one branch (stream_host.py:55-63):
//   X[k] = exp(min(lm_k, max_log_mag)) * (cos ph_k, sin ph_k), imaginary parts of bins 0 and n/2 zeroed;
//   x[t] = (1/n) sum_{k<n} X[k] w^{kt} with the Hermitian extension, w = e^{2 pi i / n};  frame = x * window.
// With M = n/2: z[m] = x[2m] + i x[2m+1] = (1/n) sum_{k<M} Z[k] W^{km}, W = w^2, where
//   Z[k] = (X[k] + conj X[M-k]) + i w^k (X[k] - conj X[M-k]).
// The length-M inverse DFT runs one Stockham pass per radix R of M's factorisation (Ns = product of the radices
// before it): output q of butterfly j is sum_r src[j + r M/R] W^{r s}, s = (j mod Ns) M/(Ns R) + q M/R, stored at
// (j / Ns) Ns R + (j mod Ns) + q Ns. The powers W^{r s} come from a recurrence re-anchored on the exact table every
// 16 terms.
__global__ void __launch_bounds__(kFrameThreads) istft_frames_kernel(FrameParams p) {
  zb::pdl_enter();
  const FrameBranch& b = p.br[blockIdx.y];
  const int n = b.n, M = n / 2, bins = M + 1;
  const int64_t frame = blockIdx.x;
  extern __shared__ double2 sm[];
  double2* X = sm;          // [M + 1], later the second Stockham buffer
  double2* A = sm + M + 1;  // [M]
  const double2* tw = b.twiddle;

  for (int k = threadIdx.x; k < bins; k += blockDim.x) {
    double lm, ph;
    if (p.y_f64) {
      const double* row = static_cast<const double*>(b.y) + frame * (n + 2);
      lm = row[k];
      ph = row[bins + k];
    } else {
      const float* row = static_cast<const float*>(b.y) + frame * (n + 2);
      lm = (double)row[k];
      ph = (double)row[bins + k];
    }
    const double mag = exp(fmin(lm, p.max_log_mag));
    double s, c;
    sincos(ph, &s, &c);
    X[k] = make_double2(mag * c, (k == 0 || k == M) ? 0.0 : mag * s);
  }
  __syncthreads();
  for (int k = threadIdx.x; k < M; k += blockDim.x) {
    const double2 xk = X[k], xc = X[M - k];
    const double2 e = make_double2(xk.x + xc.x, xk.y - xc.y);  // X[k] + conj X[M-k]
    const double2 d = make_double2(xk.x - xc.x, xk.y + xc.y);  // X[k] - conj X[M-k]
    const double2 o = cmul(__ldg(tw + k), d);
    A[k] = make_double2(e.x - o.y, e.y + o.x);
  }
  __syncthreads();

  double2* src = A;
  double2* dst = X;
  int Ns = 1;
  for (int st = 0; st < b.nstages; ++st) {
    const int R = b.radix[st];
    const int MR = M / R;
    const int span = M / (Ns * R);
    for (int t = threadIdx.x; t < M; t += blockDim.x) {
      const int j = t % MR, q = t / MR;
      const int jn = j % Ns;
      const int s = (jn * span + q * MR) % M;
      const double2 w = __ldg(tw + 2 * s);
      double2 acc = src[j];
      double2 cur = w;
      int e = s;
      for (int r = 1; r < R; ++r) {
        if ((r & 15) == 0) cur = __ldg(tw + 2 * e);
        acc = cmad(acc, src[j + r * MR], cur);
        cur = cmul(cur, w);
        e += s;
        if (e >= M) e -= M;
      }
      dst[(j / Ns) * Ns * R + jn + q * Ns] = acc;
    }
    __syncthreads();
    double2* tmp = src;
    src = dst;
    dst = tmp;
    Ns *= R;
  }

  const double inv_n = 1.0 / (double)n;
  double* out = b.out + frame * n;
  for (int m = threadIdx.x; m < M; m += blockDim.x) {
    const double2 z = src[m];
    const double2 win = *reinterpret_cast<const double2*>(b.window + 2 * m);
    *reinterpret_cast<double2*>(out + 2 * m) = make_double2(z.x * inv_n * win.x, z.y * inv_n * win.y);
  }
}

struct OlaBranch {
  const double* frames;  // [streams, cols, n]
  const double* window;  // [n]
  const double* carry_in;  // [streams, n - hop]
  double* carry_out;       // [streams, n - hop]
  double* ring;            // [streams, ring]
  int n;
};

struct OlaParams {
  OlaBranch br[2];
  int streams, cols, hop, h;
  int64_t frames_before;
  int64_t keep;  // flush: mixer-input indices >= keep are not needed
  int ring_mask;
  int flush;
};

__device__ __forceinline__ int64_t ceil_div_pos(int64_t a, int64_t b) { return a <= 0 ? 0 : (a + b - 1) / b; }

// One thread per overlap-add position P0 + t of one branch of one stream (stream_host.py:64-79 and :104-113):
// t < n - hop carries the partial sum of earlier pushes; this push's frames c cover [P0 + c hop, P0 + c hop + n).
// Positions below P1 = (frames_before + cols) hop are final: divided by the overlap-added squared window of every
// frame so far, written to the mixer input at h + p - n/2 when p >= n/2. The others are the next push's carry.
// At flush (cols == 0) every carried position is final.
__global__ void __launch_bounds__(256) istft_ola_kernel(OlaParams p) {
  zb::pdl_enter();
  const OlaBranch& b = p.br[blockIdx.z];
  const int s = blockIdx.y;
  const int n = b.n, hop = p.hop, carry = n - hop;
  const int64_t count = p.flush ? carry : (int64_t)p.cols * hop + carry;
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= count) return;
  const int64_t P0 = p.frames_before * hop;
  const int64_t P1 = P0 + (int64_t)p.cols * hop;
  const int64_t pos = P0 + t;
  double v = t < carry ? b.carry_in[(int64_t)s * carry + t] : 0.0;
  if (!p.flush) {
    const int64_t c_lo = ceil_div_pos(t - n + 1, hop);
    const int64_t c_hi = min((int64_t)p.cols - 1, t / hop);
    const double* fr = b.frames + (int64_t)s * p.cols * n;
    for (int64_t c = c_lo; c <= c_hi; ++c) v += fr[c * n + (t - c * hop)];
  }
  if (p.flush || pos < P1) {
    const int64_t total = p.frames_before + p.cols;
    const int64_t e_lo = ceil_div_pos(pos - n + 1, hop);
    const int64_t e_hi = min(total - 1, pos / hop);
    double env = 0.0;
    for (int64_t c = e_lo; c <= e_hi; ++c) {
      const double w = b.window[pos - c * hop];
      env += w * w;
    }
    if (pos >= n / 2) {
      const int64_t idx = p.h + pos - n / 2;
      if (!p.flush || idx < p.keep) b.ring[(int64_t)s * (p.ring_mask + 1) + (idx & p.ring_mask)] = v / env;
    }
  } else {
    b.carry_out[(int64_t)s * carry + (pos - P1)] = v;
  }
}

struct MixParams {
  const double* ring0;
  const double* ring1;
  const double* mixer;  // [2, K]
  float* out;           // [streams, mix_to - mix_from]
  int64_t mix_from, mix_to;
  int64_t limit;  // mixer-input indices >= limit read as zero (the zeros appended at flush)
  int K, ring_mask;
};

constexpr int kMixTile = 256;
constexpr int kMaxTaps = 1023;

// y[m] = sum_c sum_k mixer[c][k] * in_c[m + k] for m in [mix_from, mix_to) (stream_host.py:115-127): a CTA stages
// its tile's inputs (tile + K - 1 values of each branch) and the taps in shared memory.
__global__ void __launch_bounds__(kMixTile) istft_mix_kernel(MixParams p) {
  zb::pdl_enter();
  extern __shared__ double msm[];
  const int K = p.K;
  const int width = kMixTile + K - 1;
  double* taps = msm;           // [2K]
  double* in0 = msm + 2 * K;    // [width]
  double* in1 = in0 + width;    // [width]
  const int s = blockIdx.y;
  const int64_t m0 = p.mix_from + (int64_t)blockIdx.x * kMixTile;
  const int64_t ring = (int64_t)p.ring_mask + 1;
  for (int i = threadIdx.x; i < 2 * K; i += blockDim.x) taps[i] = p.mixer[i];
  for (int i = threadIdx.x; i < width; i += blockDim.x) {
    const int64_t idx = m0 + i;
    const bool live = idx < p.limit && idx < p.mix_to + K - 1;
    in0[i] = live ? p.ring0[s * ring + (idx & p.ring_mask)] : 0.0;
    in1[i] = live ? p.ring1[s * ring + (idx & p.ring_mask)] : 0.0;
  }
  __syncthreads();
  const int64_t m = m0 + threadIdx.x;
  if (m >= p.mix_to) return;
  double y0 = 0.0, y1 = 0.0;
  for (int k = 0; k < K; ++k) {
    y0 = fma(taps[k], in0[threadIdx.x + k], y0);
    y1 = fma(taps[K + k], in1[threadIdx.x + k], y1);
  }
  p.out[(int64_t)s * (p.mix_to - p.mix_from) + (m - p.mix_from)] = (float)(y0 + y1);
}

__global__ void istft_twiddle_kernel(int n, double2* out) {
  const int e = blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= n) return;
  double s, c;
  sincospi(2.0 * (double)e / (double)n, &s, &c);
  out[e] = make_double2(c, s);
}

// Radices of M: fours, then a two, then odd factors ascending.
int radix_plan(int M, int* radix) {
  int k = 0;
  while (M % 4 == 0 && M > 4 && k < kMaxStages) radix[k++] = 4, M /= 4;
  while (M % 2 == 0 && M > 2 && k < kMaxStages) radix[k++] = 2, M /= 2;
  for (int f = 3; f * f <= M && k < kMaxStages; f += 2)
    while (M % f == 0 && M > f && k < kMaxStages) radix[k++] = f, M /= f;
  if (k < kMaxStages && M > 1) radix[k++] = M;
  return k < kMaxStages ? k : -1;
}

}  // namespace

namespace {

struct AppendParams {
  const void* x;  // [streams, count] (row stride x_stride) float32 or float64
  int64_t x_stride;
  int x_f64;
  int count;
  double* ring;  // [streams, ring]
  int ring_mask;
  int64_t n_in_before;
};

__global__ void __launch_bounds__(256) resample_append_kernel(AppendParams p) {
  zb::pdl_enter();
  const int s = blockIdx.y;
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= p.count) return;
  const int64_t i = (int64_t)s * p.x_stride + t;
  const double v = p.x_f64 ? static_cast<const double*>(p.x)[i] : (double)static_cast<const float*>(p.x)[i];
  p.ring[(int64_t)s * (p.ring_mask + 1) + ((p.n_in_before + t) & p.ring_mask)] = v;
}

constexpr int kResPairs = 8;     // (stream, block) input windows per CTA
constexpr int kResThreads = 128;  // output phases per CTA

struct ResampleParams {
  const double* ring;      // [streams, ring]
  const double* kernel_t;  // [kl, new]: kernel transposed
  float* out;              // [streams, out_count]
  int64_t n_in;            // samples pushed so far (inputs at or past n_in read as zero)
  int64_t block_from;
  int64_t out_count;       // outputs per stream of this call
  int nblocks;             // blocks per stream of this call
  int streams;
  int orig, nnew, width, kl;
  int ring_mask;
};

// out[b * new + i] = sum_k kernel[i][k] * x[b * orig + k - width] (stream_host.py:145-171), inputs outside
// [0, n_in) reading zero. A CTA loads the kl-sample input windows of up to 8 (stream, block) pairs into shared memory;
// thread i then walks the kernel's column i (kernel_t row k, coalesced across the CTA's phases) once for all pairs.
__global__ void __launch_bounds__(kResThreads) resample_kernel(ResampleParams p) {
  zb::pdl_enter();
  extern __shared__ double rsm[];  // [kResPairs][kl]
  const int kl = p.kl;
  const int64_t pair0 = (int64_t)blockIdx.y * kResPairs;
  const int64_t pairs_total = (int64_t)p.streams * p.nblocks;
  const int pairs = (int)min((int64_t)kResPairs, pairs_total - pair0);
  const int64_t ring = (int64_t)p.ring_mask + 1;
  for (int g = 0; g < pairs; ++g) {
    const int64_t pr = pair0 + g;
    const int64_t s = pr / p.nblocks;
    const int64_t blk = p.block_from + pr % p.nblocks;
    const int64_t start = blk * p.orig - p.width;
    for (int k = threadIdx.x; k < kl; k += blockDim.x) {
      const int64_t t = start + k;
      rsm[g * kl + k] = (t >= 0 && t < p.n_in) ? p.ring[s * ring + (t & p.ring_mask)] : 0.0;
    }
  }
  __syncthreads();
  const int i = blockIdx.x * kResThreads + threadIdx.x;
  if (i >= p.nnew) return;
  double acc[kResPairs];
#pragma unroll
  for (int g = 0; g < kResPairs; ++g) acc[g] = 0.0;
  const double* col = p.kernel_t + i;
#pragma unroll 4
  for (int k = 0; k < kl; ++k) {
    const double kv = __ldg(col + (int64_t)k * p.nnew);
#pragma unroll
    for (int g = 0; g < kResPairs; ++g) acc[g] = fma(kv, rsm[g * kl + k], acc[g]);
  }
  for (int g = 0; g < pairs; ++g) {
    const int64_t pr = pair0 + g;
    const int64_t s = pr / p.nblocks;
    const int64_t o = (pr % p.nblocks) * p.nnew + i;
    if (o < p.out_count) p.out[s * p.out_count + o] = (float)acc[g];
  }
}

}  // namespace

ZB_API int zb_istft_twiddles(int n, double* out, cudaStream_t stream) {
  ZB_REQUIRE(n >= 2 && n <= kMaxN && out, "istft_twiddles: n=%d (2..%d) or null output", n, kMaxN);
  ZB_REQUIRE_ALIGNED(out, 16, "istft_twiddles out");
  ZB_CUDA(zb::launch(istft_twiddle_kernel, dim3((unsigned)((n + 255) / 256)), dim3(256), 0, stream, 1, n,
                     reinterpret_cast<double2*>(out)));
  return zb::check_launch("istft_twiddles");
}

ZB_API int zb_istft_head_push(const void* y0, const void* y1, int y_is_f64, int streams, int cols, int n0, int n1,
                              int hop, const double* window0, const double* window1, const double* twiddle0,
                              const double* twiddle1, double max_log_mag, const double* mixer, int taps,
                              double* carry0, double* carry1, int carry_parity, double* ring0, double* ring1,
                              int ring_size, int64_t frames_before, int64_t mix_from, int64_t mix_to, int flush,
                              double* scratch, int64_t scratch_elems, float* out, cudaStream_t stream) {
  const int ns[2] = {n0, n1};
  ZB_REQUIRE(streams >= 1 && cols >= 0 && hop >= 1 && frames_before >= 0,
             "istft_head_push: streams=%d cols=%d hop=%d frames_before=%lld", streams, cols, hop,
             (long long)frames_before);
  for (int b = 0; b < 2; ++b) {
    ZB_REQUIRE(ns[b] % 2 == 0 && ns[b] % hop == 0 && ns[b] / hop >= 2,
               "istft_head_push: n_fft %d must be even and a multiple (>= 2) of the hop %d", ns[b], hop);
    if (ns[b] > kMaxN) return zb::fail(zb::kUnsupported, "istft_head_push: n_fft %d above %d", ns[b], kMaxN);
  }
  ZB_REQUIRE(taps >= 1 && taps % 2 == 1 && taps <= kMaxTaps, "istft_head_push: mixer taps %d (odd, <= %d)", taps,
             kMaxTaps);
  ZB_REQUIRE(ring_size >= 1 && (ring_size & (ring_size - 1)) == 0, "istft_head_push: ring %d not a power of two",
             ring_size);
  ZB_REQUIRE(flush ? cols == 0 : cols >= 1, "istft_head_push: a flush pushes no frames, a push at least one");
  ZB_REQUIRE(mix_from >= 0 && mix_to >= mix_from, "istft_head_push: mixer range [%lld, %lld)", (long long)mix_from,
             (long long)mix_to);
  ZB_REQUIRE(window0 && window1 && twiddle0 && twiddle1 && mixer && carry0 && carry1 && ring0 && ring1,
             "istft_head_push: null state pointer");
  ZB_REQUIRE(carry_parity == 0 || carry_parity == 1, "istft_head_push: carry parity %d", carry_parity);
  const int h = (taps - 1) / 2;
  const int64_t L = (frames_before + cols) * (int64_t)hop;
  // every mixer input the mixer reads must still be in the ring: the newest index written is below
  // h + L - min(n)/2 (the flush writes nothing past h + L)
  const int64_t newest = flush ? h + L : h + L - std::min(n0, n1) / 2;
  ZB_REQUIRE(newest - mix_from <= ring_size,
             "istft_head_push: ring of %d samples cannot hold mixer inputs [%lld, %lld)", ring_size,
             (long long)mix_from, (long long)newest);
  if (!flush) {
    ZB_REQUIRE(y0 && y1 && scratch, "istft_head_push: null frames or scratch");
    ZB_REQUIRE(scratch_elems >= (int64_t)streams * cols * (n0 + n1), "istft_head_push: scratch of %lld < %lld",
               (long long)scratch_elems, (long long)streams * cols * (n0 + n1));
    ZB_REQUIRE_ALIGNED(scratch, 16, "istft_head_push scratch");
    ZB_REQUIRE_ALIGNED(window0, 16, "istft_head_push window0");
    ZB_REQUIRE_ALIGNED(window1, 16, "istft_head_push window1");
    ZB_REQUIRE_ALIGNED(twiddle0, 16, "istft_head_push twiddle0");
    ZB_REQUIRE_ALIGNED(twiddle1, 16, "istft_head_push twiddle1");
    FrameParams fp{};
    const void* ys[2] = {y0, y1};
    const double* wins[2] = {window0, window1};
    const double* tws[2] = {twiddle0, twiddle1};
    double* outs[2] = {scratch, scratch + (int64_t)streams * cols * n0};
    for (int b = 0; b < 2; ++b) {
      fp.br[b].y = ys[b];
      fp.br[b].window = wins[b];
      fp.br[b].twiddle = reinterpret_cast<const double2*>(tws[b]);
      fp.br[b].out = outs[b];
      fp.br[b].n = ns[b];
      fp.br[b].nstages = radix_plan(ns[b] / 2, fp.br[b].radix);
      if (fp.br[b].nstages < 0) return zb::fail(zb::kUnsupported, "istft_head_push: n_fft %d has too many factors", ns[b]);
    }
    fp.frames = streams * cols;
    fp.y_f64 = y_is_f64 != 0;
    fp.max_log_mag = max_log_mag;
    const size_t smem = (size_t)(std::max(n0, n1) + 1) * sizeof(double2);
    ZB_CUDA(cudaFuncSetAttribute(istft_frames_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    ZB_CUDA(zb::launch(istft_frames_kernel, dim3((unsigned)(streams * cols), 2), dim3(kFrameThreads), smem, stream, 1,
                       fp));
    if (int rc = zb::check_launch("istft_frames")) return rc;
  }
  OlaParams op{};
  double* carries[2] = {carry0, carry1};
  double* rings[2] = {ring0, ring1};
  const double* wins[2] = {window0, window1};
  int64_t span = 0;
  for (int b = 0; b < 2; ++b) {
    const int64_t c = ns[b] - hop;
    op.br[b].frames = scratch ? scratch + (b ? (int64_t)streams * cols * n0 : 0) : nullptr;
    op.br[b].window = wins[b];
    op.br[b].carry_in = carries[b] + (int64_t)carry_parity * streams * c;
    op.br[b].carry_out = carries[b] + (int64_t)(1 - carry_parity) * streams * c;
    op.br[b].ring = rings[b];
    op.br[b].n = ns[b];
    span = std::max(span, flush ? c : (int64_t)cols * hop + c);
  }
  op.streams = streams;
  op.cols = cols;
  op.hop = hop;
  op.h = h;
  op.frames_before = frames_before;
  op.keep = h + L;
  op.ring_mask = ring_size - 1;
  op.flush = flush != 0;
  ZB_CUDA(zb::launch(istft_ola_kernel, dim3((unsigned)((span + 255) / 256), (unsigned)streams, 2), dim3(256), 0, stream,
                     1, op));
  if (int rc = zb::check_launch("istft_ola")) return rc;
  if (mix_to == mix_from) return zb::kOk;
  ZB_REQUIRE(out, "istft_head_push: null output");
  MixParams mp{ring0, ring1, mixer, out, mix_from, mix_to, flush ? h + L : INT64_MAX, taps, ring_size - 1};
  const size_t msmem = (size_t)(2 * taps + 2 * (kMixTile + taps - 1)) * sizeof(double);
  ZB_CUDA(cudaFuncSetAttribute(istft_mix_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)msmem));
  ZB_CUDA(zb::launch(istft_mix_kernel, dim3((unsigned)((mix_to - mix_from + kMixTile - 1) / kMixTile), (unsigned)streams),
                     dim3(kMixTile), msmem, stream, 1, mp));
  return zb::check_launch("istft_mix");
}

ZB_API int zb_resample_push(const void* x, int x_is_f64, int64_t x_stride, int streams, int count, double* ring,
                            int ring_size, int64_t n_in_before, const double* kernel_t, int orig, int new_freq,
                            int width, int64_t block_from, int64_t block_to, int64_t out_count, float* out,
                            cudaStream_t stream) {
  ZB_REQUIRE(streams >= 1 && count >= 0 && n_in_before >= 0 && orig >= 1 && new_freq >= 1 && width >= 0,
             "resample_push: streams=%d count=%d orig=%d new=%d width=%d", streams, count, orig, new_freq, width);
  ZB_REQUIRE(ring && kernel_t, "resample_push: null ring or kernel");
  ZB_REQUIRE(ring_size >= 1 && (ring_size & (ring_size - 1)) == 0, "resample_push: ring %d not a power of two",
             ring_size);
  ZB_REQUIRE(block_from >= 0 && block_to >= block_from && out_count >= 0 &&
                 out_count <= (block_to - block_from) * (int64_t)new_freq,
             "resample_push: blocks [%lld, %lld) with %lld outputs", (long long)block_from, (long long)block_to,
             (long long)out_count);
  const int kl = 2 * width + orig;
  const size_t smem = (size_t)kResPairs * kl * sizeof(double);
  if (smem > 227 * 1024) return zb::fail(zb::kUnsupported, "resample_push: kernel of %d taps too long", kl);
  const int64_t n_in = n_in_before + count;
  if (count > 0) {
    ZB_REQUIRE(x && x_stride >= count, "resample_push: null input or row stride %lld < %d", (long long)x_stride,
               count);
    // this call's samples, and every earlier one a window of this call reads, must fit the ring together
    const int64_t oldest = std::min(n_in_before, std::max<int64_t>(0, block_from * orig - width));
    ZB_REQUIRE(n_in - oldest <= ring_size, "resample_push: ring of %d cannot hold inputs [%lld, %lld)", ring_size,
               (long long)oldest, (long long)n_in);
    AppendParams ap{x, x_stride, x_is_f64 != 0, count, ring, ring_size - 1, n_in_before};
    ZB_CUDA(zb::launch(resample_append_kernel, dim3((unsigned)((count + 255) / 256), (unsigned)streams), dim3(256), 0,
                       stream, 1, ap));
    if (int rc = zb::check_launch("resample_append")) return rc;
  }
  if (out_count == 0) return zb::kOk;
  ZB_REQUIRE(out, "resample_push: null output");
  ZB_REQUIRE(n_in - std::max<int64_t>(0, block_from * orig - width) <= ring_size,
             "resample_push: ring of %d cannot hold the windows from block %lld", ring_size, (long long)block_from);
  ResampleParams rp{};
  rp.ring = ring;
  rp.kernel_t = kernel_t;
  rp.out = out;
  rp.n_in = n_in;
  rp.block_from = block_from;
  rp.out_count = out_count;
  rp.nblocks = (int)(block_to - block_from);
  rp.streams = streams;
  rp.orig = orig;
  rp.nnew = new_freq;
  rp.width = width;
  rp.kl = kl;
  rp.ring_mask = ring_size - 1;
  const int64_t pairs = (int64_t)streams * rp.nblocks;
  ZB_CUDA(cudaFuncSetAttribute(resample_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  ZB_CUDA(zb::launch(resample_kernel,
                     dim3((unsigned)((new_freq + kResThreads - 1) / kResThreads), (unsigned)((pairs + kResPairs - 1) / kResPairs)),
                     dim3(kResThreads), smem, stream, 1, rp));
  return zb::check_launch("resample");
}

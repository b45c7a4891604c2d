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
//   istft_frames_group_kernel / istft_group_seams_kernel   pushes of 32 frames or more: a CTA per group of 16+
//                         frames synthesises them in turn and overlap-adds them itself (an L2-resident span), so the
//                         frames never round-trip through HBM; a second kernel joins the groups' overlapping edges.
//   istft_mix_kernel      the K-tap correlation over both branches' rings, 8 consecutive outputs per thread.
//   resample_append_kernel / resample_kernel   the resampler's input ring, then out[b*new + i] =
//                         sum_k kernel[i][k] * x[b*orig + k - width] as a tiled float64 GEMM over (stream, block)
//                         pairs x output phases (the input windows gathered from the ring while the tiles stage).
#include <algorithm>
#include <vector>

#include "common.cuh"

namespace {

constexpr int kMaxStages = 24;
constexpr int kFrameThreads = 256;
constexpr int kMaxN = 8192;  // (n + 1) complex float64 values of shared memory per frame CTA

struct FrameBranch {
  const void* y;           // [streams][cols][n + 2] float32 or float64 (stream stride y_stride): log-magnitude for
                           // n/2 + 1 bins, then phase
  int64_t y_stride;
  const double* window;    // [n]
  const double2* twiddle;  // [n]: e^{2 pi i e / n}
  double* out;             // [frames, n] windowed frames
  int n;
  int nstages;
  int radix[kMaxStages];
  uint32_t ns_magic[kMaxStages];  // ceil(2^32 / Ns) of each pass (0 when Ns = 1): j / Ns = umulhi(j, magic), j < 2^16
};

struct FrameParams {
  FrameBranch br[2];
  int first;  // branch of blockIdx.y == 0: the longer n_fft, so its (slower) CTAs are dispatched first
  int cols;
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

__device__ __forceinline__ double2 cadd(double2 a, double2 b) { return make_double2(a.x + b.x, a.y + b.y); }
__device__ __forceinline__ double2 csub(double2 a, double2 b) { return make_double2(a.x - b.x, a.y - b.y); }

// Roots of unity (cos, sin)(2 pi k / R), k < R, as compile-time constants: Taylor series of cos and sin on arguments
// reduced to [-pi/2, pi/2] (cos x = -cos(x - pi), sin x = -sin(x - pi)); within a few float64 ulps.
constexpr double kPi = 3.14159265358979323846264338327950288;

constexpr double taylor_cos(double x) {
  double term = 1.0, sum = 1.0;
  for (int k = 1; k <= 14; ++k) {
    term *= -x * x / ((2.0 * k - 1.0) * (2.0 * k));
    sum += term;
  }
  return sum;
}

constexpr double taylor_sin(double x) {
  double term = x, sum = x;
  for (int k = 1; k <= 14; ++k) {
    term *= -x * x / ((2.0 * k) * (2.0 * k + 1.0));
    sum += term;
  }
  return sum;
}

template <int R>
struct UnitRoots {
  double c[R];
  double s[R];
  constexpr UnitRoots() : c(), s() {
    for (int k = 0; k < R; ++k) {
      double a = 2.0 * kPi * k / R;  // [0, 2 pi)
      if (a > kPi) a -= 2.0 * kPi;   // (-pi, pi]
      const double sign = (a > kPi / 2 || a < -kPi / 2) ? -1.0 : 1.0;
      const double r = a > kPi / 2 ? a - kPi : (a < -kPi / 2 ? a + kPi : a);
      c[k] = sign * taylor_cos(r);
      s[k] = sign * taylor_sin(r);
    }
  }
};

// Length-R inverse DFTs (out[q * stride] = sum_r x_r e^{2 pi i r q / R}) of one Stockham butterfly.
__device__ __forceinline__ void dft2_store(double2 x0, double2 x1, double2* out, int stride) {
  out[0] = cadd(x0, x1);
  out[stride] = csub(x0, x1);
}

__device__ __forceinline__ void dft4_store(double2 x0, double2 x1, double2 x2, double2 x3, double2* out, int stride) {
  const double2 a = cadd(x0, x2), b = csub(x0, x2), c = cadd(x1, x3), d = csub(x1, x3);
  out[0] = cadd(a, c);
  out[2 * stride] = csub(a, c);
  out[stride] = make_double2(b.x - d.y, b.y + d.x);      // b + i d
  out[3 * stride] = make_double2(b.x + d.y, b.y - d.x);  // b - i d
}

// One Stockham pass of radix R over M points (Ns = product of the radices before it): butterfly j reads
// src[j + r M/R], multiplies input r by W^(r (j mod Ns) M/(Ns R)) (W = e^{2 pi i / M}, the table's entry 2 r b; r b < M
// because j mod Ns < Ns), takes the length-R inverse DFT and writes output q to (j / Ns) Ns R + (j mod Ns) + q Ns.
//
// Odd R pairs the inputs: with u_r = x_r + x_{R-r}, v_r = x_r - x_{R-r} (r = 1..H, H = (R - 1) / 2),
//   y_q = x_0 + sum_r u_r cos(2 pi r q / R) + i sum_r v_r sin(2 pi r q / R),  y_{R-q} the same with -i,
// so a pair of outputs costs 4H multiply-adds.
template <int R>
__device__ __forceinline__ void stockham_pass(const double2* src, double2* dst, int M, int Ns, uint32_t magic,
                                              const double2* tw) {
  const int MR = M / R;
  const int span = M / (Ns * R);
  for (int j = threadIdx.x; j < MR; j += blockDim.x) {
    const int jq = magic ? (int)__umulhi((unsigned)j, magic) : j, jn = j - jq * Ns;
    const int b = jn * span;
    double2* out = dst + jq * Ns * R + jn;
    auto input = [&](int r) {
      const double2 v = src[j + r * MR];
      return (r == 0 || b == 0) ? v : cmul(v, __ldg(tw + 2 * r * b));
    };
    if constexpr (R == 2) {
      dft2_store(input(0), input(1), out, Ns);
    } else if constexpr (R == 4) {
      dft4_store(input(0), input(1), input(2), input(3), out, Ns);
    } else {
      static_assert(R % 2 == 1, "odd radix");
      constexpr int H = (R - 1) / 2;
      const double2 x0 = src[j];
      static_assert(H <= 3, "radices above 7 take odd_first_pass or generic_pass");
      constexpr UnitRoots<R> w{};
      double2 A[H], B[H];
      double2 y0 = x0;
#pragma unroll
      for (int g = 0; g < H; ++g) A[g] = x0, B[g] = make_double2(0.0, 0.0);
#pragma unroll
      for (int r = 1; r <= H; ++r) {
        const double2 a = input(r), c = input(R - r);
        const double2 u = cadd(a, c), v = csub(a, c);
        y0 = cadd(y0, u);
#pragma unroll
        for (int g = 0; g < H; ++g) {
          const double cs = w.c[(r * (g + 1)) % R], sn = w.s[(r * (g + 1)) % R];
          A[g].x = fma(u.x, cs, A[g].x);
          A[g].y = fma(u.y, cs, A[g].y);
          B[g].x = fma(v.x, sn, B[g].x);
          B[g].y = fma(v.y, sn, B[g].y);
        }
      }
      out[0] = y0;
#pragma unroll
      for (int g = 0; g < H; ++g) {
        out[(g + 1) * Ns] = make_double2(A[g].x - B[g].y, A[g].y + B[g].x);
        out[(R - g - 1) * Ns] = make_double2(A[g].x + B[g].y, A[g].y - B[g].x);
      }
    }
  }
}

// The first pass (Ns = 1, so no twiddles) of a large odd radix R: each butterfly's H = (R - 1) / 2 output pairs are
// split into groups of G, one (group, butterfly) item per thread, so that ceil(H / G) * M / R items rather than M / R
// butterflies spread over the block. Items run group-major with the butterflies of a group padded to whole warps, so
// a warp's group is uniform and its roots are compile-time constants (odd_first_group<g>). An item reads butterfly
// j's R inputs from shared memory, forms u_r, v_r and accumulates its G pairs (y_q = x_0 + sum_r u_r cos + i sum_r
// v_r sin, y_{R-q} with -i; group 0 also y_0 = x_0 + sum_r u_r); outputs go to j R + q.
template <int R, int G, int g>
__device__ __forceinline__ void odd_first_group(const double2* src, double2* dst, int MR, int j) {
  constexpr int H = (R - 1) / 2;
  constexpr int q0 = 1 + g * G;
  constexpr UnitRoots<R> w{};
  const double2 x0 = src[j];
  double2 A[G], B[G];
#pragma unroll
  for (int k = 0; k < G; ++k) A[k] = x0, B[k] = make_double2(0.0, 0.0);
  double2 y0 = x0;
#pragma unroll
  for (int r = 1; r <= H; ++r) {
    const double2 a = src[j + r * MR], c = src[j + (R - r) * MR];
    const double2 u = cadd(a, c), v = csub(a, c);
    if (g == 0) y0 = cadd(y0, u);
#pragma unroll
    for (int k = 0; k < G; ++k) {
      if (q0 + k <= H) {
        const double cs = w.c[(r * (q0 + k)) % R], sn = w.s[(r * (q0 + k)) % R];
        A[k].x = fma(u.x, cs, A[k].x);
        A[k].y = fma(u.y, cs, A[k].y);
        B[k].x = fma(v.x, sn, B[k].x);
        B[k].y = fma(v.y, sn, B[k].y);
      }
    }
  }
  double2* out = dst + j * R;
  if (g == 0) out[0] = y0;
#pragma unroll
  for (int k = 0; k < G; ++k) {
    const int q = q0 + k;
    if (q <= H) {
      out[q] = make_double2(A[k].x - B[k].y, A[k].y + B[k].x);
      out[R - q] = make_double2(A[k].x + B[k].y, A[k].y - B[k].x);
    }
  }
}

template <int R, int G>
__device__ __forceinline__ void odd_first_pass(const double2* src, double2* dst, int M) {
  constexpr int H = (R - 1) / 2;
  constexpr int NG = (H + G - 1) / G;
  static_assert(NG <= 4, "odd_first_pass dispatches at most four groups");
  const int MR = M / R;
  const int MRp = (MR + 31) & ~31;  // butterflies of a group, padded to whole warps
  for (int item = threadIdx.x; item < NG * MRp; item += blockDim.x) {
    const int g = item / MRp, j = item - g * MRp;
    if (j >= MR) continue;
    switch (g) {  // uniform within a warp
      case 0: odd_first_group<R, G, 0>(src, dst, MR, j); break;
      case 1: if constexpr (NG > 1) odd_first_group<R, G, 1>(src, dst, MR, j); break;
      case 2: if constexpr (NG > 2) odd_first_group<R, G, 2>(src, dst, MR, j); break;
      default: if constexpr (NG > 3) odd_first_group<R, G, 3>(src, dst, MR, j); break;
    }
  }
}

// Any other radix: each output summed directly, the powers W^(r s) by recurrence re-anchored on the table every 16
// terms (output q of butterfly j is sum_r src[j + r M/R] W^(r s), s = (j mod Ns) M/(Ns R) + q M/R).
__device__ void generic_pass(const double2* src, double2* dst, int M, int Ns, int R, const double2* tw) {
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
}

// Windowed inverse real DFT of one head frame of one branch (stream_host.py:55-63):
//   X[k] = exp(min(lm_k, max_log_mag)) * (cos ph_k, sin ph_k), imaginary parts of bins 0 and n/2 zeroed;
//   x[t] = (1/n) sum_{k<n} X[k] w^{kt} with the Hermitian extension, w = e^{2 pi i / n};  frame = x * window.
// With M = n/2: z[m] = x[2m] + i x[2m+1] = (1/n) sum_{k<M} Z[k] W^{km}, W = w^2, where
//   Z[k] = (X[k] + conj X[M-k]) + i w^k (X[k] - conj X[M-k]).
// The length-M inverse DFT runs one Stockham pass per radix R of M's factorisation (stockham_pass: radices 2, 3, 4,
// 5 and 7 as unrolled butterflies with compile-time roots; odd_first_pass for a leading 23; generic_pass for any
// other factor).
// Synthesises head frame `frame` (= stream * cols + column) of branch b in shared memory (sm: (n + 1) complex values);
// returns the buffer that holds z[m] = n (x[2m] + i x[2m+1]) (the caller applies 1/n and the window). Ends with a
// block barrier.
__device__ __forceinline__ const double2* synth_frame(const FrameParams& p, const FrameBranch& b, int64_t frame,
                                                      double2* sm) {
  const int n = b.n, M = n / 2, bins = M + 1;
  double2* X = sm;          // [M + 1], later the second Stockham buffer
  double2* A = sm + M + 1;  // [M]
  const double2* tw = b.twiddle;
  const int64_t row_off = (frame / p.cols) * b.y_stride + (frame % p.cols) * (n + 2);
  auto bin = [&](int k) {  // X[k] = exp(min(lm, max)) (cos ph, sin ph), imaginary part zero at DC and Nyquist
    double lm, ph;
    if (p.y_f64) {
      const double* row = static_cast<const double*>(b.y) + row_off;
      lm = row[k];
      ph = row[bins + k];
    } else {
      const float* row = static_cast<const float*>(b.y) + row_off;
      lm = (double)row[k];
      ph = (double)row[bins + k];
    }
    const double mag = exp(fmin(lm, p.max_log_mag));
    double s, c;
    sincos(ph, &s, &c);
    return make_double2(mag * c, (k == 0 || k == M) ? 0.0 : mag * s);
  };
  // thread k forms the pair (k, M - k) of the packed spectrum from bins k and M - k:
  //   Z[k] = (X[k] + conj X[M-k]) + i w^k (X[k] - conj X[M-k]), and the same with k and M - k exchanged
  for (int k = threadIdx.x; k <= M / 2; k += blockDim.x) {
    const double2 xk = bin(k), xc = bin(M - k);
    {
      const double2 e = make_double2(xk.x + xc.x, xk.y - xc.y);
      const double2 d = make_double2(xk.x - xc.x, xk.y + xc.y);
      const double2 o = cmul(__ldg(tw + k), d);
      A[k] = make_double2(e.x - o.y, e.y + o.x);
    }
    if (k != 0 && 2 * k != M) {
      const double2 e = make_double2(xc.x + xk.x, xc.y - xk.y);
      const double2 d = make_double2(xc.x - xk.x, xc.y + xk.y);
      const double2 o = cmul(__ldg(tw + (M - k)), d);
      A[M - k] = make_double2(e.x - o.y, e.y + o.x);
    }
  }
  __syncthreads();

  double2* src = A;
  double2* dst = X;
  int Ns = 1;
  for (int st = 0; st < b.nstages; ++st) {
    const int R = b.radix[st];
    if (R == 23 && Ns == 1) {
      odd_first_pass<23, 3>(src, dst, M);
    } else {
      switch (R) {
        case 2: stockham_pass<2>(src, dst, M, Ns, b.ns_magic[st], tw); break;
        case 3: stockham_pass<3>(src, dst, M, Ns, b.ns_magic[st], tw); break;
        case 4: stockham_pass<4>(src, dst, M, Ns, b.ns_magic[st], tw); break;
        case 5: stockham_pass<5>(src, dst, M, Ns, b.ns_magic[st], tw); break;
        case 7: stockham_pass<7>(src, dst, M, Ns, b.ns_magic[st], tw); break;
        default: generic_pass(src, dst, M, Ns, R, tw); break;
      }
    }
    __syncthreads();
    double2* tmp = src;
    src = dst;
    dst = tmp;
    Ns *= R;
  }
  return src;
}

__global__ void __launch_bounds__(kFrameThreads, 4) istft_frames_kernel(FrameParams p) {
  zb::pdl_enter();
  const FrameBranch& b = p.br[blockIdx.y ^ p.first];
  const int n = b.n, M = n / 2;
  const int64_t frame = blockIdx.x;
  extern __shared__ double2 sm[];
  const double2* z = synth_frame(p, b, frame, sm);
  const double inv_n = 1.0 / (double)n;
  double* out = b.out + frame * n;
  for (int m = threadIdx.x; m < M; m += blockDim.x) {
    const double2 v = z[m];
    const double2 win = *reinterpret_cast<const double2*>(b.window + 2 * m);
    *reinterpret_cast<double2*>(out + 2 * m) = make_double2(v.x * inv_n * win.x, v.y * inv_n * win.y);
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

// A final overlap-add position `pos` of a branch (stream_host.py:104-113): divided by the overlap-added squared window
// of frames max(0, ceil((pos - n + 1) / hop)) .. min(total - 1, pos / hop), written to the mixer input at
// h + pos - n/2 unless it is centre padding (pos < n/2) or, at flush, past what the mixer reads (index >= keep).
__device__ __forceinline__ void finalize_sample(int64_t pos, double v, const double* window, int n, int hop,
                                                int64_t total, int h, int64_t keep, double* ring, int ring_mask) {
  if (pos < n / 2) return;
  const int64_t idx = h + pos - n / 2;
  if (idx >= keep) return;
  const int64_t e_lo = ceil_div_pos(pos - n + 1, hop);
  const int64_t e_hi = min(total - 1, pos / hop);
  double env = 0.0;
  for (int64_t c = e_lo; c <= e_hi; ++c) {
    const double w = window[pos - c * hop];
    env += w * w;
  }
  ring[idx & ring_mask] = v / env;
}


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
    finalize_sample(pos, v, b.window, n, hop, p.frames_before + p.cols, p.h, p.flush ? p.keep : INT64_MAX,
                    b.ring + (int64_t)s * (p.ring_mask + 1), p.ring_mask);
  } else {
    b.carry_out[(int64_t)s * carry + (pos - P1)] = v;
  }
}

constexpr int kGroupFrames = 16;  // frames a group CTA overlap-adds itself (>= (n - hop) / hop of the codec's branches)

struct GroupBranch {
  double* acc;           // [streams, ngroups, acc_len]: each group's overlap-add span
  const double* window;  // [n]
  const double* carry_in;  // [streams, n - hop]
  double* carry_out;       // [streams, n - hop]
  double* ring;            // [streams, ring]
};

struct GroupParams {
  FrameParams f;
  GroupBranch g[2];
  int64_t acc_len;  // doubles per group span (even)
  int ngroups;      // groups per stream: frames [g * kGroupFrames, ...), the last one takes the remainder
  int hop, h;
  int64_t frames_before;
  int ring_mask;
};

__device__ __forceinline__ int group_begin(int g) { return g * kGroupFrames; }
__device__ __forceinline__ int group_end(const GroupParams& p, int g) {
  return g == p.ngroups - 1 ? p.f.cols : (g + 1) * kGroupFrames;
}

// A long push without the frame scratch round trip: one CTA per (stream, group of >= 16 consecutive frames, branch)
// synthesises its frames in order (synth_frame) and overlap-adds each windowed frame into its group's span
// [0, size hop + n - hop) of a global accumulator (written, then read back, by this CTA alone, so it stays in L2);
// the frames of the group are the only contributors to [n - hop, size hop), which it finalises itself. The first
// n - hop positions (the previous group's tail or the carried sums overlap there) and the last n - hop ones are left
// to istft_group_seams_kernel.
__global__ void __launch_bounds__(kFrameThreads, 4) istft_frames_group_kernel(GroupParams p) {
  zb::pdl_enter();
  const FrameBranch& b = p.f.br[blockIdx.y ^ p.f.first];
  const GroupBranch& gb = p.g[blockIdx.y ^ p.f.first];
  const int n = b.n, M = n / 2, hop = p.hop;
  const int s = blockIdx.x / p.ngroups, g = blockIdx.x - s * p.ngroups;
  const int c0 = group_begin(g), size = group_end(p, g) - c0;
  double* span = gb.acc + (int64_t)blockIdx.x * p.acc_len;
  extern __shared__ double2 sm[];
  const double inv_n = 1.0 / (double)n;
  for (int i = 0; i < size; ++i) {
    const double2* z = synth_frame(p.f, b, (int64_t)s * p.f.cols + c0 + i, sm);
    double* dst = span + (int64_t)i * hop;
    for (int m = threadIdx.x; m < M; m += blockDim.x) {
      const double2 v = z[m];
      const double2 win = *reinterpret_cast<const double2*>(b.window + 2 * m);
      double2 add = make_double2(v.x * inv_n * win.x, v.y * inv_n * win.y);
      if (i > 0 && 2 * m < n - hop) {  // already holds the earlier frames of the group
        const double2 old = *reinterpret_cast<const double2*>(dst + 2 * m);
        add.x += old.x;
        add.y += old.y;
      }
      *reinterpret_cast<double2*>(dst + 2 * m) = add;
    }
    __syncthreads();  // the span's updates are visible, and shared memory is free, before the next frame
  }
  const int64_t P0 = (p.frames_before + c0) * hop;
  const int64_t total = p.frames_before + p.f.cols;
  double* ring = gb.ring + (int64_t)s * (p.ring_mask + 1);
  for (int t = n - hop + threadIdx.x; t < size * hop; t += blockDim.x)
    finalize_sample(P0 + t, span[t], gb.window, n, hop, total, p.h, INT64_MAX, ring, p.ring_mask);
}

// The seams of a grouped push, one thread per position: seam 0 = the carried sums + group 0's first n - hop
// positions; seam g = group g-1's last n - hop + group g's first n - hop; both final. Seam ngroups = the last group's
// last n - hop positions, the next push's carry.
__global__ void __launch_bounds__(256) istft_group_seams_kernel(GroupParams p) {
  zb::pdl_enter();
  const GroupBranch& gb = p.g[blockIdx.z];
  const int n = p.f.br[blockIdx.z].n, hop = p.hop, carry = n - hop;
  const int s = blockIdx.y;
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (int64_t)(p.ngroups + 1) * carry) return;
  const int seam = (int)(idx / carry), t = (int)(idx - (int64_t)seam * carry);
  const double* acc = gb.acc + (int64_t)s * p.ngroups * p.acc_len;
  if (seam == p.ngroups) {
    const int g = p.ngroups - 1;
    const int size = group_end(p, g) - group_begin(g);
    gb.carry_out[(int64_t)s * carry + t] = acc[(int64_t)g * p.acc_len + (int64_t)size * hop + t];
    return;
  }
  double v = acc[(int64_t)seam * p.acc_len + t];
  if (seam == 0) {
    v += gb.carry_in[(int64_t)s * carry + t];
  } else {
    const int size = group_end(p, seam - 1) - group_begin(seam - 1);
    v += acc[(int64_t)(seam - 1) * p.acc_len + (int64_t)size * hop + t];
  }
  const int64_t pos = (p.frames_before + group_begin(seam)) * hop + t;
  finalize_sample(pos, v, gb.window, n, hop, p.frames_before + p.f.cols, p.h, INT64_MAX,
                  gb.ring + (int64_t)s * (p.ring_mask + 1), p.ring_mask);
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

constexpr int kMixOuts = 8;                       // consecutive outputs per thread
constexpr int kMixThreads = 128;
constexpr int kMixTile = kMixThreads * kMixOuts;  // outputs per CTA
constexpr int kMaxTaps = 1023;

// Shared-memory index of input i with one pad slot per 8: thread t reads 8t + c, which lands on 9t + c + c/8, an odd
// stride of doubles, so the lanes of a half-warp hit distinct bank pairs.
__device__ __forceinline__ int mix_pad(int i) { return i + (i >> 3); }

// y[m] = sum_c sum_k mixer[c][k] * in_c[m + k] for m in [mix_from, mix_to) (stream_host.py:115-127). A CTA stages its
// tile's inputs (kMixTile + K - 1 values of each branch, zero past what the tile needs) and the taps (zero-padded to a
// multiple of 8) in shared memory; a thread owns 8 consecutive outputs and, per 8 taps, reads 15 inputs of each branch
// once and applies all 8 taps to all 8 outputs from registers.
__global__ void __launch_bounds__(kMixThreads) istft_mix_kernel(MixParams p) {
  zb::pdl_enter();
  extern __shared__ double msm[];
  const int K = p.K;
  const int Kp = (K + 7) & ~7;
  const int width = kMixTile + Kp + 8;
  const int padded = mix_pad(width) + 1;
  double* taps = msm;         // [2][Kp]
  double* in0 = msm + 2 * Kp;  // [padded]
  double* in1 = in0 + padded;  // [padded]
  const int s = blockIdx.y;
  const int64_t m0 = p.mix_from + (int64_t)blockIdx.x * kMixTile;
  const int64_t ring = (int64_t)p.ring_mask + 1;
  for (int i = threadIdx.x; i < 2 * Kp; i += blockDim.x) {
    const int c = i / Kp, k = i - c * Kp;
    taps[i] = k < K ? p.mixer[c * K + k] : 0.0;
  }
  for (int i = threadIdx.x; i < width; i += blockDim.x) {
    const int64_t idx = m0 + i;
    const bool live = idx < p.limit && idx < p.mix_to + K - 1;
    in0[mix_pad(i)] = live ? p.ring0[s * ring + (idx & p.ring_mask)] : 0.0;
    in1[mix_pad(i)] = live ? p.ring1[s * ring + (idx & p.ring_mask)] : 0.0;
  }
  __syncthreads();
  const int base = threadIdx.x * kMixOuts;
  if (m0 + base >= p.mix_to) return;
  double acc[kMixOuts];
#pragma unroll
  for (int u = 0; u < kMixOuts; ++u) acc[u] = 0.0;
  for (int k0 = 0; k0 < Kp; k0 += 8) {
    double v0[15], v1[15];
#pragma unroll
    for (int i = 0; i < 15; ++i) {
      v0[i] = in0[mix_pad(base + k0 + i)];
      v1[i] = in1[mix_pad(base + k0 + i)];
    }
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      const double t0 = taps[k0 + kk], t1 = taps[Kp + k0 + kk];
#pragma unroll
      for (int u = 0; u < kMixOuts; ++u) {
        acc[u] = fma(t0, v0[u + kk], acc[u]);
        acc[u] = fma(t1, v1[u + kk], acc[u]);
      }
    }
  }
  float* out = p.out + (int64_t)s * (p.mix_to - p.mix_from) + (m0 - p.mix_from) + base;
  const int64_t left = p.mix_to - (m0 + base);
#pragma unroll
  for (int u = 0; u < kMixOuts; ++u)
    if (u < left) out[u] = (float)acc[u];
}

__global__ void istft_twiddle_kernel(int n, double2* out) {
  const int e = blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= n) return;
  double s, c;
  sincospi(2.0 * (double)e / (double)n, &s, &c);
  out[e] = make_double2(c, s);
}

// Radices of M: fours, then a two, then odd factors ascending; the largest moves to the front when it is above 7.
int radix_plan(int M, int* radix) {
  int k = 0;
  while (M % 4 == 0 && M > 4 && k < kMaxStages) radix[k++] = 4, M /= 4;
  while (M % 2 == 0 && M > 2 && k < kMaxStages) radix[k++] = 2, M /= 2;
  for (int f = 3; f * f <= M && k < kMaxStages; f += 2)
    while (M % f == 0 && M > f && k < kMaxStages) radix[k++] = f, M /= f;
  if (k < kMaxStages && M > 1) radix[k++] = M;
  if (k >= kMaxStages) return -1;
  // a factor above 7 runs first, where it needs no twiddles (odd_first_pass for 23, generic_pass otherwise)
  int big = 0;
  for (int i = 1; i < k; ++i)
    if (radix[i] > radix[big]) big = i;
  if (radix[big] > 7) std::swap(radix[0], radix[big]);
  return k;
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

constexpr int kResBM = 32;      // (stream, block) pairs per CTA
constexpr int kResBNMax = 128;  // output phases per CTA: 16 x TN (TN = 4 or 8 per thread)      // output phases per CTA
constexpr int kResBK = 16;      // taps per step
constexpr int kResThreads = 128;  // 8 x 16 threads, 4 x TN outputs each

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
  double* partial;  // split taps: [slices, streams * nblocks, new] per-slice sums (null: one slice, written directly)
  int kchunk;       // taps per slice (a multiple of kResBK)
};

// out[b * new + i] = sum_k kernel[i][k] * x[b * orig + k - width] (stream_host.py:145-171), inputs outside [0, n_in)
// zero, as a float64 GEMM C[pairs, new] = A[pairs, kl] K^T with the rows of A the input windows of the (stream,
// block) pairs, read from the ring as the tiles are staged. A CTA owns a 32-pair x 128-phase tile and walks the taps
// 16 at a time: the next step's A and K^T tiles are copied (cp.async, zero-filled outside the data) into the other
// shared-memory buffer while the current ones (A transposed) feed 4 x 8 outputs per thread. When few tiles would cover the GPU, the taps split into slices
// (blockIdx.z) whose sums resample_reduce_kernel adds in slice order, so the result does not depend on timing.
__device__ __forceinline__ void cp_async8(double* dst, const double* src, bool live) {
  // 8-byte global -> shared copy; a dead element copies nothing and zero-fills (src-size 0)
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;" ::"r"(zb::smem_addr(dst)), "l"(src),
               "r"(live ? 8 : 0)
               : "memory");
}

template <int TN>
__global__ void __launch_bounds__(kResThreads, TN == 4 ? 5 : 4) resample_kernel(ResampleParams p) {
  constexpr int kResBN = 16 * TN;
  zb::pdl_enter();
  __shared__ __align__(16) double As[2][kResBK][kResBM + 2];  // [buffer][tap][pair], padded rows
  __shared__ __align__(16) double Bs[2][kResBK][kResBN];  // [buffer][tap][phase]
  const int tid = threadIdx.x;
  const int64_t pair0 = (int64_t)blockIdx.y * kResBM;
  const int i0 = blockIdx.x * kResBN;
  const int64_t pairs_total = (int64_t)p.streams * p.nblocks;
  const int64_t ring = (int64_t)p.ring_mask + 1;

  // A staging: element e = tid + 128 u (u < 4) of the [32 pairs][16 taps] tile: pair e / 16, tap e % 16 (16 lanes
  // read 16 consecutive taps of one window)
  const int a_tap = tid % kResBK;
  int64_t a_row[4], a_start[4];
  bool a_live[4];
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    const int64_t pr = pair0 + (tid + kResThreads * u) / kResBK;
    a_live[u] = pr < pairs_total;
    const int64_t sidx = a_live[u] ? pr / p.nblocks : 0;
    const int64_t blk = p.block_from + (a_live[u] ? pr % p.nblocks : 0);
    a_row[u] = sidx * ring;
    a_start[u] = blk * p.orig - p.width;
  }
  // B staging: element e = tid + 128 u of the [16 taps][16 TN phases] tile: phase e % BN, tap e / BN
  constexpr int kBStep = kResThreads / kResBN;  // taps between a thread's consecutive elements
  const int b_col = tid % kResBN, b_tap0 = tid / kResBN;
  const bool b_live = i0 + b_col < p.nnew;
  const int k_begin = blockIdx.z * p.kchunk;
  const int k_end = min(p.kl, k_begin + p.kchunk);

  auto issue = [&](int k0, int buf) {
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int k = k0 + a_tap;
      const int64_t t = a_start[u] + k;
      const bool live = a_live[u] && k < k_end && t >= 0 && t < p.n_in;
      cp_async8(&As[buf][a_tap][(tid + kResThreads * u) / kResBK], live ? p.ring + a_row[u] + (t & p.ring_mask) : p.ring,
                live);
    }
#pragma unroll
    for (int u = 0; u < kResBK / kBStep; ++u) {
      const int tap = b_tap0 + kBStep * u;
      const int k = k0 + tap;
      const bool live = b_live && k < k_end;
      cp_async8(&Bs[buf][tap][b_col], live ? p.kernel_t + (int64_t)k * p.nnew + i0 + b_col : p.kernel_t, live);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };

  // thread (tr, tc): pairs tr*4 .. tr*4+3, phases 32 q + 2 tc + {0, 1} for q < TN / 2 (each fragment load is a
  // contiguous 16 bytes per lane, so a half-warp's 256 bytes hit every bank once)
  const int tr = tid / 16, tc = tid % 16;
  double acc[4][TN];
#pragma unroll
  for (int x = 0; x < 4; ++x)
#pragma unroll
    for (int y = 0; y < TN; ++y) acc[x][y] = 0.0;

  const int steps = (k_end - k_begin + kResBK - 1) / kResBK;
  issue(k_begin, 0);
  for (int st = 0; st < steps; ++st) {
    const int buf = st & 1;
    if (st + 1 < steps) {
      issue(k_begin + (st + 1) * kResBK, buf ^ 1);
      asm volatile("cp.async.wait_group 1;" ::: "memory");  // this step's group has landed
    } else {
      asm volatile("cp.async.wait_group 0;" ::: "memory");
    }
    __syncthreads();
#pragma unroll
    for (int k = 0; k < kResBK; ++k) {
      const double2 a01 = *reinterpret_cast<const double2*>(&As[buf][k][tr * 4]);
      const double2 a23 = *reinterpret_cast<const double2*>(&As[buf][k][tr * 4 + 2]);
      double bv[TN];
#pragma unroll
      for (int q = 0; q < TN / 2; ++q) {
        const double2 b = *reinterpret_cast<const double2*>(&Bs[buf][k][32 * q + tc * 2]);
        bv[2 * q] = b.x;
        bv[2 * q + 1] = b.y;
      }
      const double av[4] = {a01.x, a01.y, a23.x, a23.y};
#pragma unroll
      for (int x = 0; x < 4; ++x)
#pragma unroll
        for (int y = 0; y < TN; ++y) acc[x][y] = fma(av[x], bv[y], acc[x][y]);
    }
    __syncthreads();  // this buffer is refilled two steps on
  }
#pragma unroll
  for (int x = 0; x < 4; ++x) {
    const int64_t pr = pair0 + tr * 4 + x;
    if (pr >= pairs_total) break;
    if (p.partial) {
      double* dst = p.partial + ((int64_t)blockIdx.z * pairs_total + pr) * p.nnew;
#pragma unroll
      for (int y = 0; y < TN; ++y) {
        const int i = i0 + 32 * (y >> 1) + tc * 2 + (y & 1);
        if (i < p.nnew) dst[i] = acc[x][y];
      }
      continue;
    }
    const int64_t sidx = pr / p.nblocks;
    const int64_t o0 = (pr % p.nblocks) * p.nnew;
#pragma unroll
    for (int y = 0; y < TN; ++y) {
      const int i = i0 + 32 * (y >> 1) + tc * 2 + (y & 1);
      const int64_t o = o0 + i;
      if (i < p.nnew && o < p.out_count) p.out[sidx * p.out_count + o] = (float)acc[x][y];
    }
  }
}

// Sums the tap slices of resample_kernel in slice order: out[s, o] for o < out_count, o = (pair's block) * new + i.
__global__ void __launch_bounds__(256) resample_reduce_kernel(ResampleParams p, int slices) {
  zb::pdl_enter();
  const int64_t pairs_total = (int64_t)p.streams * p.nblocks;
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= pairs_total * p.nnew) return;
  const int64_t pr = idx / p.nnew;
  const int i = (int)(idx - pr * p.nnew);
  const int64_t sidx = pr / p.nblocks;
  const int64_t o = (pr % p.nblocks) * p.nnew + i;
  if (o >= p.out_count) return;
  double v = 0.0;
  for (int z = 0; z < slices; ++z) v += p.partial[((int64_t)z * pairs_total + pr) * p.nnew + i];
  p.out[sidx * p.out_count + o] = (float)v;
}

}  // namespace

ZB_API int zb_istft_twiddles(int n, double* out, cudaStream_t stream) {
  ZB_REQUIRE(n >= 2 && n <= kMaxN && out, "istft_twiddles: n=%d (2..%d) or null output", n, kMaxN);
  ZB_REQUIRE_ALIGNED(out, 16, "istft_twiddles out");
  ZB_CUDA(zb::launch(istft_twiddle_kernel, dim3((unsigned)((n + 255) / 256)), dim3(256), 0, stream, 1, n,
                     reinterpret_cast<double2*>(out)));
  return zb::check_launch("istft_twiddles");
}

ZB_API int zb_istft_head_push(const void* y0, int64_t y0_stride, const void* y1, int64_t y1_stride, int y_is_f64,
                              int streams, int cols, int n0, int n1,
                              int hop, const double* window0, const double* window1, const double* twiddle0,
                              const double* twiddle1, double max_log_mag, const double* mixer, int taps,
                              double* carry0, double* carry1, int carry_parity, double* ring0, double* ring1,
                              int ring_size, int64_t frames_before, int64_t mix_from, int64_t mix_to, int flush,
                              double* scratch, int64_t scratch_elems, float* out, cudaStream_t stream) {
  const int ns[2] = {n0, n1};
  ZB_REQUIRE(streams >= 1 && streams <= 65535 && cols >= 0 && hop >= 1 && frames_before >= 0,
             "istft_head_push: streams=%d (1..65535) cols=%d hop=%d frames_before=%lld", streams, cols, hop,
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
  // A push of at least two groups of frames overlap-adds in the frame CTAs (istft_frames_group_kernel) when the
  // scratch holds the groups' spans, the hop is even (16-byte accesses) and a group covers an n_fft; otherwise the
  // frames go through the scratch to istft_ola_kernel.
  const int ngroups = cols / kGroupFrames;
  const int64_t acc_len = ((int64_t)(2 * kGroupFrames - 1) * hop + std::max(n0, n1) - hop + 1) & ~(int64_t)1;
  const bool grouped = !flush && ngroups >= 2 && hop % 2 == 0 && std::max(n0, n1) <= (kGroupFrames + 1) * hop &&
                       scratch_elems >= 2 * (int64_t)streams * ngroups * acc_len;
  if (!flush) {
    ZB_REQUIRE(y0 && y1 && scratch, "istft_head_push: null frames or scratch");
    ZB_REQUIRE(grouped || scratch_elems >= (int64_t)streams * cols * (n0 + n1),
               "istft_head_push: scratch of %lld < %lld", (long long)scratch_elems,
               (long long)streams * cols * (n0 + n1));
    ZB_REQUIRE_ALIGNED(scratch, 16, "istft_head_push scratch");
    ZB_REQUIRE_ALIGNED(window0, 16, "istft_head_push window0");
    ZB_REQUIRE_ALIGNED(window1, 16, "istft_head_push window1");
    ZB_REQUIRE_ALIGNED(twiddle0, 16, "istft_head_push twiddle0");
    ZB_REQUIRE_ALIGNED(twiddle1, 16, "istft_head_push twiddle1");
    FrameParams fp{};
    const void* ys[2] = {y0, y1};
    const int64_t ystrides[2] = {y0_stride, y1_stride};
    const double* wins[2] = {window0, window1};
    const double* tws[2] = {twiddle0, twiddle1};
    double* outs[2] = {scratch, scratch + (int64_t)streams * cols * n0};
    for (int b = 0; b < 2; ++b) {
      ZB_REQUIRE(streams == 1 || ystrides[b] >= (int64_t)cols * (ns[b] + 2),
                 "istft_head_push: branch %d stream stride %lld below cols * (n + 2)", b, (long long)ystrides[b]);
      fp.br[b].y = ys[b];
      fp.br[b].y_stride = ystrides[b];
      fp.br[b].window = wins[b];
      fp.br[b].twiddle = reinterpret_cast<const double2*>(tws[b]);
      fp.br[b].out = outs[b];
      fp.br[b].n = ns[b];
      fp.br[b].nstages = radix_plan(ns[b] / 2, fp.br[b].radix);
      if (fp.br[b].nstages < 0) return zb::fail(zb::kUnsupported, "istft_head_push: n_fft %d has too many factors", ns[b]);
      for (int st = 0, Ns = 1; st < fp.br[b].nstages; Ns *= fp.br[b].radix[st++])
        fp.br[b].ns_magic[st] = Ns == 1 ? 0u : (uint32_t)(((1ull << 32) + Ns - 1) / Ns);
    }
    fp.first = n1 > n0 ? 1 : 0;
    fp.cols = cols;
    fp.y_f64 = y_is_f64 != 0;
    fp.max_log_mag = max_log_mag;
    const size_t smem = (size_t)(std::max(n0, n1) + 1) * sizeof(double2);
    if (grouped) {
      GroupParams gp{};
      gp.f = fp;
      double* carries[2] = {carry0, carry1};
      double* rings[2] = {ring0, ring1};
      for (int b = 0; b < 2; ++b) {
        const int64_t c = ns[b] - hop;
        gp.g[b].acc = scratch + (int64_t)b * streams * ngroups * acc_len;
        gp.g[b].window = wins[b];
        gp.g[b].carry_in = carries[b] + (int64_t)carry_parity * streams * c;
        gp.g[b].carry_out = carries[b] + (int64_t)(1 - carry_parity) * streams * c;
        gp.g[b].ring = rings[b];
      }
      gp.acc_len = acc_len;
      gp.ngroups = ngroups;
      gp.hop = hop;
      gp.h = h;
      gp.frames_before = frames_before;
      gp.ring_mask = ring_size - 1;
      ZB_CUDA(cudaFuncSetAttribute(istft_frames_group_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
      ZB_CUDA(zb::launch(istft_frames_group_kernel, dim3((unsigned)(streams * ngroups), 2), dim3(kFrameThreads), smem,
                         stream, 1, gp));
      if (int rc = zb::check_launch("istft_frames_group")) return rc;
      const int64_t seam_positions = (int64_t)(ngroups + 1) * (std::max(n0, n1) - hop);
      ZB_CUDA(zb::launch(istft_group_seams_kernel, dim3((unsigned)((seam_positions + 255) / 256), (unsigned)streams, 2),
                         dim3(256), 0, stream, 1, gp));
      if (int rc = zb::check_launch("istft_group_seams")) return rc;
    } else {
      ZB_CUDA(cudaFuncSetAttribute(istft_frames_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
      ZB_CUDA(zb::launch(istft_frames_kernel, dim3((unsigned)(streams * cols), 2), dim3(kFrameThreads), smem, stream,
                         1, fp));
      if (int rc = zb::check_launch("istft_frames")) return rc;
    }
  }
  if (!grouped) {
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
  }
  if (mix_to == mix_from) return zb::kOk;
  ZB_REQUIRE(out, "istft_head_push: null output");
  MixParams mp{ring0, ring1, mixer, out, mix_from, mix_to, flush ? h + L : INT64_MAX, taps, ring_size - 1};
  const int Kp = (taps + 7) & ~7;
  const int width = kMixTile + Kp + 8;
  const size_t msmem = (size_t)(2 * Kp + 2 * (width + (width >> 3) + 1)) * sizeof(double);
  ZB_CUDA(cudaFuncSetAttribute(istft_mix_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)msmem));
  ZB_CUDA(zb::launch(istft_mix_kernel, dim3((unsigned)((mix_to - mix_from + kMixTile - 1) / kMixTile), (unsigned)streams),
                     dim3(kMixThreads), msmem, stream, 1, mp));
  return zb::check_launch("istft_mix");
}

ZB_API int zb_resample_push(const void* x, int x_is_f64, int64_t x_stride, int streams, int count, double* ring,
                            int ring_size, int64_t n_in_before, const double* kernel_t, int orig, int new_freq,
                            int width, int64_t block_from, int64_t block_to, int64_t out_count, float* out,
                            double* workspace, int64_t workspace_elems, cudaStream_t stream) {
  ZB_REQUIRE(streams >= 1 && streams <= 65535 && count >= 0 && n_in_before >= 0 && orig >= 1 && new_freq >= 1 &&
                 width >= 0,
             "resample_push: streams=%d (1..65535) count=%d orig=%d new=%d width=%d", streams, count, orig, new_freq,
             width);
  ZB_REQUIRE(ring && kernel_t, "resample_push: null ring or kernel");
  ZB_REQUIRE(ring_size >= 1 && (ring_size & (ring_size - 1)) == 0, "resample_push: ring %d not a power of two",
             ring_size);
  ZB_REQUIRE(block_from >= 0 && block_to >= block_from && out_count >= 0 &&
                 out_count <= (block_to - block_from) * (int64_t)new_freq,
             "resample_push: blocks [%lld, %lld) with %lld outputs", (long long)block_from, (long long)block_to,
             (long long)out_count);
  const int kl = 2 * width + orig;
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
  ZB_REQUIRE((pairs + kResBM - 1) / kResBM < 65536, "resample_push: %lld (stream, block) pairs in one call",
             (long long)pairs);
  // 4 x 8 outputs per thread when the tiles cover the GPU several times over, else 4 x 4 (twice the CTAs); then
  // split the taps while the tiles alone would leave most of the GPU idle (four resample CTAs fit an SM)
  const int64_t pair_tiles = (pairs + kResBM - 1) / kResBM;
  const bool wide = pair_tiles * ((new_freq + kResBNMax - 1) / kResBNMax) >= 8 * zb::sm_count();
  const int bn = wide ? kResBNMax : kResBNMax / 2;
  const int64_t tiles = (int64_t)((new_freq + bn - 1) / bn) * pair_tiles;
  const int steps = (kl + kResBK - 1) / kResBK;
  int slices = (int)std::min<int64_t>({8, steps, std::max<int64_t>(1, 4 * zb::sm_count() / tiles)});
  if (!workspace || workspace_elems < (int64_t)slices * pairs * new_freq) slices = 1;
  rp.kchunk = (steps + slices - 1) / slices * kResBK;
  slices = (kl + rp.kchunk - 1) / rp.kchunk;
  rp.partial = slices > 1 ? workspace : nullptr;
  if (slices > 1) ZB_REQUIRE_ALIGNED(workspace, 16, "resample_push workspace");
  const dim3 rgrid((unsigned)((new_freq + bn - 1) / bn), (unsigned)pair_tiles, (unsigned)slices);
  if (wide) {
    ZB_CUDA(zb::launch(resample_kernel<8>, rgrid, dim3(kResThreads), 0, stream, 1, rp));
  } else {
    ZB_CUDA(zb::launch(resample_kernel<4>, rgrid, dim3(kResThreads), 0, stream, 1, rp));
  }
  if (int rc = zb::check_launch("resample")) return rc;
  if (slices == 1) return zb::kOk;
  const int64_t n = pairs * new_freq;
  ZB_CUDA(zb::launch(resample_reduce_kernel, dim3((unsigned)((n + 255) / 256)), dim3(256), 0, stream, 1, rp, slices));
  return zb::check_launch("resample_reduce");
}

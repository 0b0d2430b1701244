// spectral_kernels.cuh — fused segment -> window -> detrend -> FFT -> spectrum
// kernels for welch / csd / spectrogram / stft (sm_100a).
//
// Framing follows the reference frontend (src/ops/signal/spectral_analysis.cpp):
//   step = nperseg - noverlap, n_seg = (n - nperseg)/step + 1 (tail dropped),
//   segment s covers samples [s*step, s*step + nperseg)            (:124,:133)
//   x_w = x_seg * win (in the input dtype)                          (:75-76)
//   constant detrend subtracts mean(x_w) after windowing            (:79-82)
//   X = FFT_nfft(x_w) (zero padded to nfft)                         (:90-91)
//   csd/welch accumulate Re(conj(X) * Y) over segments in F64        (:93-148)
//   spectrogram/stft store per-segment columns                      (:258-300)
//
// Two real sequences share one complex transform: Z = FFT(a + i*b), then
//   A[k] = (Z[k] + conj(Z[L-k])) / 2,  B[k] = (Z[k] - conj(Z[L-k])) / (2i).
// welch pairs consecutive segments (a = x_s, b = x_{s+1}) and uses
//   |A[k]|^2 + |B[k]|^2 = (|Z[k]|^2 + |Z[L-k]|^2) / 2,
// so each thread accumulates |Z[k]|^2 of the bins it owns and the fold
// k <-> L-k happens once per work unit.  csd pairs x_s with y_s and uses
//   conj(A[k]) * B[k] = Im(Z[L-k] Z[k]) / 2 - i (|Z[k]|^2 - |Z[L-k]|^2) / 4.
// Constant detrend after windowing removes mean(x_w) * FFT(rect_nperseg):
// with nfft == nperseg that is exactly the DC bin (Z[0] := 0); with zero
// padding Z[k] -= (Z[0]/nperseg) * D[k], D[k] = sum_{n<nperseg} W^{nk}
// (linearity of the DFT; Z[0] is the windowed segment sum).
#pragma once
#include "fft_core.cuh"
#include "launch.h"

namespace ib200 {

// Values per thread: 16 (f32) / 8 (f64) for long transforms; short
// transforms keep at least 32 threads per group where possible.
#ifndef IB200_F64_E16_FROM
#define IB200_F64_E16_FROM 2048
#endif
template <typename T> __host__ __device__ constexpr int values_per_thread(int L) {
  const int big = std::is_same<T, float>::value || L >= (IB200_F64_E16_FROM) ? 16 : 8;
  const int minE = 2;
  int e = L / 32;
  if (e > big)
    e = big;
  if (e < minE)
    e = minE;
  return e;
}

// csd / coherence pair consecutive segments of one signal per transform and
// stage the x and y spectra side by side, except where two spectra do not
// fit in shared memory (f64, L = 8192): there a task is one segment and
// x_s, y_s share a transform.  Host and device agree through this function.
template <typename T, int L> __host__ __device__ constexpr bool packs_xy() {
  return sizeof(T) == 8 && L >= 8192;
}

// ACC_COH accumulates, per one-sided bin, Sxx = sum |X|^2, Syy = sum |Y|^2
// and Sxy = sum Re(conj(X) Y) (magnitude-squared coherence).
enum AccMode { ACC_PSD = 0, ACC_CSD = 1, ACC_COH = 2 };



template <typename T> struct SpecArgs {
  using V = typename V2T<T>::type;
  const T *x;          // channel 0, sample 0 of x (offset applied)
  const T *y;          // same for y (csd); equals x otherwise
  int64_t x_cs, x_ss;  // channel / sample strides of x, in elements
  int64_t y_cs, y_ss;
  int64_t C;           // channels
  int64_t nperseg, step;
  int64_t seg0;        // first segment of this launch (segment-range shard)
  int64_t S;           // segments handled by this launch (per channel)
  const T *win;        // [nfft], window in T, zero past nperseg
  const V *tw;         // [nfft], W_nfft^m
  const V *dtab;       // [nfft], D[k] (dc_mode 2 only)
  int dc_mode;         // 0 none, 1 DC bin := 0, 2 zero-padded correction,
                       // 3 least-squares line removal (native 'linear_lsq')
  int64_t Tc;          // transforms per channel
  // accumulate kernels
  int64_t nq;          // work units per channel
  int64_t Qt;          // transforms per unit
  int64_t U;           // work units in total
  double *scratch;     // PSD: U*F doubles; CSD: U*F double2
  int64_t F;           // output bins
  // store kernels
  void *out;
  int64_t o_cs, o_rs, o_ts; // channel / bin / segment strides (elements)
  int out_kind;
  double psd_scale;    // spectrogram 'psd' scale
  int onesided_mask;   // 1: double bins 1..F-2
};

// Loads the windowed pass-0 inputs of one transform: re from a, im from b.
template <typename T, int L, int E, int P>
__device__ __forceinline__ void load_pair(typename V2T<T>::type *v,
                                          const T *__restrict__ pa,
                                          const T *__restrict__ pb,
                                          int64_t sa, int64_t sb, bool hasb,
                                          int64_t nperseg,
                                          const T *__restrict__ win, int t) {
  static_for<0, E>([&](auto eIC) {
    constexpr int e = decltype(eIC)::value;
    const int n = in_index<L, E, P>(t, e);
    T a = T(0), b = T(0);
    if (n < nperseg) {
      const T w = __ldg(win + n);
      a = __ldg(pa + n * sa) * w;
      if (hasb)
        b = __ldg(pb + n * sb) * w;
    }
    v[e] = {a, b};
  });
}

// Least-squares line removal (detrend after the window, as the constant
// detrend of the reference frontend, spectral_analysis.cpp:75-82) from both
// sequences of a packed pair (re = a, im = b) held in pass-0 order; samples
// at n >= M are zero padding and stay zero.  This is the native 'linear_lsq'
// option: the reference's 'linear' does not detrend at all.  Sums are
// reduced in f64 over the group: xor shuffles within a warp (or within the
// group's lanes when P < 32), then red[(P/32) * 4] per group in shared memory.
template <typename T, int L, int E, int P, int G, typename V>
__device__ __forceinline__ void detrend_linear(V *v, int t, int g, int64_t M,
                                               double *red) {
  double s0a = 0.0, s1a = 0.0, s0b = 0.0, s1b = 0.0;
  static_for<0, E>([&](auto eIC) {
    constexpr int e = decltype(eIC)::value;
    const double n = (double)in_index<L, E, P>(t, e);
    s0a += (double)v[e].x;
    s1a = fma(n, (double)v[e].x, s1a);
    s0b += (double)v[e].y;
    s1b = fma(n, (double)v[e].y, s1b);
  });
  constexpr int W = P < 32 ? P : 32;
  const unsigned lane = threadIdx.x & 31u;
  const unsigned mask =
      W == 32 ? 0xffffffffu : (((1u << W) - 1u) << (lane & ~(unsigned)(W - 1)));
#pragma unroll
  for (int off = W / 2; off > 0; off >>= 1) {
    s0a += __shfl_xor_sync(mask, s0a, off);
    s1a += __shfl_xor_sync(mask, s1a, off);
    s0b += __shfl_xor_sync(mask, s0b, off);
    s1b += __shfl_xor_sync(mask, s1b, off);
  }
  if constexpr (P > 32) {
    double *r = red + g * (P / 32) * 4;
    if ((t & 31) == 0) {
      const int w = t / 32;
      r[4 * w] = s0a;
      r[4 * w + 1] = s1a;
      r[4 * w + 2] = s0b;
      r[4 * w + 3] = s1b;
    }
    group_sync<G, P>(g);
    s0a = s1a = s0b = s1b = 0.0;
    for (int w = 0; w < P / 32; ++w) {
      s0a += r[4 * w];
      s1a += r[4 * w + 1];
      s0b += r[4 * w + 2];
      s1b += r[4 * w + 3];
    }
    group_sync<G, P>(g); // red is free for the next transform
  }
  const double Md = (double)M, nb = 0.5 * (Md - 1.0);
  const double snn = Md * (Md * Md - 1.0) / 12.0; // sum (n - nb)^2
  const double ba = snn > 0.0 ? (s1a - nb * s0a) / snn : 0.0;
  const double bb = snn > 0.0 ? (s1b - nb * s0b) / snn : 0.0;
  const double aa = s0a / Md - ba * nb, ab = s0b / Md - bb * nb;
  static_for<0, E>([&](auto eIC) {
    constexpr int e = decltype(eIC)::value;
    const int n = in_index<L, E, P>(t, e);
    if (n < M) {
      v[e].x -= (T)fma(ba, (double)n, aa);
      v[e].y -= (T)fma(bb, (double)n, ab);
    }
  });
}

// ---------------------------------------------------------------------------
// welch / csd: accumulate per work unit, one transform group per CTA.
// ---------------------------------------------------------------------------
template <typename T, int L, int E, int MODE>
__global__ void __launch_bounds__(L / E)
    spectral_accum_kernel(const SpecArgs<T> p) {
  using V = typename V2T<T>::type;
  constexpr int P = L / E;
  constexpr int FH = L / 2 + 1;        // one-sided bins kept per unit
  constexpr int NB = (FH + P - 1) / P; // csd bins per thread
  constexpr int NACC = MODE == ACC_PSD ? E : (MODE == ACC_CSD ? 2 : 3) * NB;
  // csd / coherence stage the x-pair and y-pair spectra side by side; where
  // two spectra do not fit in shared memory (f64, L = 8192) a task is one
  // segment and x_s, y_s share one transform (Z = X + iY) instead.
  constexpr bool PACKXY = packs_xy<T, L>() && MODE != ACC_PSD;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  V *buf = reinterpret_cast<V *>(smem_raw);   // x pair (welch: the pair)
  V *buf2 = buf + spad_size(L);               // y pair (csd, coherence)
  __shared__ V zdc;
  __shared__ double red[P > 32 ? (P / 32) * 4 : 1];
  const int t = threadIdx.x;

  // Z = FFT(w a + i w b) of segments a = 2 task, b = 2 task + 1 of channel
  // base xc (stride ss); with dc_mode 2 the windowed means are removed in
  // the frequency domain afterwards, with dc_mode 3 the least-squares lines
  // before the transform.
  auto transform = [&](V *v, const T *xc, int64_t ss, int64_t task, V *b) {
    const int64_t s = p.seg0 + 2 * task;
    const bool hasb = (2 * task + 1) < p.S;
    load_pair<T, L, E, P>(v, xc + s * p.step * ss, xc + (s + 1) * p.step * ss,
                          ss, ss, hasb, p.nperseg, p.win, t);
    if (p.dc_mode == 3)
      detrend_linear<T, L, E, P, 1>(v, t, 0, p.nperseg, red);
    fft_group<T, L, E, P, 1>(v, b, t, 0, p.tw);
  };
  // Bin k of a staged pair spectrum after the detrend of dc_mode.
  auto bin = [&](const V *b, int k, V m) -> V {
    V z = b[spad(k)];
    // constant and least-squares detrends leave a residual of zero sum: the
    // DC bin is exactly zero
    if ((p.dc_mode == 1 || p.dc_mode == 3) && k == 0)
      z = {T(0), T(0)};
    else if (p.dc_mode == 2)
      z = vsub(z, vmul(m, p.dtab[k]));
    return z;
  };

  for (int64_t u = blockIdx.x; u < p.U; u += gridDim.x) {
    const int64_t c = u / p.nq;
    const int64_t q = u - c * p.nq;
    const int64_t task0 = q * p.Qt;
    const int64_t task1 = min(task0 + p.Qt, p.Tc);
    const T *xc = p.x + c * p.x_cs;
    const T *yc = p.y + c * p.y_cs;

    double acc[NACC];
#pragma unroll
    for (int i = 0; i < NACC; ++i)
      acc[i] = 0.0;

    for (int64_t task = task0; task < task1; ++task) {
      V v[E];
      if constexpr (!PACKXY)
        transform(v, xc, p.x_ss, task, buf);
      if constexpr (MODE == ACC_PSD) {
        if (p.dc_mode == 1 || p.dc_mode == 3) {
          if (t == 0)
            v[0] = {T(0), T(0)}; // out_bin(0, 0) == 0
        } else if (p.dc_mode == 2) {
          if (t == 0)
            zdc = v[0];
          __syncthreads();
          const V z0 = zdc;
          const T inv = T(1) / T(p.nperseg);
          const V m = {z0.x * inv, z0.y * inv};
#pragma unroll
          for (int e = 0; e < E; ++e)
            v[e] = vsub(v[e], vmul(m, p.dtab[out_bin<L, E, P>(t, e)]));
          __syncthreads();
        }
#pragma unroll
        for (int e = 0; e < E; ++e)
          acc[e] += (double)fma(v[e].x, v[e].x, v[e].y * v[e].y);
      } else if constexpr (PACKXY) {
        // Z = FFT(w x_s + i w y_s), s = task (tasks are segments here)
        const int64_t s = p.seg0 + task;
        load_pair<T, L, E, P>(v, xc + s * p.step * p.x_ss, yc + s * p.step * p.y_ss,
                              p.x_ss, p.y_ss, true, p.nperseg, p.win, t);
        if (p.dc_mode == 3)
          detrend_linear<T, L, E, P, 1>(v, t, 0, p.nperseg, red);
        fft_group<T, L, E, P, 1>(v, buf, t, 0, p.tw);
        store_bins<L, E, P>(v, buf, t);
        __syncthreads();
        const T inv = T(1) / T(p.nperseg);
        V mz = {T(0), T(0)};
        if (p.dc_mode == 2)
          mz = {buf[0].x * inv, buf[0].y * inv};
        // 2X = Z[k] + conj Z[L-k], 2Y = -i (Z[k] - conj Z[L-k])
#pragma unroll
        for (int i = 0; i < NB; ++i) {
          const int k = t + i * P;
          if (k < FH) {
            const int m = (L - k) & (L - 1);
            const V zk = bin(buf, k, mz), zm = bin(buf, m, mz);
            const T xr = zk.x + zm.x, xi = zk.y - zm.y;
            const T yr = zk.y + zm.y, yi = zm.x - zk.x;
            const T re = fma(xr, yr, xi * yi);
            if constexpr (MODE == ACC_COH) {
              acc[3 * i] += (double)fma(xr, xr, xi * xi);
              acc[3 * i + 1] += (double)fma(yr, yr, yi * yi);
              acc[3 * i + 2] += (double)re;
            } else {
              acc[2 * i] += (double)re;
              acc[2 * i + 1] += (double)fma(xr, yi, -xi * yr);
            }
          }
        }
        __syncthreads();
      } else {
        store_bins<L, E, P>(v, buf, t);
        transform(v, yc, p.y_ss, task, buf2);
        store_bins<L, E, P>(v, buf2, t);
        __syncthreads();
        const T inv = T(1) / T(p.nperseg);
        V mx = {T(0), T(0)}, my = {T(0), T(0)};
        if (p.dc_mode == 2) {
          mx = {buf[0].x * inv, buf[0].y * inv};
          my = {buf2[0].x * inv, buf2[0].y * inv};
        }
        // partials: 4 (conj(Xa) Ya + conj(Xb) Yb), 4 |X|^2, 4 |Y|^2 (see
        // accum_fast_kernel)
#pragma unroll
        for (int i = 0; i < NB; ++i) {
          const int k = t + i * P;
          if (k < FH) {
            const int m = (L - k) & (L - 1);
            const V xk = bin(buf, k, mx), xm = bin(buf, m, mx);
            const V yk = bin(buf2, k, my), ym = bin(buf2, m, my);
            const T xar = xk.x + xm.x, xai = xk.y - xm.y;
            const T xbr = xk.y + xm.y, xbi = xm.x - xk.x;
            const T yar = yk.x + ym.x, yai = yk.y - ym.y;
            const T ybr = yk.y + ym.y, ybi = ym.x - yk.x;
            const T re = fma(xar, yar, fma(xai, yai, fma(xbr, ybr, xbi * ybi)));
            if constexpr (MODE == ACC_COH) {
              acc[3 * i] +=
                  (double)fma(xar, xar, fma(xai, xai, fma(xbr, xbr, xbi * xbi)));
              acc[3 * i + 1] +=
                  (double)fma(yar, yar, fma(yai, yai, fma(ybr, ybr, ybi * ybi)));
              acc[3 * i + 2] += (double)re;
            } else {
              const T im =
                  fma(xar, yai, fma(-xai, yar, fma(xbr, ybi, -xbi * ybr)));
              acc[2 * i] += (double)re;
              acc[2 * i + 1] += (double)im;
            }
          }
        }
        __syncthreads();
      }
    }

    // Unit partial -> scratch (fixed order, no atomics).
    if constexpr (MODE == ACC_PSD) {
      double *sm = reinterpret_cast<double *>(smem_raw);
#pragma unroll
      for (int e = 0; e < E; ++e)
        sm[out_bin<L, E, P>(t, e)] = acc[e];
      __syncthreads();
      for (int k = t; k < FH; k += P)
        p.scratch[u * FH + k] = sm[k] + sm[(L - k) & (L - 1)];
      __syncthreads();
    } else if constexpr (MODE == ACC_CSD) {
      double2 *s2 = reinterpret_cast<double2 *>(p.scratch);
#pragma unroll
      for (int i = 0; i < NB; ++i) {
        const int k = t + i * P;
        if (k < FH)
          s2[u * FH + k] = make_double2(acc[2 * i], acc[2 * i + 1]);
      }
    } else {
      // [slot][bin] of (Sxx, Syy), (Sxy, 0)
      double2 *s2 = reinterpret_cast<double2 *>(p.scratch);
#pragma unroll
      for (int i = 0; i < NB; ++i) {
        const int k = t + i * P;
        if (k < FH) {
          s2[2 * (u * FH + k)] = make_double2(acc[3 * i], acc[3 * i + 1]);
          s2[2 * (u * FH + k) + 1] = make_double2(acc[3 * i + 2], 0.0);
        }
      }
    }
  }
}

// Flat work split: CTA b of n owns the flattened (channel, transform)
// indices [flat_start(b), flat_start(b + 1)) of T; flat_owner(j) is the CTA
// that owns index j.
__host__ __device__ inline int64_t flat_start(int64_t b, int64_t T, int64_t n) {
  return b * T / n;
}
__host__ __device__ inline int64_t flat_owner(int64_t j, int64_t T, int64_t n) {
  int64_t b = j * n / T; // flat_start(b) <= j
  while (b + 1 < n && flat_start(b + 1, T, n) <= j)
    ++b;
  return b;
}

// Sum the partials of each channel in slot order, scale, mask, store.
// Slots: with flat_T == 0, the nq units of channel c are c*nq .. c*nq+nq-1;
// with flat_T = C * Tc > 0 (flat split over nq CTAs), CTA b's partial of
// channel c is slot b + c for the CTAs b whose range meets the channel.
// Partials hold the one-sided bins k <= L/2 (PSD partials hold A[k] + A[L-k],
// the pair average is the factor 1/2).  For real inputs the two-sided
// spectrum is the conjugate mirror: P[L-k] = conj(P[k]).
__device__ __forceinline__ void finalize_slots(int64_t c, int64_t C, int64_t nq,
                                               int64_t flat_T, int64_t *lo,
                                               int64_t *hi) {
  if (flat_T > 0) {
    const int64_t Tc = flat_T / C;
    *lo = flat_owner(c * Tc, flat_T, nq) + c;
    *hi = flat_owner((c + 1) * Tc - 1, flat_T, nq) + c + 1;
  } else {
    *lo = c * nq;
    *hi = *lo + nq;
  }
}

// Slot values summed for one bin: s[0], s[1] (s[2] for coherence) of the
// slots [q0, hi) with stride dq.
template <int MODE>
__device__ __forceinline__ void finalize_sum(const double *__restrict__ scratch,
                                             int64_t FH, int64_t kk, int64_t q0,
                                             int64_t hi, int64_t dq, double *s) {
  // slot values of one bin, read B at a time (independent loads in flight)
  // and added in slot order, so the sums do not depend on B
  constexpr int B = 8;
  auto run = [&](auto ld, auto add) {
    using X = decltype(ld(int64_t(0)));
    int64_t q = q0;
    for (; q + (B - 1) * dq < hi; q += B * dq) {
      X a[B];
#pragma unroll
      for (int j = 0; j < B; ++j)
        a[j] = ld(q + j * dq);
#pragma unroll
      for (int j = 0; j < B; ++j)
        add(a[j]);
    }
    for (; q < hi; q += dq)
      add(ld(q));
  };
  const double2 *s2 = reinterpret_cast<const double2 *>(scratch);
  if constexpr (MODE == ACC_COH) {
    run([&](int64_t q) {
          const double2 a = s2[2 * (q * FH + kk)];
          return make_double3(a.x, a.y, s2[2 * (q * FH + kk) + 1].x);
        },
        [&](double3 a) {
          s[0] += a.x;
          s[1] += a.y;
          s[2] += a.z;
        });
  } else if constexpr (MODE == ACC_PSD) {
    run([&](int64_t q) { return scratch[q * FH + kk]; },
        [&](double a) { s[0] += a; });
  } else {
    run([&](int64_t q) { return s2[q * FH + kk]; },
        [&](double2 a) {
          s[0] += a.x;
          s[1] += a.y;
        });
  }
}

// Scale, mask and store output bin k of channel c from its summed slots.
template <int MODE>
__device__ __forceinline__ void finalize_store(const double *s, int64_t c,
                                               int64_t k, int64_t F, bool mirror,
                                               double avg_scale, int onesided_mask,
                                               void *out, int64_t o_cs,
                                               int out_kind) {
  if (MODE == ACC_COH) {
    // Reference coherence (spectral_analysis.cpp:199-221): Pxx, Pyy from
    // welch, Pxy = Re(csd) (the reference's csd returns the real part), all
    // with the same scale and mask; Cxy = Pxy^2 / max(Pxx Pyy, 1e-30), and 0
    // where Pxx Pyy <= 1e-30.
    double f = 0.25 * avg_scale; // partials are 4x the sums
    if (onesided_mask && k >= 1 && k <= F - 2)
      f *= 2.0;
    const double pxx = s[0] * f, pyy = s[1] * f, pxy = s[2] * f;
    const double den = pxx * pyy;
    const double eps = 1e-30;
    reinterpret_cast<double *>(out)[c * o_cs + k] =
        den <= eps ? 0.0 : (pxy * pxy) / (den > eps ? den : eps);
    return;
  }
  double re, im = 0.0;
  if (MODE == ACC_PSD) {
    re = s[0] * 0.5;
  } else {
    re = s[0] * 0.25; // partials are 4 conj(X) Y
    im = s[1] * 0.25;
    if (mirror)
      im = -im;
  }
  double f = (out_kind == OUT_RAW_F64_K) ? 1.0 : avg_scale;
  if (out_kind != OUT_RAW_F64_K && onesided_mask && k >= 1 && k <= F - 2)
    f *= 2.0;
  re *= f;
  im *= f;
  switch (out_kind) {
  case OUT_C64_K:
    reinterpret_cast<float2 *>(out)[c * o_cs + k] =
        make_float2((float)re, (float)im);
    break;
  case OUT_C128_K:
    reinterpret_cast<double2 *>(out)[c * o_cs + k] = make_double2(re, im);
    break;
  case OUT_RAW_F64_K:
    if (MODE == ACC_PSD) {
      reinterpret_cast<double *>(out)[c * o_cs + k] = re;
    } else {
      reinterpret_cast<double2 *>(out)[c * o_cs + k] = make_double2(re, im);
    }
    break;
  default: // OUT_REAL_F64_K
    reinterpret_cast<double *>(out)[c * o_cs + k] = re;
    break;
  }
}

// One thread per output bin: for few slots per channel (many channels).
template <int MODE>
__global__ void spectral_finalize_kernel(const double *__restrict__ scratch,
                                         int64_t C, int64_t nq, int64_t flat_T,
                                         int64_t L, int64_t F, double avg_scale,
                                         int onesided_mask, void *out,
                                         int64_t o_cs, int out_kind) {
  const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i >= C * F)
    return;
  const int64_t FH = L / 2 + 1;
  const int64_t c = i / F, k = i - c * F;
  const bool mirror = k >= FH;
  const int64_t kk = mirror ? L - k : k;
  int64_t lo, hi;
  finalize_slots(c, C, nq, flat_T, &lo, &hi);
  double s[3] = {0.0, 0.0, 0.0};
  finalize_sum<MODE>(scratch, FH, kk, lo, hi, 1, s);
  finalize_store<MODE>(s, c, k, F, mirror, avg_scale, onesided_mask, out, o_cs,
                       out_kind);
}

// Many slots per channel (few channels): a CTA of 32 x FW threads handles 32
// consecutive output bins; warp w sums the slots lo + w, lo + w + FW, ...
// (32 consecutive bins of one slot are one coalesced read), and warp 0 adds
// the FW partial sums in warp order, so the result is deterministic.
constexpr int kFinalizeWideWarps = 8;
constexpr int kFinalizeWideFrom = 32; // slots per channel that select this kernel

template <int MODE>
__global__ void __launch_bounds__(32 * kFinalizeWideWarps)
    spectral_finalize_wide_kernel(const double *__restrict__ scratch, int64_t C,
                                  int64_t nq, int64_t flat_T, int64_t L,
                                  int64_t F, double avg_scale, int onesided_mask,
                                  void *out, int64_t o_cs, int out_kind) {
  constexpr int FW = kFinalizeWideWarps;
  __shared__ double part[FW][3][32];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int64_t i = blockIdx.x * (int64_t)32 + lane;
  const bool valid = i < C * F;
  const int64_t FH = L / 2 + 1;
  const int64_t c = valid ? i / F : 0, k = valid ? i - c * F : 0;
  const bool mirror = k >= FH;
  const int64_t kk = mirror ? L - k : k;
  double s[3] = {0.0, 0.0, 0.0};
  if (valid) {
    int64_t lo, hi;
    finalize_slots(c, C, nq, flat_T, &lo, &hi);
    finalize_sum<MODE>(scratch, FH, kk, lo + w, hi, FW, s);
  }
  part[w][0][lane] = s[0];
  part[w][1][lane] = s[1];
  part[w][2][lane] = s[2];
  __syncthreads();
  if (w != 0 || !valid)
    return;
  double t[3] = {0.0, 0.0, 0.0};
  for (int ww = 0; ww < FW; ++ww) {
    t[0] += part[ww][0][lane];
    t[1] += part[ww][1][lane];
    t[2] += part[ww][2][lane];
  }
  finalize_store<MODE>(t, c, k, F, mirror, avg_scale, onesided_mask, out, o_cs,
                       out_kind);
}

// Launch the finalize kernel that suits the slot count per channel.
template <int MODE>
cudaError_t launch_finalize(const double *scratch, int64_t C, int64_t nq,
                            int64_t flat_T, int64_t L, int64_t F, double avg_scale,
                            int onesided_mask, void *out, int64_t o_cs,
                            int out_kind, cudaStream_t stream) {
  const int64_t n = C * F;
  // slots per channel: nq units, or about nq / C CTAs of the flat split
  const int64_t per = flat_T > 0 ? (nq + C - 1) / C + 1 : nq;
  if (per >= kFinalizeWideFrom) {
    spectral_finalize_wide_kernel<MODE>
        <<<(unsigned)((n + 31) / 32), 32 * kFinalizeWideWarps, 0, stream>>>(
            scratch, C, nq, flat_T, L, F, avg_scale, onesided_mask, out, o_cs,
            out_kind);
  } else {
    const int threads = 256;
    spectral_finalize_kernel<MODE><<<(unsigned)((n + threads - 1) / threads),
                                     threads, 0, stream>>>(
        scratch, C, nq, flat_T, L, F, avg_scale, onesided_mask, out, o_cs,
        out_kind);
  }
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// spectrogram / stft: G transform groups per CTA, columns staged in shared
// memory, stored bin-major so each bin row gets 2*G adjacent segments.
// ---------------------------------------------------------------------------
template <typename T, int L, int E, int G>
__global__ void __launch_bounds__(G *(L / E))
    spectral_store_kernel(const SpecArgs<T> p) {
  using V = typename V2T<T>::type;
  constexpr int P = L / E;
  constexpr int GS = spad_size(L) + 2; // +2 slots: conflict-free (k, g) reads
  extern __shared__ __align__(16) unsigned char smem_raw[];
  V *smem = reinterpret_cast<V *>(smem_raw);
  const int g = threadIdx.x / P;
  const int t = threadIdx.x - g * P;
  V *buf = smem + g * GS;
  __shared__ double red[P > 32 ? G * (P / 32) * 4 : 1];
  const int64_t tpc = (p.Tc + G - 1) / G; // tiles per channel
  const int64_t ntiles = p.C * tpc;
  const T inv_nps = T(1) / T(p.nperseg);

  for (int64_t tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
    const int64_t c = tile / tpc;
    const int64_t task0 = (tile - c * tpc) * G;
    const int64_t task = task0 + g;
    if (task < p.Tc) {
      const T *xc = p.x + c * p.x_cs;
      const int64_t s = p.seg0 + 2 * task;
      const bool hasb = (2 * task + 1) < p.S;
      V v[E];
      load_pair<T, L, E, P>(v, xc + s * p.step * p.x_ss,
                            xc + (s + 1) * p.step * p.x_ss, p.x_ss, p.x_ss,
                            hasb, p.nperseg, p.win, t);
      if (p.dc_mode == 3)
        detrend_linear<T, L, E, P, G>(v, t, g, p.nperseg, red);
      fft_group<T, L, E, P, G>(v, buf, t, g, p.tw);
      store_bins<L, E, P>(v, buf, t);
    }
    __syncthreads();

    const int64_t F = p.F;
    for (int64_t idx = threadIdx.x; idx < F * G; idx += blockDim.x) {
      const int gg = (int)(idx % G);
      const int k = (int)(idx / G);
      const int64_t tk = task0 + gg;
      if (tk >= p.Tc)
        continue;
      const V *bg = smem + gg * GS;
      V zk = bg[spad(k)];
      V zm = bg[spad((L - k) & (L - 1))];
      if (p.dc_mode == 1 || p.dc_mode == 3) {
        if (k == 0)
          zk = zm = {T(0), T(0)};
      } else if (p.dc_mode == 2) {
        const V z0 = bg[0];
        const V m = {z0.x * inv_nps, z0.y * inv_nps};
        zk = vsub(zk, vmul(m, p.dtab[k]));
        zm = vsub(zm, vmul(m, p.dtab[(L - k) & (L - 1)]));
      }
      // A = (zk + conj zm)/2, B = (zk - conj zm)/(2i)
      const V A = {T(0.5) * (zk.x + zm.x), T(0.5) * (zk.y - zm.y)};
      const V B = {T(0.5) * (zk.y + zm.y), T(0.5) * (zm.x - zk.x)};
      const bool hasb = (2 * tk + 1) < p.S;
      const int64_t o = c * p.o_cs + k * p.o_rs + (2 * tk) * p.o_ts;
      switch (p.out_kind) {
      case OUT_C64_K:
      case OUT_C128_K: {
        V *out = reinterpret_cast<V *>(p.out);
        out[o] = A;
        if (hasb)
          out[o + p.o_ts] = B;
        break;
      }
      case OUT_REAL_F64_K: {
        double *out = reinterpret_cast<double *>(p.out);
        out[o] = (double)A.x;
        if (hasb)
          out[o + p.o_ts] = (double)B.x;
        break;
      }
      case OUT_PSD_F64_K: {
        double *out = reinterpret_cast<double *>(p.out);
        double f = p.psd_scale;
        if (p.onesided_mask && k >= 1 && k <= F - 2)
          f *= 2.0;
        out[o] = (double)fma(A.x, A.x, A.y * A.y) * f;
        if (hasb)
          out[o + p.o_ts] = (double)fma(B.x, B.x, B.y * B.y) * f;
        break;
      }
      default: { // OUT_MAG_F64_K
        double *out = reinterpret_cast<double *>(p.out);
        out[o] = (double)sqrt(fma(A.x, A.x, A.y * A.y));
        if (hasb)
          out[o + p.o_ts] = (double)sqrt(fma(B.x, B.x, B.y * B.y));
        break;
      }
      }
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// STFT fast path: contiguous channels (unit sample stride), nperseg == nfft,
// one-sided, no detrend or DC-only detrend, complex<T> output (C, F, S) with
// unit segment stride.
//
// Work unit: NSUB consecutive tiles of one channel, one CTA.  A tile is Q =
// G*M consecutive segment pairs; each of the G transform groups (P threads)
// runs M pairs at once, interleaved in registers.
//   * loads: with SH > 0 the second segment's samples that overlap the first
//     come from the first segment's registers (hop = SH * L/R0);
//   * the window rows (pre-scaled by 1/2, the unpack factor; exact in binary
//     floating point) and, with TWS, each thread's Stockham twiddles live in
//     shared memory, filled once per CTA;
//   * the transforms are staged in shared memory; the whole CTA then unpacks
//     A[k] = Z[k] + conj Z[L-k], B[k] = -i (Z[k] - conj Z[L-k]) (halves folded
//     into the window), 2Q lanes per bin row.
// Bin rows of the (C, F, S) output start at arbitrary element offsets (S is
// odd in general), so a tile's 2Q columns do not cover whole 32-byte
// sectors; sectors completed by two CTAs become masked DRAM writes.  The
// lanes of a row therefore write the 2Q columns that end on a sector
// boundary, shifted back by the row's phase phi, and keep the phi trailing
// columns in a per-row carry for the unit's next tile: every sector of a
// row is written once, whole, except at the two ends of a unit.
// ---------------------------------------------------------------------------
template <typename T, int L, int E, int G, int M, int SH, bool TWS>
__global__ void __launch_bounds__(G *(L / E))
    stft_fast_kernel(const SpecArgs<T> p, int nsub) {
  using V = typename V2T<T>::type;
  using PL = Plan<L, E>;
  using TT = ThreadTw<T, L, E>;
  constexpr int P = L / E;
  constexpr int NT = G * P;
  constexpr int Q = G * M;               // segment pairs per tile
  constexpr int R0 = PL::radix(0);
  constexpr int GS = spad_size(L) + 2;   // slot spad(L) holds a copy of Z[0]
  constexpr int SPR = 2 * Q;             // columns (segments) per tile row
  constexpr int RPI = NT / SPR;          // bin rows per store iteration
  constexpr int FH = L / 2 + 1;
  constexpr int NIT = (FH + RPI - 1) / RPI;
  constexpr int WS = E + 16 / (int)sizeof(T);
  constexpr int SEC = 32 / (int)sizeof(V); // output values per 32-byte sector
  // carry slots, rounded to 16 bytes so the window rows after them stay
  // aligned for 128-bit reads
  constexpr int CN = (FH * (SEC - 1) * (int)sizeof(V) + 15) / 16 * 16 / (int)sizeof(V);
  static_assert(SPR % SEC == 0 && SPR >= SEC, "tile rows are whole sectors");
  static_assert(SH >= 0 && SH < R0, "overlap shift");
  static_assert(TWS || M == 1, "interleaved transforms use twiddle rows");
  extern __shared__ __align__(16) unsigned char smem_raw[];
  V *smem = reinterpret_cast<V *>(smem_raw);
  V *tws = smem + Q * GS;                                   // [P][stride]
  V *carry = tws + (TWS ? P * TT::stride() : 0);            // [FH][SEC-1]
  T *wsm = reinterpret_cast<T *>(carry + CN);                // [P][WS]
  const int g = threadIdx.x / P;
  const int t = threadIdx.x - g * P;
  V *buf = smem + g * M * GS; // pairs g*M .. g*M + M - 1

  fill_batched<8>(
      threadIdx.x, P * E, NT,
      [&](int i) { return T(0.5) * p.win[in_index<L, E, P>(i / E, i % E)]; },
      [&](int i, T v) { wsm[(i / E) * WS + i % E] = v; });
  if constexpr (TWS)
    fill_thread_twiddles<T, L, E, P>(tws, p.tw, threadIdx.x, NT);
  __syncthreads();
  const V *row = tws + t * TT::stride();

  const int lane = threadIdx.x % SPR;
  const int kr0 = threadIdx.x / SPR;
  static_assert(RPI % SEC == 0, "a thread's rows share one sector phase");

  const int64_t tpc = (p.Tc + Q - 1) / Q;       // tiles per channel
  const int64_t upc = (tpc + nsub - 1) / nsub;  // units per channel
  const int64_t nunits = p.C * upc;
  V *out = reinterpret_cast<V *>(p.out);

  // Windowed inputs of the group's M pairs of a tile into v; false when the
  // group's first pair is past the channel's end (the whole group idles).
  V v[M][E];
  auto load_tile = [&](int64_t c, int64_t task0) -> bool {
    const int64_t taskg = task0 + g * M;
    if (taskg >= p.Tc)
      return false;
    T wv[E];
    if constexpr (sizeof(T) == 4 && E % 4 == 0) {
      const float4 *w4 = reinterpret_cast<const float4 *>(wsm + t * WS);
      static_for<0, E / 4>([&](auto qIC) {
        constexpr int q = decltype(qIC)::value;
        const float4 f = w4[q];
        wv[4 * q] = f.x;
        wv[4 * q + 1] = f.y;
        wv[4 * q + 2] = f.z;
        wv[4 * q + 3] = f.w;
      });
    } else if constexpr (sizeof(T) == 8 && E % 2 == 0) {
      const double2 *w2 = reinterpret_cast<const double2 *>(wsm + t * WS);
      static_for<0, E / 2>([&](auto qIC) {
        constexpr int q = decltype(qIC)::value;
        const double2 f = w2[q];
        wv[2 * q] = f.x;
        wv[2 * q + 1] = f.y;
      });
    } else {
      static_for<0, E>([&](auto eIC) {
        constexpr int e = decltype(eIC)::value;
        wv[e] = wsm[t * WS + e];
      });
    }
    static_for<0, M>([&](auto mIC) {
      constexpr int m = decltype(mIC)::value;
      const int64_t task = taskg + m;
      // a missing pair (channel tail) transforms zeros, never stored
      const bool hasa = task < p.Tc;
      const bool hasb = (2 * task + 1) < p.S;
      const T *xa = p.x + c * p.x_cs +
                    (p.seg0 + 2 * (hasa ? task : taskg)) * p.step + t;
      if (!hasa) {
        static_for<0, E>([&](auto eIC) {
          constexpr int e = decltype(eIC)::value;
          v[m][e] = {T(0), T(0)};
        });
        return;
      }
      T ra[E];
      static_for<0, E>([&](auto eIC) {
        constexpr int e = decltype(eIC)::value;
        ra[e] = __ldg(xa + in_index<L, E, P>(0, e));
      });
      if (hasb) {
        static_for<0, E>([&](auto eIC) {
          constexpr int e = decltype(eIC)::value;
          constexpr int n = in_index<L, E, P>(0, e);
          constexpr int r = e % R0;
          T b;
          if constexpr (SH > 0 && r + SH < R0)
            b = ra[e + SH];
          else
            b = __ldg(xa + p.step + n);
          v[m][e] = {ra[e] * wv[e], b * wv[e]};
        });
      } else {
        static_for<0, E>([&](auto eIC) {
          constexpr int e = decltype(eIC)::value;
          v[m][e] = {ra[e] * wv[e], T(0)};
        });
      }
    });
    return true;
  };
  for (int64_t unit = blockIdx.x; unit < nunits; unit += gridDim.x) {
    const int64_t c = unit / upc;
    const int64_t tile0 = (unit - c * upc) * nsub;
    const int ntile = (int)min((int64_t)nsub, tpc - tile0);
    const int64_t ucol0 = 2 * tile0 * Q; // first column of the unit
    V *outc = out + c * p.o_cs;
    // this thread's store role for the unit (see the store below)
    const int phi = (int)((reinterpret_cast<uint64_t>(outc + (int64_t)kr0 * p.o_rs +
                                                       ucol0) /
                           sizeof(V)) & (SEC - 1));
    const bool carry_lane = lane < phi;
    const int jj = carry_lane ? SPR - phi + lane : lane - phi; // tile column
    const bool odd = jj & 1;
    const V *zkp = smem + (jj >> 1) * GS + spad(kr0);
    const V *zmp = smem + (jj >> 1) * GS + spad(L - kr0);
    for (int it = 0; it < ntile; ++it) {
      const int64_t task0 = (tile0 + it) * Q;
      if (load_tile(c, task0)) {
        if constexpr (TWS)
          fft_group_tw_m<T, L, E, P, G, M>(v, buf, GS, t, g, row);
        else
          fft_group<T, L, E, P, G>(v[0], buf, t, g, p.tw);
        static_for<0, M>([&](auto mIC) {
          constexpr int m = decltype(mIC)::value;
          if (p.dc_mode == 1 && t == 0)
            v[m][0] = {T(0), T(0)};
          store_bins<L, E, P>(v[m], buf + m * GS, t);
          if (t == 0)
            buf[m * GS + spad_size(L)] = v[m][0];
        });
      }
      __syncthreads();

      // Store.  A thread's bin rows are k = kr0 + ii*RPI with RPI a multiple
      // of the sector length, so the row's sector phase phi (its columns
      // col0 - phi + lane, lane < 2Q, are whole sectors) is fixed for the
      // unit; lanes >= phi write columns col0 + lane - phi of this tile,
      // lanes < phi write the previous tile's carried column and compute this
      // tile's trailing column SPR - phi + lane (carried, or written at the
      // unit's end).
      const bool first = it == 0;
      const bool last = it == ntile - 1;
      const int64_t col0 = 2 * task0;
      V *rp0 = outc + (int64_t)kr0 * p.o_rs + col0 - phi;
      const int64_t rstep = (int64_t)RPI * p.o_rs;
      // per-tile predicates: write this lane's column (this tile's value, or
      // the carried one), write this tile's trailing column, or carry it
      const bool wmain = (col0 - phi + lane) < p.S && (!carry_lane || !first);
      const bool wtrail = carry_lane && last && (col0 + jj) < p.S;
      const bool wcarry = carry_lane && !last;
      static_for<0, NIT>([&](auto iIC) {
        constexpr int ii = decltype(iIC)::value;
        const int k = kr0 + ii * RPI;
        if (ii + 1 < NIT || k < FH) {
          const V zk = zkp[ii * pad_off<RPI>()];
          const V zm = zmp[-ii * pad_off<RPI>()];
          // even: A = zk + conj zm; odd: B = -i (zk - conj zm)
          const T u = odd ? zk.y : zk.x;
          const T w = odd ? zm.y : zm.x;
          const T u2 = odd ? zm.x : zk.y;
          const T w2 = odd ? zk.x : zm.y;
          const V val = V{u + w, u2 - w2};
          V *rp = rp0 + ii * rstep;
          V *cr = carry + k * (SEC - 1) + lane;
          V sv = val;
          if (carry_lane)
            sv = *cr;
          if (wmain)
            rp[lane] = sv;
          if (wtrail)
            rp[phi + jj] = val;
          if (wcarry)
            *cr = val;
        }
      });
      __syncthreads();
    }
  }
}

} // namespace ib200

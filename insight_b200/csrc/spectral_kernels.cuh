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

enum AccMode { ACC_PSD = 0, ACC_CSD = 1 };


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
  int dc_mode;         // 0 none, 1 DC bin := 0, 2 zero-padded correction
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
  extern __shared__ __align__(16) unsigned char smem_raw[];
  V *buf = reinterpret_cast<V *>(smem_raw);
  __shared__ V zdc;
  const int t = threadIdx.x;

  for (int64_t u = blockIdx.x; u < p.U; u += gridDim.x) {
    const int64_t c = u / p.nq;
    const int64_t q = u - c * p.nq;
    const int64_t task0 = q * p.Qt;
    const int64_t task1 = min(task0 + p.Qt, p.Tc);
    const T *xc = p.x + c * p.x_cs;
    const T *yc = p.y + c * p.y_cs;

    double acc[MODE == ACC_PSD ? E : 2 * NB];
#pragma unroll
    for (int i = 0; i < (MODE == ACC_PSD ? E : 2 * NB); ++i)
      acc[i] = 0.0;

    for (int64_t task = task0; task < task1; ++task) {
      V v[E];
      if constexpr (MODE == ACC_PSD) {
        const int64_t s = p.seg0 + 2 * task;
        const bool hasb = (2 * task + 1) < p.S;
        load_pair<T, L, E, P>(v, xc + s * p.step * p.x_ss,
                              xc + (s + 1) * p.step * p.x_ss, p.x_ss, p.x_ss,
                              hasb, p.nperseg, p.win, t);
      } else {
        const int64_t s = p.seg0 + task;
        load_pair<T, L, E, P>(v, xc + s * p.step * p.x_ss,
                              yc + s * p.step * p.y_ss, p.x_ss, p.y_ss, true,
                              p.nperseg, p.win, t);
      }
      fft_group<T, L, E, P, 1>(v, buf, t, 0, p.tw);

      if constexpr (MODE == ACC_PSD) {
        if (p.dc_mode == 1) {
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
      } else {
#pragma unroll
        for (int e = 0; e < E; ++e)
          buf[spad(out_bin<L, E, P>(t, e))] = v[e];
        __syncthreads();
        V m = {T(0), T(0)};
        if (p.dc_mode == 2) {
          const V z0 = buf[0];
          const T inv = T(1) / T(p.nperseg);
          m = {z0.x * inv, z0.y * inv};
        }
#pragma unroll
        for (int i = 0; i < NB; ++i) {
          const int k = t + i * P;
          if (k < FH) {
            V zk = buf[spad(k)];
            V zm = buf[spad((L - k) & (L - 1))];
            if (p.dc_mode == 1) {
              if (k == 0)
                zk = zm = {T(0), T(0)};
            } else if (p.dc_mode == 2) {
              zk = vsub(zk, vmul(m, p.dtab[k]));
              zm = vsub(zm, vmul(m, p.dtab[(L - k) & (L - 1)]));
            }
            const T re = T(0.5) * fma(zm.x, zk.y, zm.y * zk.x);
            const T im = T(0.25) * (fma(zm.x, zm.x, zm.y * zm.y) -
                                    fma(zk.x, zk.x, zk.y * zk.y));
            acc[2 * i] += (double)re;
            acc[2 * i + 1] += (double)im;
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
    } else {
      double2 *s2 = reinterpret_cast<double2 *>(p.scratch);
#pragma unroll
      for (int i = 0; i < NB; ++i) {
        const int k = t + i * P;
        if (k < FH)
          s2[u * FH + k] = make_double2(acc[2 * i], acc[2 * i + 1]);
      }
    }
  }
}

// Sum the unit partials of each channel in unit order, scale, mask, store.
// Partials hold the one-sided bins k <= L/2 (PSD partials hold A[k] + A[L-k],
// the pair average is the factor 1/2).  For real inputs the two-sided
// spectrum is the conjugate mirror: P[L-k] = conj(P[k]).
template <int MODE>
__global__ void spectral_finalize_kernel(const double *__restrict__ scratch,
                                         int64_t C, int64_t nq, int64_t L,
                                         int64_t F, double avg_scale,
                                         int onesided_mask, void *out,
                                         int64_t o_cs, int out_kind) {
  const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i >= C * F)
    return;
  const int64_t FH = L / 2 + 1;
  const int64_t c = i / F, k = i - c * F;
  const bool mirror = k >= FH;
  const int64_t kk = mirror ? L - k : k;
  double re = 0.0, im = 0.0;
  if (MODE == ACC_PSD) {
    for (int64_t q = 0; q < nq; ++q)
      re += scratch[(c * nq + q) * FH + kk];
    re *= 0.5;
  } else {
    const double2 *s2 = reinterpret_cast<const double2 *>(scratch);
    for (int64_t q = 0; q < nq; ++q) {
      const double2 v = s2[(c * nq + q) * FH + kk];
      re += v.x;
      im += v.y;
    }
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
      fft_group<T, L, E, P, G>(v, buf, t, g, p.tw);
#pragma unroll
      for (int e = 0; e < E; ++e)
        buf[spad(out_bin<L, E, P>(t, e))] = v[e];
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
      if (p.dc_mode == 1) {
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

} // namespace ib200

// spectral_istft.cuh — inverse STFT (overlap-add), reference
// ins::signal::istft (src/ops/signal/spectral_analysis.cpp:340-457).
//
// Per frame the reference rebuilds the full spectrum from the one-sided
// column (bins 1..F-2 mirrored as conjugates) when n_freq == nfft/2 + 1 and
// nfft > 2, takes Re(ifft(full, nfft)) (1/nfft scaling), truncates it to
// nperseg samples and multiplies by the window; the frames are overlap-added
// with hop = nperseg - noverlap and divided by the overlap-added squared
// window wherever that exceeds 1e-10.
//
// istft_frames_kernel: one task per pair of frames a, b (one-sided input):
// the Hermitian spectra A, B (imaginary parts of the DC and Nyquist bins
// dropped, which is what taking the real part does) are packed as Z = A + iB,
// so one complex inverse transform gives both real frames,
// IFFT(Z) = a + i b.  The inverse runs on the forward kernels:
// IFFT(Z) = conj(FFT(conj Z)) / nfft.  Other inputs (n_freq != nfft/2 + 1)
// take one frame per task and Re(IFFT(Z)) of the zero-padded / truncated
// column.  Windowed frames go to an f64 frame buffer [C][S][nperseg].
// The transforms run in f64 for complex64 input too: the overlap-add divides
// by the summed squared window, which is tiny where the window ends, so an
// f32 transform's rounding would be amplified there far above 1e-5.
// istft_ola_kernel: every output sample sums its frames in frame order and
// divides by the summed squared window (f64, as the reference).
#pragma once
#include "launch.h"
#include "spectral_kernels.cuh"

namespace ib200 {

template <typename T, typename TZ> struct IstftArgs {
  using VZ = typename V2T<TZ>::type;
  using V = typename V2T<T>::type;
  const VZ *z;           // Zxx, element (c, k, i) at z[c*z_cs + k*z_fs + i*z_ts]
  int64_t z_cs, z_fs, z_ts;
  int64_t C, F, S;       // channels, bins, frames
  int64_t nperseg;
  int pack;              // 1: Hermitian frame pairs, 0: one frame per task
  int64_t Tc;            // tasks per channel
  const T *win;          // [nperseg] window in T
  const V *tw;           // [L] W_L^m
  double *frames;        // [C][S][nperseg]
};

template <typename T, typename TZ, int L, int E, int G>
__global__ void __launch_bounds__(G *(L / E))
    istft_frames_kernel(const IstftArgs<T, TZ> p) {
  using V = typename V2T<T>::type;
  constexpr int P = L / E;
  constexpr int GS = spad_size(L);
  extern __shared__ __align__(16) unsigned char smem_raw[];
  V *buf = reinterpret_cast<V *>(smem_raw) + (threadIdx.x / P) * GS;
  const int g = threadIdx.x / P;
  const int t = threadIdx.x - g * P;
  const int64_t tpc = (p.Tc + G - 1) / G;
  const int64_t ntiles = p.C * tpc;
  const T inv = T(1) / T(L);

  for (int64_t tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
    const int64_t c = tile / tpc;
    const int64_t task = (tile - c * tpc) * G + g;
    if (task >= p.Tc)
      continue; // the whole group idles (no CTA-wide barrier below)
    const int64_t ia = p.pack ? 2 * task : task;
    const bool hasb = p.pack && ia + 1 < p.S;
    const auto *za = p.z + c * p.z_cs + ia * p.z_ts;
    auto ld = [&](int64_t i) -> V {
      const auto q = za[i];
      return V{(T)q.x, (T)q.y};
    };
    V v[E];
    static_for<0, E>([&](auto eIC) {
      constexpr int e = decltype(eIC)::value;
      const int k = in_index<L, E, P>(t, e);
      V zc;
      if (p.pack) {
        const bool mirror = k > L / 2;
        const int kk = mirror ? L - k : k;
        V a = ld(kk * p.z_fs);
        V b = hasb ? ld(kk * p.z_fs + p.z_ts) : V{T(0), T(0)};
        if (kk == 0 || kk == L / 2) {
          a.y = T(0);
          b.y = T(0);
        }
        if (mirror) {
          a.y = -a.y;
          b.y = -b.y;
        }
        zc = {a.x - b.y, -(a.y + b.x)}; // conj(A + iB)
      } else {
        zc = k < p.F ? ld(k * p.z_fs) : V{T(0), T(0)};
        zc.y = -zc.y;
      }
      v[e] = zc;
    });
    fft_group<T, L, E, P, G>(v, buf, t, g, p.tw);
    double *fa = p.frames + (c * p.S + ia) * p.nperseg;
    static_for<0, E>([&](auto eIC) {
      constexpr int e = decltype(eIC)::value;
      const int n = out_bin<L, E, P>(t, e);
      if (n < p.nperseg) {
        const T w = p.win[n];
        fa[n] = (double)(v[e].x * inv * w);
        if (hasb)
          fa[p.nperseg + n] = (double)(-v[e].y * inv * w);
      }
    });
  }
}

// out[c, m] = sum_i frames[c, i, m - i*hop] / sum_i w[m - i*hop]^2 over the
// frames i covering m (unchanged where the squared-window sum is <= 1e-10).
__global__ void istft_ola_kernel(const double *__restrict__ frames, int64_t C,
                                 int64_t S, int64_t nperseg, int64_t hop,
                                 int64_t n_total, const double *__restrict__ win,
                                 double *out, int64_t o_cs, int64_t o_ss) {
  const int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (idx >= C * n_total)
    return;
  const int64_t c = idx / n_total, m = idx - c * n_total;
  int64_t i0 = m - nperseg + 1 <= 0 ? 0 : (m - nperseg + hop) / hop;
  int64_t i1 = m / hop;
  if (i1 > S - 1)
    i1 = S - 1;
  double s = 0.0, nrm = 0.0;
  for (int64_t i = i0; i <= i1; ++i) {
    const int64_t n = m - i * hop;
    const double w = win[n];
    s += frames[(c * S + i) * nperseg + n];
    nrm += w * w;
  }
  if (fabs(nrm) > 1e-10)
    s /= nrm;
  out[c * o_cs + m * o_ss] = s;
}

template <typename T, typename TZ, int L>
cudaError_t run_istft_len(const IstftDesc &d, int num_sms, cudaStream_t stream,
                          int64_t *launches) {
  using V = typename V2T<T>::type;
  using VZ = typename V2T<TZ>::type;
  constexpr int E = values_per_thread<T>(L);
  constexpr int P = L / E;
  constexpr int G = (P >= 32 && P <= 256) ? 256 / P : 1;
  auto kern = istft_frames_kernel<T, TZ, L, E, G>;
  const size_t smem = (size_t)G * spad_size(L) * sizeof(V);
  static bool attr = false;
  if (!attr) {
    cudaError_t e = cudaFuncSetAttribute(
        kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess)
      return e;
    attr = true;
  }
  IstftArgs<T, TZ> a{};
  a.z = reinterpret_cast<const VZ *>(d.z);
  a.z_cs = d.z_cs;
  a.z_fs = d.z_fs;
  a.z_ts = d.z_ts;
  a.C = d.C;
  a.F = d.F;
  a.S = d.S;
  a.nperseg = d.nperseg;
  a.pack = d.pack ? 1 : 0;
  a.Tc = d.pack ? (d.S + 1) / 2 : d.S;
  a.win = reinterpret_cast<const T *>(d.win);
  a.tw = reinterpret_cast<const V *>(d.tw);
  a.frames = d.frames;
  const int64_t tiles = d.C * ((a.Tc + G - 1) / G);
  const int64_t grid = std::max<int64_t>(
      1, std::min<int64_t>(tiles, (int64_t)num_sms * 8));
  kern<<<(unsigned)grid, G * P, smem, stream>>>(a);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess)
    return e;
  const int64_t n = d.C * d.n_total;
  const int threads = 256;
  istft_ola_kernel<<<(unsigned)((n + threads - 1) / threads), threads, 0,
                     stream>>>(d.frames, d.C, d.S, d.nperseg, d.hop, d.n_total,
                               d.win64, d.out, d.o_cs, d.o_ss);
  if (launches)
    *launches += 2;
  return cudaGetLastError();
}

template <typename T, typename TZ>
cudaError_t run_istft_t(const IstftDesc &d, int num_sms, cudaStream_t stream,
                        int64_t *launches) {
  switch (d.nfft) {
  case 16: return run_istft_len<T, TZ, 16>(d, num_sms, stream, launches);
  case 32: return run_istft_len<T, TZ, 32>(d, num_sms, stream, launches);
  case 64: return run_istft_len<T, TZ, 64>(d, num_sms, stream, launches);
  case 128: return run_istft_len<T, TZ, 128>(d, num_sms, stream, launches);
  case 256: return run_istft_len<T, TZ, 256>(d, num_sms, stream, launches);
  case 512: return run_istft_len<T, TZ, 512>(d, num_sms, stream, launches);
  case 1024: return run_istft_len<T, TZ, 1024>(d, num_sms, stream, launches);
  case 2048: return run_istft_len<T, TZ, 2048>(d, num_sms, stream, launches);
  case 4096: return run_istft_len<T, TZ, 4096>(d, num_sms, stream, launches);
  case 8192: return run_istft_len<T, TZ, 8192>(d, num_sms, stream, launches);
  default: return cudaErrorInvalidValue;
  }
}

} // namespace ib200

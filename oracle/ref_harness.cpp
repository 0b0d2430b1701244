// oracle/ref_harness.cpp — test infrastructure, never shipped.
//
// Drives the reference's own spectral frontend (ins::signal::welch / csd /
// spectrogram / stft in src/ops/signal/spectral_analysis.cpp) from plain C
// entry points so Python tests and the CPU baseline can call it with ctypes.
//
// The reference registers its CPU "fft" kernel only when FFTW3 is present
// (backends/cpu/kernels/fft/fft_c2c.cpp:23,68-71).  FFTW3 is not installed
// here, so this file registers a substitute "fft" kernel for F32/F64/C32/C64
// through the reference's public C ABI (insight_register_kernel,
// include/insight/c_api/kernel.h:35), with the same argument layout as
// fft_c2c_kernel_cpu (fft_c2c.cpp:9-16):
//   inputs  = {out, x, &fft_len, &batch, &inverse, &real_input, &norm, NULL}
//   outputs = {out, NULL}
// The substitute computes the unnormalised DFT
//   X[k] = sum_n x[n] exp(-2*pi*i*k*n/N)   (FFTW_FORWARD convention)
// with an iterative radix-2 Cooley-Tukey for powers of two and a direct
// O(N^2) DFT otherwise, in the precision of the input dtype (float for C32,
// double for C64), as FFTW's fftwf_/fftw_ families do.  Twiddles are
// evaluated in double and rounded once.
#include "insight/c_api/array.h"
#include "insight/c_api/kernel.h"
#include "insight/c_api/place.h"
#include "insight/core/array.h"
#include "insight/core/op_registry.h"
#include "insight/init.h"
#include "insight/ops/creation.h"
#include "insight/ops/signal/spectral_analysis.h"
#include "insight/ops/signal/windows.h"

#include <omp.h>

#include <cmath>
#include <complex>
#include <cstring>
#include <string>
#include <vector>

namespace {

thread_local std::string g_err;

template <typename T>
void dft_inplace(std::complex<T> *a, int64_t n, int inverse) {
  const double sgn = inverse ? 1.0 : -1.0;
  if (n <= 1)
    return;
  if ((n & (n - 1)) == 0) {
    // bit reversal
    for (int64_t i = 1, j = 0; i < n; ++i) {
      int64_t bit = n >> 1;
      for (; j & bit; bit >>= 1)
        j ^= bit;
      j ^= bit;
      if (i < j)
        std::swap(a[i], a[j]);
    }
    for (int64_t len = 2; len <= n; len <<= 1) {
      const int64_t half = len / 2;
      std::vector<std::complex<T>> w(half);
      for (int64_t k = 0; k < half; ++k) {
        double ang = sgn * 2.0 * M_PI * (double)k / (double)len;
        w[k] = std::complex<T>((T)std::cos(ang), (T)std::sin(ang));
      }
      for (int64_t i = 0; i < n; i += len) {
        for (int64_t k = 0; k < half; ++k) {
          std::complex<T> u = a[i + k];
          std::complex<T> v = a[i + k + half] * w[k];
          a[i + k] = u + v;
          a[i + k + half] = u - v;
        }
      }
    }
    return;
  }
  std::vector<std::complex<T>> out(n);
  for (int64_t k = 0; k < n; ++k) {
    std::complex<double> acc(0.0, 0.0);
    for (int64_t m = 0; m < n; ++m) {
      double ang = sgn * 2.0 * M_PI * (double)((k * m) % n) / (double)n;
      acc += std::complex<double>(a[m]) * std::complex<double>(std::cos(ang), std::sin(ang));
    }
    out[k] = std::complex<T>(acc);
  }
  std::memcpy((void *)a, out.data(), sizeof(std::complex<T>) * n);
}

C_Status substitute_fft_kernel(void **inputs, void **outputs) {
  InsightArray *out = (InsightArray *)outputs[0];
  InsightArray *x = (InsightArray *)inputs[1];
  int64_t fft_len = *(int64_t *)inputs[2];
  int64_t batch = *(int64_t *)inputs[3];
  int inverse = *(int *)inputs[4];
  if (!out || !x)
    return C_FAILED;
  int64_t total = fft_len * batch;
  if (x->dtype == INSIGHT_DTYPE_F64 || x->dtype == INSIGHT_DTYPE_C64) {
    auto *d = (std::complex<double> *)out->data;
    std::memcpy(d, x->data, total * sizeof(std::complex<double>));
    for (int64_t b = 0; b < batch; ++b)
      dft_inplace<double>(d + b * fft_len, fft_len, inverse);
  } else if (x->dtype == INSIGHT_DTYPE_F32 || x->dtype == INSIGHT_DTYPE_C32) {
    auto *d = (std::complex<float> *)out->data;
    std::memcpy(d, x->data, total * sizeof(std::complex<float>));
    for (int64_t b = 0; b < batch; ++b)
      dft_inplace<float>(d + b * fft_len, fft_len, inverse);
  } else {
    return C_FAILED;
  }
  return C_SUCCESS;
}

ins::Array make_input(const void *x, int64_t n, int dtype) {
  if (dtype == INSIGHT_DTYPE_F32)
    return ins::to_array((const float *)x, ins::Shape({n}), ins::CPUPlace());
  return ins::to_array((const double *)x, ins::Shape({n}), ins::CPUPlace());
}

int64_t copy_out(const ins::Array &a, double *dst, int64_t cap) {
  ins::Array c = a.to(ins::CPUPlace()).contiguous();
  if (c.dtype() != ins::DType::F64)
    c = c.to(ins::DType::F64);
  int64_t n = c.numel();
  if (dst && n <= cap)
    std::memcpy(dst, c.data<double>(), n * sizeof(double));
  return n;
}

} // namespace

extern "C" {

const char *ref_last_error(void) { return g_err.c_str(); }

// OpenMP threads of the reference's parallel loops on the calling thread
// (a launcher such as torchrun may have set OMP_NUM_THREADS=1 already).
int ref_set_threads(int n) {
  if (n > 0)
    omp_set_num_threads(n);
  return omp_get_max_threads();
}

int ref_init(const char *backend_dir) {
  try {
    if (backend_dir && backend_dir[0])
      ins::add_backend_search_path(backend_dir);
    if (!ins::is_initialized())
      ins::init(std::vector<std::string>{"cpu"});
    const int32_t dts[4] = {INSIGHT_DTYPE_F32, INSIGHT_DTYPE_F64,
                            INSIGHT_DTYPE_C32, INSIGHT_DTYPE_C64};
    for (int32_t dt : dts)
      if (!insight_has_kernel("fft", INSIGHT_DEVICE_CPU, dt))
        insight_register_kernel("fft", INSIGHT_DEVICE_CPU, dt,
                                substitute_fft_kernel);
    return 0;
  } catch (const std::exception &e) {
    g_err = e.what();
    return 1;
  }
}

// Pxy/Pxx of the reference csd (x != y) or welch (y == NULL).
int ref_csd(const void *x, const void *y, int64_t n, int dtype, double fs,
            const char *window, int64_t nperseg, int64_t noverlap, int64_t nfft,
            const char *detrend, int onesided, const char *scaling,
            double *f_out, double *p_out, int64_t cap, int64_t *n_freq) {
  try {
    ins::Array xa = make_input(x, n, dtype);
    ins::signal::SpectralResult r =
        y ? ins::signal::csd(xa, make_input(y, n, dtype), fs, window, nperseg,
                             noverlap, nfft, detrend, onesided != 0, scaling)
          : ins::signal::welch(xa, fs, window, nperseg, noverlap, nfft,
                               detrend, onesided != 0, scaling);
    *n_freq = copy_out(r.f, f_out, cap);
    copy_out(r.Pxx, p_out, cap);
    return 0;
  } catch (const std::exception &e) {
    g_err = e.what();
    return 1;
  }
}

// Reference coherence(x, y) (mode 1) or periodogram(x) (mode 2; nperseg and
// noverlap are not arguments of the reference's periodogram).
int ref_coherence(const void *x, const void *y, int64_t n, int dtype, int mode,
                  double fs, const char *window, int64_t nperseg,
                  int64_t noverlap, int64_t nfft, const char *detrend,
                  int onesided, const char *scaling, double *f_out,
                  double *p_out, int64_t cap, int64_t *n_freq) {
  try {
    ins::Array xa = make_input(x, n, dtype);
    ins::signal::SpectralResult r =
        mode == 1 ? ins::signal::coherence(xa, make_input(y, n, dtype), fs, window,
                                           nperseg, noverlap, nfft, detrend)
                  : ins::signal::periodogram(xa, fs, window, nfft, detrend,
                                             onesided != 0, scaling);
    *n_freq = copy_out(r.f, f_out, cap);
    copy_out(r.Pxx, p_out, cap);
    return 0;
  } catch (const std::exception &e) {
    g_err = e.what();
    return 1;
  }
}

// Reference istft of a C64 (n_freq, n_frames) row-major Zxx given as
// interleaved (re, im) doubles.
int ref_istft(const double *z, int64_t n_freq, int64_t n_frames,
              const char *window, int64_t nperseg, int64_t noverlap,
              int64_t nfft, double *out, int64_t cap, int64_t *n_out) {
  try {
    std::vector<std::complex<double>> zc(n_freq * n_frames);
    for (size_t i = 0; i < zc.size(); ++i)
      zc[i] = std::complex<double>(z[2 * i], z[2 * i + 1]);
    ins::Array za = ins::to_array(zc, ins::Shape({n_freq, n_frames}),
                                  ins::CPUPlace());
    ins::Array r = ins::signal::istft(za, 1.0, window, nperseg, noverlap, nfft);
    *n_out = copy_out(r, out, cap);
    return 0;
  } catch (const std::exception &e) {
    g_err = e.what();
    return 1;
  }
}

// Reference spectrogram; S is returned (n_seg, n_freq) row-major (the
// reference returns a transposed view of an (n_freq, n_seg) buffer).
int ref_spectrogram(const void *x, int64_t n, int dtype, double fs,
                    const char *window, int64_t nperseg, int64_t noverlap,
                    int64_t nfft, const char *detrend, int onesided,
                    const char *mode, int is_stft, double *f_out,
                    double *t_out, double *s_out, int64_t cap, int64_t *n_seg,
                    int64_t *n_freq) {
  try {
    ins::Array xa = make_input(x, n, dtype);
    ins::signal::SpectrogramResult r =
        is_stft ? ins::signal::stft(xa, fs, window, nperseg, noverlap, nfft)
                : ins::signal::spectrogram(xa, fs, window, nperseg, noverlap,
                                           nfft, detrend, onesided != 0, mode);
    *n_freq = copy_out(r.f, f_out, cap);
    *n_seg = copy_out(r.t, t_out, cap);
    copy_out(r.Sxx, s_out, cap);
    return 0;
  } catch (const std::exception &e) {
    g_err = e.what();
    return 1;
  }
}

// ---------------------------------------------------------------------------
// The B200 plugin reached only through the reference's own core.
//
// ref_load_gpu_backend: the reference's loader (src/init.cpp: load_backend ->
// try_load_backend) finds libinsight_<name>_backend.so in search_dir, calls
// its InitPluginGPU with the core's insight_register_kernel, installs the
// C_DeviceInterface it fills and initialises device 0.  The calling thread's
// default place is then set back to the CPU so the reference's CPU
// composites above keep computing on the CPU (the core would otherwise make
// GPUPlace(0) the default once a GPU backend is present,
// src/core/place.cpp:252-261).
int ref_load_gpu_backend(const char *search_dir, const char *name) {
  try {
    if (search_dir && search_dir[0])
      ins::add_backend_search_path(search_dir);
    ins::load_backend(name);
    if (!ins::has_device(ins::DeviceKind::GPU)) {
      g_err = std::string("the core did not load libinsight_") + name +
              "_backend as its GPU backend";
      return 1;
    }
    ins::set_device(ins::CPUPlace());
    return 0;
  } catch (const std::exception &e) {
    g_err = e.what();
    return 1;
  }
}

// insight_has_kernel of the core's registry for a GPU kernel.
int ref_has_gpu_kernel(const char *op, int dtype) {
  return insight_has_kernel(op, INSIGHT_DEVICE_GPU, dtype);
}

namespace {

// compute_psd_scale (spectral_analysis.cpp:57-67): (fs or 1) / sum(w^2), the
// window taken in the input dtype.
double psd_scale_of(const ins::Array &win_cpu, int dtype, double fs,
                    const std::string &scaling) {
  ins::Array w = win_cpu.contiguous();
  const double *wv = w.data<double>();
  double ss = 0.0;
  for (int64_t i = 0; i < w.numel(); ++i) {
    const double v = dtype == INSIGHT_DTYPE_F32 ? (double)(float)wv[i] : wv[i];
    ss += v * v;
  }
  return (scaling == "density" ? fs : 1.0) / ss;
}

} // namespace

// The GPU branch a maintainer adds at the top of the reference's csd / welch
// / coherence (op = "csd", "welch" or "coherence"): inputs moved to
// GPUPlace(0) by the core's Array::to (the plugin's device interface does
// the allocation and the copy), the window made by the reference's own
// get_window and moved to the GPU, the output allocated on the GPU by the
// core, the kernel launched by ops().launch with the registry layout, and
// the result brought back by Array::to(CPUPlace()).
int ref_gpu_csd(const char *op, const void *x, const void *y, int64_t n,
                int dtype, double fs, const char *window, int64_t nperseg,
                int64_t noverlap, int64_t nfft, const char *detrend,
                int onesided, const char *scaling, double *f_out,
                double *p_out, int64_t cap, int64_t *n_freq) {
  try {
    const ins::Place gpu = ins::GPUPlace(0);
    ins::Array xg = make_input(x, n, dtype).to(gpu);
    ins::Array yg = y ? make_input(y, n, dtype).to(gpu) : xg;
    if (nfft == 0)
      nfft = nperseg;
    if (noverlap == 0)
      noverlap = nperseg / 2;
    ins::Array win = ins::signal::get_window(window, nperseg, false);
    const double scale = psd_scale_of(win.to(ins::CPUPlace()), dtype, fs, scaling);
    ins::Array wg = win.to(gpu);
    const int64_t F = onesided ? nfft / 2 + 1 : nfft;
    ins::Array P(ins::Shape({F}), ins::DType::F64, gpu); // every bin is written
    int32_t dcode = std::string(detrend) == "constant" ? 1 : 0;
    int32_t os = onesided ? 1 : 0;
    double sc = scale;
    int64_t axis = -1;
    ins::ops().launch(op, gpu, xg.dtype(),
                      {P.layout_ptr(), xg.layout_ptr(), yg.layout_ptr(),
                       wg.layout_ptr(), &nperseg, &noverlap, &nfft, &dcode, &os,
                       &sc, &axis},
                      {P.layout_ptr()});
    *n_freq = F;
    for (int64_t i = 0; i < F && i < cap; ++i)
      f_out[i] = (double)i * (fs / (double)nfft);
    copy_out(P, p_out, cap);
    return 0;
  } catch (const std::exception &e) {
    g_err = e.what();
    return 1;
  }
}

// The GPU branch of the reference's stft (spectrogram with mode complex,
// detrend none, one-sided): the (n_freq, n_seg) F64 buffer of Re(X) that the
// reference builds before its transposed view, written by the registered
// "stft" kernel and returned as that (n_freq, n_seg) row-major buffer.
int ref_gpu_stft(const void *x, int64_t n, int dtype, double fs,
                 const char *window, int64_t nperseg, int64_t noverlap,
                 int64_t nfft, double *s_out, int64_t cap, int64_t *n_seg,
                 int64_t *n_freq) {
  try {
    const ins::Place gpu = ins::GPUPlace(0);
    ins::Array xg = make_input(x, n, dtype).to(gpu);
    if (nfft == 0)
      nfft = nperseg;
    if (noverlap == 0)
      noverlap = nperseg / 8;
    const int64_t step = nperseg - noverlap;
    const int64_t S = n >= nperseg ? (n - nperseg) / step + 1 : 0;
    const int64_t F = nfft / 2 + 1;
    ins::Array wg = ins::signal::get_window(window, nperseg, false).to(gpu);
    // the (n_freq, n_seg) buffer, passed as the (n_seg, n_freq) transposed
    // view the reference returns (spectral_analysis.cpp:256,321)
    ins::Array out(ins::Shape({F, S}), ins::DType::F64, gpu); // fully written
    ins::Array view = out.transpose({1, 0});
    int32_t dcode = 0, os = 1, mode = 1;
    double sc = 1.0;
    int64_t axis = -1;
    ins::ops().launch("stft", gpu, xg.dtype(),
                      {view.layout_ptr(), xg.layout_ptr(), wg.layout_ptr(),
                       &nperseg, &noverlap, &nfft, &dcode, &os, &mode, &sc,
                       &axis},
                      {view.layout_ptr()});
    *n_seg = S;
    *n_freq = F;
    copy_out(out, s_out, cap);
    return 0;
  } catch (const std::exception &e) {
    g_err = e.what();
    return 1;
  }
}

} // extern "C"

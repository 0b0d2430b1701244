// spectral_noalloc.cu — welch for callers that cannot allocate device memory.
//
// Some callers own every byte of device memory themselves: a host framework
// that hands out all GPU buffers from its own pool (an Insight Place
// allocator, a caching allocator) and forbids libraries from calling
// cudaMalloc behind its back, or a latency-critical path where the implicit
// device synchronisation of cudaMalloc / cudaFree is not acceptable.  For them
// insight_b200_welch_noalloc runs the same fused welch kernels as
// insight_b200_welch, but takes device pointers for the input and the result
// and allocates nothing: the kernels' working memory (twiddles, the window and
// the per-work-unit partial sums) lives in the file-scope array below.
//
// The array is NOALLOC_SCRATCH_BYTES (8 MiB) of device memory that every GPU
// which loads this library holds until the process exits.  It is shared by
// all calls on a device and keeps the last call's contents; each call
// rewrites the tables it uses and every partial-sum slot it reads, so nothing
// has to start at zero.  Calls that overlap on the same GPU (other host
// threads, other streams) race on it.
#include "frontend.h"
#include "launch.h"
#include "windows.h"

#include <cmath>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#ifndef M_PI
#define M_PI 3.14159265358979323846
#endif

namespace {

constexpr size_t NOALLOC_SCRATCH_BYTES = size_t(8) << 20;
constexpr int MAX_DEVICES = 64;

static __device__ __align__(256) unsigned char g_noalloc_scratch[NOALLOC_SCRATCH_BYTES];

std::mutex g_mu;
void *g_scratch_ptr[MAX_DEVICES] = {};

// Device address of the scratch array on the current device.  In host code
// g_noalloc_scratch names a host-side stand-in, so the address is looked up
// once per device (with that device current) and cached.
void *scratch_address(int dev, std::string &err) {
  if (dev < 0 || dev >= MAX_DEVICES) {
    err = "welch_noalloc: device index out of range";
    return nullptr;
  }
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_scratch_ptr[dev]) {
    void *p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) {
      err = std::string("welch_noalloc: cudaGetSymbolAddress: ") +
            cudaGetErrorString(e);
      return nullptr;
    }
    g_scratch_ptr[dev] = p;
  }
  return g_scratch_ptr[dev];
}

size_t align256(size_t n) { return (n + 255) & ~size_t(255); }

} // namespace

extern "C" __attribute__((visibility("default"))) C_Status
insight_b200_welch_noalloc(const void *x, int32_t dtype, int64_t n_channels,
                           int64_t n_samples, int64_t channel_stride,
                           int64_t sample_stride, double fs, const char *window,
                           int64_t nperseg, int64_t noverlap, int64_t nfft,
                           const char *detrend, int32_t return_onesided,
                           const char *scaling, double *pxx, void *stream) {
  using ib200::set_last_error;
  const cudaStream_t st = (cudaStream_t)stream;
  if (!x || !pxx) {
    set_last_error("welch_noalloc: inputs are undefined");
    return C_FAILED;
  }
  if (dtype != INSIGHT_DTYPE_F32 && dtype != INSIGHT_DTYPE_F64) {
    set_last_error("welch_noalloc: dtype must be F32 or F64");
    return C_FAILED;
  }
  if (n_channels < 1 || sample_stride < 1 || channel_stride < 0) {
    set_last_error("welch_noalloc: need n_channels >= 1, sample_stride >= 1, "
                   "channel_stride >= 0");
    return C_FAILED;
  }
  if (nperseg <= 0) {
    set_last_error("welch_noalloc: nperseg must be positive");
    return C_FAILED;
  }
  // Defaults and framing as the reference csd (spectral_analysis.cpp:114-125).
  if (nfft == 0)
    nfft = nperseg;
  if (noverlap == 0)
    noverlap = nperseg / 2;
  const int64_t step = nperseg - noverlap;
  if (step <= 0) {
    set_last_error("welch_noalloc: noverlap must be less than nperseg");
    return C_FAILED;
  }
  const int64_t S =
      (n_samples >= nperseg) ? ((n_samples - nperseg) / step + 1) : 0;
  if (S < 1) {
    set_last_error("welch_noalloc: signal too short for given nperseg");
    return C_FAILED;
  }
  if (!ib200::nfft_supported(nfft) || nfft < nperseg) {
    set_last_error("welch_noalloc: nfft must be a power of two in [16, 8192] "
                   "and >= nperseg on the B200 backend");
    return C_FAILED;
  }
  std::vector<double> w;
  try {
    w = ib200::get_window(window ? window : "hann", nperseg, false);
  } catch (const std::exception &e) {
    set_last_error(e.what());
    return C_FAILED;
  }
  const bool constant = detrend && std::string(detrend) == "constant";
  if (constant && nfft != nperseg) {
    set_last_error("welch_noalloc: detrend='constant' needs nfft == nperseg "
                   "(zero padding with constant detrend uses a device table "
                   "that this entry point does not hold)");
    return C_FAILED;
  }
  const bool f64 = dtype == INSIGHT_DTYPE_F64;
  const bool onesided = return_onesided != 0;
  const int64_t F = onesided ? nfft / 2 + 1 : nfft;
  const int64_t FH = nfft / 2 + 1;

  // Layout of the scratch array: [twiddles | window | unit partial sums].
  const size_t tsz = f64 ? 8 : 4;
  const size_t tw_off = 0;
  const size_t win_off = align256(tw_off + (size_t)nfft * 2 * tsz);
  const size_t part_off = align256(win_off + (size_t)nfft * tsz);
  const size_t per_unit = (size_t)FH * 8;
  const int64_t max_units =
      part_off < NOALLOC_SCRATCH_BYTES
          ? (int64_t)((NOALLOC_SCRATCH_BYTES - part_off) / per_unit)
          : 0;
  if (max_units < n_channels) {
    set_last_error("welch_noalloc: n_channels * (nfft/2 + 1) * 8 bytes of partial "
                   "sums exceed the 8 MiB scratch of the no-allocation entry "
                   "point; use insight_b200_welch or fewer channels per call");
    return C_FAILED;
  }

  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    set_last_error(std::string("welch_noalloc: ") + cudaGetErrorString(e));
    return C_FAILED;
  }
  std::string err;
  unsigned char *base = (unsigned char *)scratch_address(dev, err);
  if (!base) {
    set_last_error(err);
    return C_FAILED;
  }
  int num_sms = 0;
  e = cudaDeviceGetAttribute(&num_sms, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess || num_sms < 1) {
    set_last_error(std::string("welch_noalloc: multiprocessor count: ") +
                   cudaGetErrorString(e));
    return C_FAILED;
  }

  // Tables on the host, copied into the scratch array on the caller's stream
  // (the copies from pageable memory have left the host buffers on return).
  std::vector<unsigned char> tw((size_t)nfft * 2 * tsz), win((size_t)nfft * tsz, 0);
  double wss = 0.0;
  for (int64_t m = 0; m < nfft; ++m) {
    const double a = 2.0 * M_PI * (double)m / (double)nfft;
    if (f64) {
      reinterpret_cast<double *>(tw.data())[2 * m] = std::cos(a);
      reinterpret_cast<double *>(tw.data())[2 * m + 1] = -std::sin(a);
    } else {
      reinterpret_cast<float *>(tw.data())[2 * m] = (float)std::cos(a);
      reinterpret_cast<float *>(tw.data())[2 * m + 1] = (float)-std::sin(a);
    }
  }
  for (int64_t i = 0; i < nperseg; ++i) {
    const double v = f64 ? w[i] : (double)(float)w[i];
    wss += v * v;
    if (f64)
      reinterpret_cast<double *>(win.data())[i] = w[i];
    else
      reinterpret_cast<float *>(win.data())[i] = (float)w[i];
  }
  // Every check that can reject the call is done above: from here on a
  // failure first waits for what this call queued, so no copy of a failed
  // call is still writing the shared array when the call returns.
  e = cudaMemcpyAsync(base + tw_off, tw.data(), tw.size(), cudaMemcpyHostToDevice, st);
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(base + win_off, win.data(), win.size(),
                        cudaMemcpyHostToDevice, st);
  if (e != cudaSuccess) {
    cudaStreamSynchronize(st);
    set_last_error(std::string("welch_noalloc: ") + cudaGetErrorString(e));
    return C_FAILED;
  }

  const double scale =
      ((scaling && std::string(scaling) != "density") ? 1.0 : fs) / wss;

  ib200::LaunchDesc d;
  d.kind = ib200::LK_PSD;
  d.f64 = f64;
  d.nfft = nfft;
  d.nperseg = nperseg;
  d.step = step;
  d.C = n_channels;
  d.seg0 = 0;
  d.S = S;
  d.x = x;
  d.x_cs = channel_stride;
  d.x_ss = sample_stride;
  d.win = base + win_off;
  d.tw = base + tw_off;
  d.dtab = nullptr;
  d.dc_mode = !constant ? 0 : 1;
  d.F = F;
  d.onesided_mask = onesided && nfft > 1;
  d.avg_scale = scale / (double)S;
  d.out_kind = ib200::OUT_REAL_F64_K;
  d.out = pxx;
  d.o_cs = F;
  d.max_units = max_units;
  int64_t nl = 0;
  e = ib200::launch(d, base + part_off, num_sms, st, &nl);
  ib200::add_launches(nl);
  const cudaError_t es = cudaStreamSynchronize(st);
  if (e == cudaSuccess)
    e = es;
  if (e != cudaSuccess) {
    set_last_error(std::string("welch_noalloc: ") + cudaGetErrorString(e));
    return C_FAILED;
  }
  return C_SUCCESS;
}

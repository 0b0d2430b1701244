// frontend.cpp — host side of the B200 spectral backend.
//
// Mirrors the reference frontend ins::signal::{csd, welch, spectrogram, stft}
// (src/ops/signal/spectral_analysis.cpp:104-334): argument defaults, framing,
// window and scale, result arrays and error messages.  Instead of the
// reference's per-segment composite loop (~25 registry ops per segment) it
// plans one launch of the fused kernel family (spectral_kernels.cuh) over
// every segment of every channel.
//
// Differences from the reference, all deliberate:
//  * F32 welch/csd/spectrogram('psd') work (the reference throws in
//    compute_psd_scale, :63, because it calls item<double>() on an F32 sum);
//    the scale is computed in F64 from the F32-rounded window.
//  * 2-D inputs are a batch of channels (the reference accepts 1-D only).
//  * nfft must be a power of two in [16, 8192] and >= nperseg; noverlap must
//    be < nperseg (the reference divides by a non-positive step otherwise).
#include "frontend.h"
#include "launch.h"
#include "windows.h"

#include <atomic>
#include <cmath>
#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <sstream>
#include <vector>

#ifndef M_PI
#define M_PI 3.14159265358979323846
#endif

namespace ib200 {

namespace {
thread_local std::string g_last_error;
std::atomic<int64_t> g_launches{0};
// True while this thread captures a call into a plan's CUDA graph: the call
// then only enqueues kernels (its tables and buffers were made by the plan's
// warm-up run), without event waits, event records or allocations.
thread_local bool g_capturing = false;
} // namespace

void set_last_error(const std::string &msg) { g_last_error = msg; }
const char *last_error() { return g_last_error.c_str(); }
int64_t launch_count() { return g_launches.load(); }
void add_launches(int64_t n) { g_launches += n; }

struct Fail : std::runtime_error {
  using std::runtime_error::runtime_error;
};

static void check(bool ok, const std::string &msg) {
  if (!ok)
    throw Fail(msg);
}

static void cuda_check(cudaError_t e, const char *what) {
  if (e != cudaSuccess) {
    std::ostringstream o;
    o << what << ": " << cudaGetErrorString(e);
    throw Fail(o.str());
  }
}

// ---------------------------------------------------------------------------
// Per-device state: stream, grow-only buffers, constant tables.
// ---------------------------------------------------------------------------
namespace {

struct DevBuf {
  void *p = nullptr;
  size_t n = 0;
};

// A constant table: device copy, the host bytes it was copied from (kept so
// the asynchronous upload never reads freed memory) and an event recorded
// after the upload on the stream that made it; users on any stream wait for
// that event instead of synchronising the host.
struct Table {
  DevBuf buf;
  std::vector<unsigned char> host;
  cudaEvent_t ready = nullptr;
};

// Working buffers a launch reads and writes on the device (welch/csd partial
// sums, istft frames), one set per stream: calls on different streams never
// share them, so asynchronous calls on two streams can run at the same time.
// `last` is recorded after each use; a later use waits for it, which keeps a
// set correct even if its stream handle is reused by a new stream.
struct StreamBufs {
  DevBuf scratch, frames;
  cudaEvent_t last = nullptr;
};

struct DeviceState {
  int dev = 0;
  int num_sms = 0;
  cudaStream_t stream = nullptr;
  // host-I/O pipeline: channel chunks alternate over these streams so the
  // host->device copy of one chunk, the kernel of another and the
  // device->host copy of a third overlap (PCIe is full duplex)
  static constexpr int kPipe = 3;
  cudaStream_t pipe[kPipe] = {};
  cudaEvent_t pipe_start = nullptr;
  std::mutex mu;
  // staging of host inputs / outputs: used only by calls that synchronise
  // their stream before returning
  DevBuf xin, yin, out, win_tmp;
  std::map<cudaStream_t, StreamBufs> per_stream;
  std::map<std::string, Table> tables;
};

std::mutex g_states_mu;
std::map<int, std::unique_ptr<DeviceState>> g_states;

DeviceState &device_state(int dev) {
  std::lock_guard<std::mutex> lk(g_states_mu);
  auto &slot = g_states[dev];
  if (!slot) {
    auto st = std::make_unique<DeviceState>();
    st->dev = dev;
    cuda_check(cudaSetDevice(dev), "cudaSetDevice");
    cuda_check(cudaDeviceGetAttribute(&st->num_sms,
                                      cudaDevAttrMultiProcessorCount, dev),
               "cudaDeviceGetAttribute");
    int major = 0;
    cuda_check(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor,
                                      dev),
               "cudaDeviceGetAttribute");
    check(major == 10, "insight_b200: device " + std::to_string(dev) +
                           " is not an sm_100 (B200) GPU");
    cuda_check(cudaStreamCreateWithFlags(&st->stream, cudaStreamNonBlocking),
               "cudaStreamCreate");
    slot = std::move(st);
  }
  return *slot;
}

// Grow-only buffer, stream-ordered: the old block is released and the new
// one taken on `stream` (cudaFreeAsync / cudaMallocAsync), after the work
// already queued there, without synchronising the device.
void ensure(DevBuf &b, size_t bytes, cudaStream_t stream) {
  if (b.n >= bytes && b.p)
    return;
  check(!g_capturing, "plan: a buffer would grow while the call is captured");
  if (b.p) {
    cuda_check(cudaFreeAsync(b.p, stream), "cudaFreeAsync");
    b.p = nullptr;
    b.n = 0;
  }
  size_t n = std::max<size_t>(bytes, 256);
  cuda_check(cudaMallocAsync(&b.p, n, stream), "cudaMallocAsync");
  b.n = n;
}

// The per-stream working buffers of `stream`, ordered after their last use.
StreamBufs &stream_bufs(DeviceState &st, cudaStream_t stream) {
  StreamBufs &sb = st.per_stream[stream];
  if (g_capturing)
    return sb;
  if (!sb.last)
    cuda_check(cudaEventCreateWithFlags(&sb.last, cudaEventDisableTiming),
               "cudaEventCreate");
  else
    cuda_check(cudaStreamWaitEvent(stream, sb.last, 0), "cudaStreamWaitEvent");
  return sb;
}

void mark_used(StreamBufs &sb, cudaStream_t stream) {
  if (!g_capturing)
    cuda_check(cudaEventRecord(sb.last, stream), "cudaEventRecord");
}

size_t dtype_size(int32_t dt) {
  switch (dt) {
  case INSIGHT_DTYPE_F32: return 4;
  case INSIGHT_DTYPE_F64: return 8;
  case INSIGHT_DTYPE_C32: return 8;
  case INSIGHT_DTYPE_C64: return 16;
  default: return 0;
  }
}

template <typename T>
std::vector<unsigned char> pack_complex(const std::vector<double> &re,
                                        const std::vector<double> &im) {
  std::vector<unsigned char> b(re.size() * 2 * sizeof(T));
  T *p = reinterpret_cast<T *>(b.data());
  for (size_t i = 0; i < re.size(); ++i) {
    p[2 * i] = (T)re[i];
    p[2 * i + 1] = (T)im[i];
  }
  return b;
}

// Constant table `key`, uploaded on first use with an asynchronous copy on
// the call's stream; every use makes the call's stream wait for the upload.
const void *table(DeviceState &st, const std::string &key,
                  std::vector<unsigned char> bytes, cudaStream_t stream) {
  auto it = st.tables.find(key);
  if (it != st.tables.end()) {
    if (!g_capturing)
      cuda_check(cudaStreamWaitEvent(stream, it->second.ready, 0),
                 "cudaStreamWaitEvent");
    return it->second.buf.p;
  }
  check(!g_capturing, "plan: a table would be uploaded while the call is captured");
  Table &t = st.tables[key];
  t.host = std::move(bytes);
  ensure(t.buf, t.host.size(), stream);
  cuda_check(cudaMemcpyAsync(t.buf.p, t.host.data(), t.host.size(),
                             cudaMemcpyHostToDevice, stream),
             "cudaMemcpyAsync");
  cuda_check(cudaEventCreateWithFlags(&t.ready, cudaEventDisableTiming),
             "cudaEventCreate");
  cuda_check(cudaEventRecord(t.ready, stream), "cudaEventRecord");
  return t.buf.p;
}

// W_L^m = exp(-2 pi i m / L), evaluated in double.
const void *twiddles(DeviceState &st, int64_t L, bool f64, cudaStream_t stream) {
  std::vector<double> re(L), im(L);
  for (int64_t m = 0; m < L; ++m) {
    const double a = 2.0 * M_PI * (double)m / (double)L;
    re[m] = std::cos(a);
    im[m] = -std::sin(a);
  }
  std::string key = std::string("tw|") + (f64 ? "d|" : "f|") + std::to_string(L);
  return table(st, key,
               f64 ? pack_complex<double>(re, im) : pack_complex<float>(re, im),
               stream);
}

// D[k] = sum_{n < M} W_L^{nk} = (1 - W^{kM}) / (1 - W^k), D[0] = M.
const void *dc_table(DeviceState &st, int64_t L, int64_t M, bool f64,
                     cudaStream_t stream) {
  std::vector<double> re(L), im(L);
  for (int64_t k = 0; k < L; ++k) {
    if (k == 0) {
      re[k] = (double)M;
      im[k] = 0.0;
      continue;
    }
    const double a1 = -2.0 * M_PI * (double)k / (double)L;
    const double aM = -2.0 * M_PI * (double)((k * M) % L) / (double)L;
    const double nr = 1.0 - std::cos(aM), ni = -std::sin(aM);
    const double dr = 1.0 - std::cos(a1), di = -std::sin(a1);
    const double den = dr * dr + di * di;
    re[k] = (nr * dr + ni * di) / den;
    im[k] = (ni * dr - nr * di) / den;
  }
  std::string key = std::string("dc|") + (f64 ? "d|" : "f|") +
                    std::to_string(L) + "|" + std::to_string(M);
  return table(st, key,
               f64 ? pack_complex<double>(re, im) : pack_complex<float>(re, im),
               stream);
}

// Window values cast to the compute dtype and zero padded to nfft.
std::vector<unsigned char> window_bytes(const std::vector<double> &w,
                                        int64_t nfft, bool f64) {
  std::vector<unsigned char> b(nfft * (f64 ? 8 : 4), 0);
  for (size_t i = 0; i < w.size(); ++i) {
    if (f64)
      reinterpret_cast<double *>(b.data())[i] = w[i];
    else
      reinterpret_cast<float *>(b.data())[i] = (float)w[i];
  }
  return b;
}

// compute_psd_scale (spectral_analysis.cpp:57-67) on the window as the
// kernel sees it (rounded to the compute dtype), summed in F64.
double window_sum_sq(const std::vector<double> &w, bool f64) {
  double s = 0.0;
  for (double v : w) {
    const double r = f64 ? v : (double)(float)v;
    s += r * r;
  }
  return s;
}

// Element view of one input: channel c, sample n at base + c*cs + n*ss.
struct InView {
  const InsightArray *a = nullptr;
  int64_t C = 1, N = 0, cs = 0, ss = 1;
  bool gpu = false;
  int dev = 0;
  int32_t dtype = 0;
  int64_t span = 0; // elements from the first addressed element to the last
};

InView view_input(const InsightArray *a, int axis, const char *op) {
  InView v;
  check(a != nullptr && a->ndim >= 1,
        std::string(op) + ": inputs are undefined");
  check(a->dtype == INSIGHT_DTYPE_F32 || a->dtype == INSIGHT_DTYPE_F64,
        std::string(op) + ": input dtype must be F32 or F64 on the B200 backend");
  check(a->ndim <= 2, std::string(op) +
                          ": inputs must be 1-D or 2-D (channels x samples)");
  v.a = a;
  v.dtype = a->dtype;
  v.gpu = a->device_type == INSIGHT_DEVICE_GPU;
  v.dev = a->device_id;
  if (a->ndim == 1) {
    v.N = a->dims[0];
    v.ss = a->strides[0];
  } else {
    int ax = axis < 0 ? axis + 2 : axis;
    check(ax == 0 || ax == 1, std::string(op) + ": axis out of range");
    v.N = a->dims[ax];
    v.ss = a->strides[ax];
    v.C = a->dims[1 - ax];
    v.cs = a->strides[1 - ax];
  }
  check(v.ss > 0 && v.cs >= 0,
        std::string(op) + ": negative or zero sample strides are not supported");
  v.span = (v.N > 0 ? (v.N - 1) * v.ss : 0) + (v.C > 0 ? (v.C - 1) * v.cs : 0) + 1;
  return v;
}

const char *base_ptr(const InsightArray *a) {
  return reinterpret_cast<const char *>(a->data) +
         a->offset * (int64_t)dtype_size(a->dtype);
}

int64_t numel(const InsightArray *a) {
  int64_t n = 1;
  for (int i = 0; i < a->ndim; ++i)
    n *= a->dims[i];
  return n;
}

bool contiguous(const InsightArray *a) {
  int64_t s = 1;
  for (int i = a->ndim - 1; i >= 0; --i) {
    if (a->dims[i] != 1 && a->strides[i] != s)
      return false;
    s *= a->dims[i];
  }
  return true;
}

// The f (F values) or t (S values) axis array of a call: checked, and the
// address of element 0 (nullptr when the caller passed none).
double *axis_array(InsightArray *dst, int64_t n, const char *what, int dev) {
  if (!dst)
    return nullptr;
  check(dst->dtype == INSIGHT_DTYPE_F64,
        std::string(what) + " must be an F64 array");
  check(numel(dst) == n, std::string(what) + " has " + std::to_string(numel(dst)) +
                             " elements, expected " + std::to_string(n));
  check(contiguous(dst), std::string(what) + " must be contiguous");
  check(dst->device_type != INSIGHT_DEVICE_GPU || dst->device_id == dev,
        std::string(what) + " on a different device");
  return reinterpret_cast<double *>(dst->data) + dst->offset;
}

// f[i] = i * (fs / nfft) and t[i] = (i * step + nperseg / 2) / fs
// (spectral_analysis.cpp:47-55, :250-253): host arrays are filled here, GPU
// arrays by a kernel on the call's stream with the same double operations
// (bit-identical values, no host buffer and no synchronisation).
void write_axes(int64_t F, int64_t S, InsightArray *f, InsightArray *t, double df,
                int64_t step, double half, double fs, int dev, cudaStream_t stream) {
  double *fp = axis_array(f, F, "f", dev);
  double *tp = axis_array(t, S, "t", dev);
  const bool fg = fp && f->device_type == INSIGHT_DEVICE_GPU;
  const bool tg = tp && t->device_type == INSIGHT_DEVICE_GPU;
  if (fp && !fg)
    for (int64_t i = 0; i < F; ++i)
      fp[i] = i * df;
  if (tp && !tg)
    for (int64_t i = 0; i < S; ++i)
      tp[i] = (i * step + half) / fs;
  if (fg || tg) {
    cuda_check(write_axes_device(fg ? fp : nullptr, F, df, tg ? tp : nullptr, S,
                                 step, half, fs, stream),
               "axes kernel");
    g_launches += 1;
  }
}

// Window values by (name, length), computed once per process (the table
// uploads are cached per device below).
const std::vector<double> &window_values_of(const std::string &name, int64_t n) {
  static std::mutex mu;
  static std::map<std::pair<std::string, int64_t>, std::vector<double>> cache;
  std::lock_guard<std::mutex> lk(mu);
  const auto key = std::make_pair(name, n);
  auto it = cache.find(key);
  if (it != cache.end())
    return it->second;
  std::vector<double> w;
  try {
    w = get_window(name, n, false);
  } catch (const std::invalid_argument &e) {
    throw Fail(e.what());
  }
  return cache.emplace(key, std::move(w)).first->second;
}

} // namespace

// ---------------------------------------------------------------------------
// One spectral call.
// ---------------------------------------------------------------------------
C_Status run(const Call &c) {
  try {
    // welch runs csd(x, x) in the reference (spectral_analysis.cpp:177-183)
    // and stft runs spectrogram (:330-334), so their messages carry those names.
    // coherence runs welch(x) first (:204), so its messages are csd's too.
    const bool two = c.op == INSIGHT_B200_OP_CSD || c.op == INSIGHT_B200_OP_COHERENCE;
    const bool acc = two || c.op == INSIGHT_B200_OP_WELCH;
    const char *op = acc ? "csd" : "spectrogram";
    check(c.op >= INSIGHT_B200_OP_WELCH && c.op <= INSIGHT_B200_OP_COHERENCE,
          "insight_b200: unknown operation code");
    check(c.nperseg > 0, std::string(op) + ": nperseg must be positive");
    InView xv = view_input(c.x, c.axis, op);
    InView yv = xv;
    if (two) {
      check(c.y != nullptr, "csd: inputs are undefined");
      yv = view_input(c.y, c.axis, op);
      check(yv.dtype == xv.dtype, "csd: x and y must have the same dtype");
      check(yv.N == xv.N && yv.C == xv.C,
            "csd: x and y must have the same shape");
      check(yv.gpu == xv.gpu && (!xv.gpu || yv.dev == xv.dev),
            "csd: x and y must be on the same device");
    }
    const bool f64 = xv.dtype == INSIGHT_DTYPE_F64;

    // Defaults (spectral_analysis.cpp:114-117 and :235-238).
    int64_t nfft = c.nfft == 0 ? c.nperseg : c.nfft;
    int64_t noverlap = c.noverlap;
    if (noverlap == 0)
      noverlap = acc ? c.nperseg / 2 : c.nperseg / 8;
    const int64_t step = c.nperseg - noverlap;
    check(step > 0, std::string(op) + ": noverlap must be less than nperseg");
    const int64_t N = xv.N;
    const int64_t S = (N >= c.nperseg) ? ((N - c.nperseg) / step + 1) : 0;
    check(S >= 1, acc ? std::string(op) + ": signal too short for given nperseg"
                      : std::string("spectrogram: signal too short"));
    check(nfft_supported(nfft),
          std::string(op) + ": nfft must be a power of two in [16, 8192] on the "
                            "B200 backend (got " + std::to_string(nfft) + ")");
    check(nfft >= c.nperseg,
          std::string(op) + ": nfft must be >= nperseg on the B200 backend");
    const bool onesided = c.onesided;
    const int64_t F = onesided ? nfft / 2 + 1 : nfft;

    int64_t seg0 = c.seg_begin, seg1 = c.seg_end <= 0 ? S : c.seg_end;
    check(seg0 >= 0 && seg0 < seg1 && seg1 <= S,
          std::string(op) + ": segment range out of bounds");

    // Window: caller values (registry kernels) or by name.
    const std::vector<double> &w =
        c.window_values ? *c.window_values : window_values_of(c.window, c.nperseg);
    check((int64_t)w.size() == c.nperseg,
          std::string(op) + ": window must have nperseg values");
    double scale = c.has_scale ? c.scale
                               : ((c.scaling == "density" ? c.fs : 1.0) /
                                  window_sum_sq(w, f64));
    const int dc_mode = c.detrend_linear ? 3
                        : !c.detrend_constant ? 0
                                              : (nfft == c.nperseg ? 1 : 2);

    // Result geometry (the f and t axes are written at the end, if asked for).
    const double df = c.fs / (double)nfft;

    const int dev = xv.gpu ? xv.dev : c.default_device;
    cuda_check(cudaSetDevice(dev), "cudaSetDevice");
    DeviceState &st = device_state(dev);
    std::lock_guard<std::mutex> lk(st.mu);
    cudaStream_t stream = c.stream ? c.stream : st.stream;

    LaunchDesc d;
    d.f64 = f64;
    d.nfft = nfft;
    d.nperseg = c.nperseg;
    d.step = step;
    d.C = xv.C;
    d.seg0 = seg0;
    d.S = seg1 - seg0;
    d.x_cs = xv.cs;
    d.x_ss = xv.ss;
    d.y_cs = yv.cs;
    d.y_ss = yv.ss;
    d.F = F;
    d.onesided_mask = onesided && nfft > 1;
    d.dc_mode = dc_mode;

    // Inputs: GPU arrays in place, CPU arrays copied over their span.
    auto stage = [&](const InView &v, DevBuf &buf) -> const void * {
      const size_t es = dtype_size(v.dtype);
      if (v.gpu) {
        check(v.dev == dev, std::string(op) + ": inputs on different devices");
        return base_ptr(v.a);
      }
      ensure(buf, v.span * es, stream);
      cuda_check(cudaMemcpyAsync(buf.p, base_ptr(v.a), v.span * es,
                                 cudaMemcpyHostToDevice, stream),
                 "cudaMemcpyAsync");
      return buf.p;
    };
    // Host input and host output of a channel batch of spectrogram / stft:
    // copies and launches are pipelined per channel chunk (below), so the
    // input is only reserved here.
    const bool host_pipe = !acc && !xv.gpu && c.out &&
                           c.out->device_type != INSIGHT_DEVICE_GPU &&
                           xv.C >= 2 && xv.cs >= (xv.N - 1) * xv.ss + 1;
    if (host_pipe) {
      ensure(st.xin, xv.span * dtype_size(xv.dtype), stream);
      d.x = st.xin.p;
    } else {
      d.x = stage(xv, st.xin);
    }
    d.y = two ? stage(yv, st.yin) : nullptr;

    // Tables.  Caller window values (registry kernels) are copied from `wb`,
    // which lives until the call returns; such calls synchronise their
    // stream before returning (must_sync below).
    std::vector<unsigned char> wb;
    if (c.window_values) {
      wb = window_bytes(w, nfft, f64);
      ensure(st.win_tmp, wb.size(), stream);
      cuda_check(cudaMemcpyAsync(st.win_tmp.p, wb.data(), wb.size(),
                                 cudaMemcpyHostToDevice, stream),
                 "cudaMemcpyAsync");
      d.win = st.win_tmp.p;
    } else {
      std::string key = std::string("win|") + (f64 ? "d|" : "f|") + c.window +
                        "|" + std::to_string(c.nperseg) + "|" +
                        std::to_string(nfft);
      d.win = table(st, key, window_bytes(w, nfft, f64), stream);
    }
    d.tw = twiddles(st, nfft, f64, stream);
    d.dtab = dc_mode == 2 ? dc_table(st, nfft, c.nperseg, f64, stream) : nullptr;

    // Output array.
    InsightArray *out = c.out;
    check(out != nullptr, std::string(op) + ": output array is undefined");
    const bool out_complex =
        out->dtype == INSIGHT_DTYPE_C32 || out->dtype == INSIGHT_DTYPE_C64;
    check(out->dtype == INSIGHT_DTYPE_F64 || out_complex,
          std::string(op) + ": output must be F64, C32 or C64");
    const size_t oes = dtype_size(out->dtype);
    const bool out_gpu = out->device_type == INSIGHT_DEVICE_GPU;
    check(!out_gpu || out->device_id == dev,
          std::string(op) + ": output on a different device");
    const int64_t Sl = seg1 - seg0;
    int64_t o_cs = 0, o_rs = 0, o_ts = 0;
    int64_t out_elems = 0;
    if (acc) {
      // [F] or [C, F]
      out_elems = xv.C * F;
      check(numel(out) == out_elems,
            std::string(op) + ": output must have " + std::to_string(out_elems) +
                " elements");
      check(out->dims[out->ndim - 1] == F && out->strides[out->ndim - 1] == 1,
            std::string(op) + ": output bins must be the last, unit-stride axis");
      o_cs = out->ndim >= 2 ? out->strides[out->ndim - 2] : F;
      if (c.op == INSIGHT_B200_OP_WELCH) {
        d.kind = LK_PSD;
        check(out->dtype == INSIGHT_DTYPE_F64, "welch: output must be F64");
        d.out_kind = c.raw_sums ? OUT_RAW_F64_K : OUT_REAL_F64_K;
      } else if (c.op == INSIGHT_B200_OP_COHERENCE) {
        d.kind = LK_COH;
        check(out->dtype == INSIGHT_DTYPE_F64, "coherence: output must be F64");
        check(!c.raw_sums, "coherence: raw sums are not available");
        check(onesided, "coherence: the result is one-sided");
        d.out_kind = OUT_REAL_F64_K;
      } else {
        d.kind = LK_CSD;
        if (c.raw_sums) {
          check(out->dtype == INSIGHT_DTYPE_C64,
                "csd: raw sums need a C64 (complex128) output");
          d.out_kind = OUT_RAW_F64_K;
        } else if (out->dtype == INSIGHT_DTYPE_F64) {
          d.out_kind = OUT_REAL_F64_K;
        } else {
          d.out_kind = out->dtype == INSIGHT_DTYPE_C32 ? OUT_C64_K : OUT_C128_K;
        }
      }
      check(c.avg_segments >= 0, std::string(op) + ": avg_segments must be >= 0");
      d.avg_scale = scale / (double)(c.avg_segments > 0 ? c.avg_segments : S);
    } else {
      d.kind = LK_STORE;
      // complex: [C?, F, Sl]; F64: [C?, Sl, F] (the reference's transposed view)
      out_elems = xv.C * F * Sl;
      check(numel(out) == out_elems,
            std::string(op) + ": output must have " + std::to_string(out_elems) +
                " elements");
      const int nd = out->ndim;
      check(nd >= 2 && (nd == 2 ? xv.C == 1 : nd == 3),
            std::string(op) + ": output must be 2-D (or 3-D for a batch)");
      if (out_complex) {
        o_rs = out->strides[nd - 2];
        o_ts = out->strides[nd - 1];
        check(out->dims[nd - 2] == F && out->dims[nd - 1] == Sl,
              std::string(op) + ": complex output must be (n_freq, n_seg)");
      } else {
        o_ts = out->strides[nd - 2];
        o_rs = out->strides[nd - 1];
        check(out->dims[nd - 2] == Sl && out->dims[nd - 1] == F,
              std::string(op) + ": F64 output must be (n_seg, n_freq)");
      }
      o_cs = nd == 3 ? out->strides[0] : 0;
      if (out_complex) {
        const bool want = f64 ? out->dtype == INSIGHT_DTYPE_C64
                              : out->dtype == INSIGHT_DTYPE_C32;
        check(want, std::string(op) +
                        ": complex output must be C32 for F32 input, C64 for F64");
        d.out_kind = f64 ? OUT_C128_K : OUT_C64_K;
      } else if (c.mode == "psd") {
        d.out_kind = OUT_PSD_F64_K;
      } else if (c.mode == "complex") {
        d.out_kind = OUT_REAL_F64_K;
      } else {
        d.out_kind = OUT_MAG_F64_K;
      }
      d.psd_scale = scale; // spectrogram psd uses 'density' scaling (:304)
    }

    // Where the kernel writes: the caller's GPU array, or a device buffer
    // that is copied back to the caller's CPU array.
    bool direct = out_gpu;
    int64_t span = 0;
    {
      int64_t lo = 0, hi = 0;
      for (int i = 0; i < out->ndim; ++i) {
        check(out->strides[i] >= 0, std::string(op) + ": negative output strides");
        hi += (out->dims[i] - 1) * out->strides[i];
      }
      span = hi - lo + 1;
    }
    void *obase;
    if (direct) {
      obase = reinterpret_cast<char *>(out->data) + out->offset * (int64_t)oes;
    } else {
      ensure(st.out, span * oes, stream);
      obase = st.out.p;
    }
    d.out = obase;
    d.o_cs = o_cs;
    d.o_rs = o_rs;
    d.o_ts = o_ts;

    // Pipelined host I/O (see host_pipe): chunk j of channels [c0, c1) is
    // copied in, transformed and copied out on stream j % kPipe.
    const int64_t span_c = span - (xv.C - 1) * o_cs; // one channel's output
    if (host_pipe && o_cs >= span_c) {
      const size_t xes = dtype_size(xv.dtype);
      const int64_t xspan_c = (xv.N - 1) * xv.ss + 1;
      const int64_t K = std::min<int64_t>(xv.C, 8);
      for (int i = 0; i < DeviceState::kPipe; ++i)
        if (!st.pipe[i])
          cuda_check(cudaStreamCreateWithFlags(&st.pipe[i], cudaStreamNonBlocking),
                     "cudaStreamCreate");
      if (!st.pipe_start)
        cuda_check(cudaEventCreateWithFlags(&st.pipe_start, cudaEventDisableTiming),
                   "cudaEventCreate");
      // table uploads above were issued on `stream`
      cuda_check(cudaEventRecord(st.pipe_start, stream), "cudaEventRecord");
      const char *xh = base_ptr(xv.a);
      char *oh = reinterpret_cast<char *>(out->data) + out->offset * (int64_t)oes;
      int64_t nl = 0;
      for (int64_t j = 0; j < K; ++j) {
        const int64_t c0 = xv.C * j / K, c1 = xv.C * (j + 1) / K;
        cudaStream_t ps = st.pipe[j % DeviceState::kPipe];
        if (j < DeviceState::kPipe)
          cuda_check(cudaStreamWaitEvent(ps, st.pipe_start, 0), "cudaStreamWaitEvent");
        const size_t xoff = (size_t)(c0 * xv.cs) * xes;
        const size_t xlen = (size_t)((c1 - c0 - 1) * xv.cs + xspan_c) * xes;
        cuda_check(cudaMemcpyAsync(static_cast<char *>(st.xin.p) + xoff, xh + xoff,
                                   xlen, cudaMemcpyHostToDevice, ps),
                   "cudaMemcpyAsync");
        LaunchDesc dj = d;
        dj.C = c1 - c0;
        dj.x = static_cast<const char *>(st.xin.p) + xoff;
        dj.out = static_cast<char *>(obase) + (size_t)(c0 * o_cs) * oes;
        cuda_check(launch(dj, nullptr, st.num_sms, ps, &nl), "kernel launch");
        const size_t ooff = (size_t)(c0 * o_cs) * oes;
        const size_t olen = (size_t)((c1 - c0 - 1) * o_cs + span_c) * oes;
        cuda_check(cudaMemcpyAsync(oh + ooff, static_cast<char *>(obase) + ooff, olen,
                                   cudaMemcpyDeviceToHost, ps),
                   "cudaMemcpyAsync");
      }
      g_launches += nl;
      for (int i = 0; i < DeviceState::kPipe; ++i)
        cuda_check(cudaStreamSynchronize(st.pipe[i]), "cudaStreamSynchronize");
      write_axes(F, S, c.f, c.t, df, step, c.nperseg / 2.0, c.fs, dev, stream);
      cuda_check(cudaStreamSynchronize(stream), "cudaStreamSynchronize");
      return C_SUCCESS;
    }
    if (host_pipe) // output channels interleave: one copy of the whole input
      cuda_check(cudaMemcpyAsync(st.xin.p, base_ptr(xv.a),
                                 xv.span * dtype_size(xv.dtype),
                                 cudaMemcpyHostToDevice, stream),
                 "cudaMemcpyAsync");

    // Scratch (this stream's own) and launch.
    const size_t sb = scratch_bytes(d, st.num_sms);
    StreamBufs *sbuf = nullptr;
    if (sb) {
      sbuf = &stream_bufs(st, stream);
      ensure(sbuf->scratch, sb, stream);
    }
    int64_t nl = 0;
    cuda_check(launch(d, sbuf ? sbuf->scratch.p : nullptr, st.num_sms, stream, &nl),
               "kernel launch");
    g_launches += nl;
    if (sbuf)
      mark_used(*sbuf, stream);

    if (!direct) {
      char *hp = reinterpret_cast<char *>(out->data) + out->offset * (int64_t)oes;
      cuda_check(cudaMemcpyAsync(hp, obase, span * oes, cudaMemcpyDeviceToHost,
                                 stream),
                 "cudaMemcpyAsync");
    }
    write_axes(F, S, c.f, c.t, df, step, c.nperseg / 2.0, c.fs, dev, stream);
    const bool must_sync = c.sync || !xv.gpu || !direct || (two && !yv.gpu) ||
                           c.window_values != nullptr;
    if (must_sync)
      cuda_check(cudaStreamSynchronize(stream), "cudaStreamSynchronize");
    else
      cuda_check(cudaGetLastError(), "kernel launch");
    return C_SUCCESS;
  } catch (const std::exception &e) {
    set_last_error(e.what());
    return C_FAILED;
  }
}

// ---------------------------------------------------------------------------
// Inverse STFT.
// ---------------------------------------------------------------------------
namespace {

struct IstftGeom {
  int64_t C = 1, F = 0, S = 0, nfft = 0, nperseg = 0, hop = 0, n_total = 0;
  int64_t cs = 0, fs = 0, ts = 0; // element strides of Zxx
  bool f64 = false, pack = true;
};

// Defaults and checks of the reference istft (spectral_analysis.cpp:342-356).
IstftGeom istft_geom(const IstftCall &c) {
  IstftGeom g;
  const InsightArray *z = c.z;
  check(z != nullptr, "istft: Zxx is undefined");
  check(z->ndim == 2 || z->ndim == 3,
        "istft: Zxx must be 2D (or 3D for a batch of channels)");
  check(z->dtype == INSIGHT_DTYPE_C32 || z->dtype == INSIGHT_DTYPE_C64,
        "istft: Zxx must be complex (C32 or C64) on the B200 backend");
  g.f64 = z->dtype == INSIGHT_DTYPE_C64;
  const int nd = z->ndim;
  g.F = z->dims[nd - 2];
  g.S = z->dims[nd - 1];
  g.fs = z->strides[nd - 2];
  g.ts = z->strides[nd - 1];
  if (nd == 3) {
    g.C = z->dims[0];
    g.cs = z->strides[0];
  }
  check(g.F >= 1 && g.S >= 1, "istft: Zxx is empty");
  check(g.fs >= 0 && g.ts >= 0 && g.cs >= 0,
        "istft: negative strides are not supported");
  g.nfft = c.nfft <= 0 ? 2 * (g.F - 1) : c.nfft;
  g.nperseg = c.nperseg <= 0 ? g.nfft : c.nperseg;
  const int64_t noverlap = c.noverlap <= 0 ? g.nperseg / 2 : c.noverlap;
  g.hop = g.nperseg - noverlap;
  check(g.hop > 0, "istft: noverlap must be less than nperseg");
  check(nfft_supported(g.nfft),
        "istft: nfft must be a power of two in [16, 8192] on the B200 backend "
        "(got " + std::to_string(g.nfft) + ")");
  check(g.nperseg <= g.nfft, "istft: nperseg must be <= nfft");
  g.pack = g.F == g.nfft / 2 + 1 && g.nfft > 2;
  g.n_total = (g.S - 1) * g.hop + g.nperseg;
  return g;
}

} // namespace

C_Status istft_shape(const IstftCall &c, int64_t *n_channels, int64_t *n_total) {
  try {
    IstftGeom g = istft_geom(c);
    if (n_channels)
      *n_channels = g.C;
    if (n_total)
      *n_total = g.n_total;
    return C_SUCCESS;
  } catch (const std::exception &e) {
    set_last_error(e.what());
    return C_FAILED;
  }
}

C_Status run_istft(const IstftCall &c) {
  try {
    IstftGeom g = istft_geom(c);
    const InsightArray *z = c.z;
    InsightArray *out = c.out;
    check(out != nullptr && out->dtype == INSIGHT_DTYPE_F64,
          "istft: output must be an F64 array");
    check(numel(out) == g.C * g.n_total,
          "istft: output must have " + std::to_string(g.C * g.n_total) +
              " elements");
    check(out->ndim == (z->ndim == 3 ? 2 : 1) &&
              out->dims[out->ndim - 1] == g.n_total,
          "istft: output must be [n_total] (or [C, n_total] for a batch)");
    const std::vector<double> &w = c.window_values
                                       ? *c.window_values
                                       : window_values_of(c.window, g.nperseg);
    check((int64_t)w.size() == g.nperseg, "istft: window must have nperseg values");
    const bool zgpu = z->device_type == INSIGHT_DEVICE_GPU;
    const bool ogpu = out->device_type == INSIGHT_DEVICE_GPU;
    const int dev = zgpu ? z->device_id : (ogpu ? out->device_id : c.default_device);
    check(!ogpu || out->device_id == dev, "istft: output on a different device");
    cuda_check(cudaSetDevice(dev), "cudaSetDevice");
    DeviceState &st = device_state(dev);
    std::lock_guard<std::mutex> lk(st.mu);
    cudaStream_t stream = c.stream ? c.stream : st.stream;

    IstftDesc d;
    d.f64 = g.f64;
    d.C = g.C;
    d.F = g.F;
    d.S = g.S;
    d.nfft = g.nfft;
    d.nperseg = g.nperseg;
    d.hop = g.hop;
    d.n_total = g.n_total;
    d.pack = g.pack;
    d.z_cs = g.cs;
    d.z_fs = g.fs;
    d.z_ts = g.ts;
    const size_t zes = dtype_size(z->dtype);
    if (zgpu) {
      d.z = base_ptr(z);
    } else {
      const int64_t span = (g.C - 1) * g.cs + (g.F - 1) * g.fs + (g.S - 1) * g.ts + 1;
      ensure(st.xin, span * zes, stream);
      cuda_check(cudaMemcpyAsync(st.xin.p, base_ptr(z), span * zes,
                                 cudaMemcpyHostToDevice, stream),
                 "cudaMemcpyAsync");
      d.z = st.xin.p;
    }
    // tables: window in the compute dtype and in f64, twiddles
    std::vector<unsigned char> w64(w.size() * 8);
    std::memcpy(w64.data(), w.data(), w64.size());
    // the transforms run in f64 for both input precisions; caller window
    // values (registry kernel) are copied from wb / w64, which live until the
    // call returns (such calls synchronise their stream before returning)
    std::vector<unsigned char> wb;
    if (c.window_values) {
      wb = window_bytes(w, g.nperseg, true);
      const size_t off = (wb.size() + 15) / 16 * 16; // f64 copy after it
      ensure(st.win_tmp, off + w64.size(), stream);
      char *p = reinterpret_cast<char *>(st.win_tmp.p);
      cuda_check(cudaMemcpyAsync(p, wb.data(), wb.size(), cudaMemcpyHostToDevice,
                                 stream),
                 "cudaMemcpyAsync");
      cuda_check(cudaMemcpyAsync(p + off, w64.data(), w64.size(),
                                 cudaMemcpyHostToDevice, stream),
                 "cudaMemcpyAsync");
      d.win = p;
      d.win64 = reinterpret_cast<const double *>(p + off);
    } else {
      const std::string k = c.window + "|" + std::to_string(g.nperseg);
      d.win = table(st, std::string("win|d|") + k + "|" + std::to_string(g.nperseg),
                    window_bytes(w, g.nperseg, true), stream);
      d.win64 = reinterpret_cast<const double *>(
          table(st, "win64|" + k, w64, stream));
    }
    d.tw = twiddles(st, g.nfft, true, stream);
    StreamBufs &sbuf = stream_bufs(st, stream);
    ensure(sbuf.frames, (size_t)g.C * g.S * g.nperseg * (g.f64 ? 8 : 4), stream);
    d.frames = sbuf.frames.p;
    // output: the caller's GPU array, or a device buffer copied back
    d.o_ss = out->strides[out->ndim - 1];
    d.o_cs = out->ndim == 2 ? out->strides[0] : 0;
    int64_t ospan = (g.n_total - 1) * d.o_ss + (g.C - 1) * d.o_cs + 1;
    if (ogpu) {
      d.out = reinterpret_cast<double *>(out->data) + out->offset;
    } else {
      ensure(st.out, ospan * 8, stream);
      d.out = reinterpret_cast<double *>(st.out.p);
    }
    int64_t nl = 0;
    cuda_check(launch_istft(d, st.num_sms, stream, &nl), "istft launch");
    g_launches += nl;
    mark_used(sbuf, stream);
    if (!ogpu) {
      cuda_check(cudaMemcpyAsync(reinterpret_cast<double *>(out->data) + out->offset,
                                 d.out, ospan * 8, cudaMemcpyDeviceToHost, stream),
                 "cudaMemcpyAsync");
    }
    if (c.sync || !zgpu || !ogpu || c.window_values)
      cuda_check(cudaStreamSynchronize(stream), "cudaStreamSynchronize");
    else
      cuda_check(cudaGetLastError(), "istft launch");
    return C_SUCCESS;
  } catch (const std::exception &e) {
    set_last_error(e.what());
    return C_FAILED;
  }
}

C_Status shape(const Call &c, int64_t *n_channels, int64_t *n_seg,
               int64_t *n_freq) {
  try {
    const bool acc = c.op == INSIGHT_B200_OP_WELCH || c.op == INSIGHT_B200_OP_CSD ||
                     c.op == INSIGHT_B200_OP_COHERENCE;
    const char *op = acc ? "csd" : "spectrogram";
    check(c.nperseg > 0, std::string(op) + ": nperseg must be positive");
    InView xv = view_input(c.x, c.axis, op);
    int64_t nfft = c.nfft == 0 ? c.nperseg : c.nfft;
    int64_t noverlap = c.noverlap == 0 ? (acc ? c.nperseg / 2 : c.nperseg / 8)
                                       : c.noverlap;
    const int64_t step = c.nperseg - noverlap;
    check(step > 0, std::string(op) + ": noverlap must be less than nperseg");
    const int64_t N = xv.N;
    const int64_t S = (N >= c.nperseg) ? ((N - c.nperseg) / step + 1) : 0;
    if (n_channels)
      *n_channels = xv.C;
    if (n_seg)
      *n_seg = S;
    if (n_freq)
      *n_freq = c.onesided ? nfft / 2 + 1 : nfft;
    return C_SUCCESS;
  } catch (const std::exception &e) {
    set_last_error(e.what());
    return C_FAILED;
  }
}

// Scale and mask reduced raw sums in place (after a cross-device reduction).
C_Status finalize_sums(const Call &c, int64_t S_total, InsightArray *sums) {
  try {
    check(sums && sums->device_type == INSIGHT_DEVICE_GPU,
          "finalize_sums: sums must be a GPU array");
    const bool f64 = c.x_dtype == INSIGHT_DTYPE_F64;
    const std::vector<double> &w = window_values_of(c.window, c.nperseg);
    const double scale =
        (c.scaling == "density" ? c.fs : 1.0) / window_sum_sq(w, f64);
    const int64_t nfft = c.nfft == 0 ? c.nperseg : c.nfft;
    const int64_t F = c.onesided ? nfft / 2 + 1 : nfft;
    const bool cplx = sums->dtype == INSIGHT_DTYPE_C64;
    check(sums->dtype == INSIGHT_DTYPE_F64 || cplx,
          "finalize_sums: sums must be F64 or C64");
    check(contiguous(sums) && numel(sums) % F == 0,
          "finalize_sums: sums must be a contiguous [C, n_freq] array");
    const int64_t C = numel(sums) / F;
    cuda_check(cudaSetDevice(sums->device_id), "cudaSetDevice");
    DeviceState &st = device_state(sums->device_id);
    std::lock_guard<std::mutex> lk(st.mu);
    cudaStream_t stream = c.stream ? c.stream : st.stream;
    double *p = reinterpret_cast<double *>(sums->data) +
                sums->offset * (cplx ? 2 : 1);
    cuda_check(scale_sums(p, C, F, cplx, scale / (double)S_total,
                          c.onesided && nfft > 1, stream),
               "finalize_sums");
    g_launches += 1;
    if (c.sync)
      cuda_check(cudaStreamSynchronize(stream), "cudaStreamSynchronize");
    return C_SUCCESS;
  } catch (const std::exception &e) {
    set_last_error(e.what());
    return C_FAILED;
  }
}

// ---------------------------------------------------------------------------
// Plans: one call captured into a CUDA graph.
// ---------------------------------------------------------------------------
struct Plan {
  int dev = 0;
  cudaStream_t cs = nullptr; // capture stream (owns the plan's scratch)
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
  DevBuf scratch, frames;    // taken over from the capture stream's buffers
};

C_Status plan_create(const Call &c0, void **plan_out) {
  Plan *pl = nullptr;
  try {
    check(plan_out != nullptr, "plan: output handle is NULL");
    check(c0.x && c0.x->device_type == INSIGHT_DEVICE_GPU && c0.out &&
              c0.out->device_type == INSIGHT_DEVICE_GPU &&
              (!c0.y || c0.y->device_type == INSIGHT_DEVICE_GPU),
          "plan: inputs and output must be GPU arrays");
    check(!c0.f && !c0.t, "plan: the f and t axes are not part of a plan");
    pl = new Plan();
    pl->dev = c0.x->device_id;
    cuda_check(cudaSetDevice(pl->dev), "cudaSetDevice");
    cuda_check(cudaStreamCreateWithFlags(&pl->cs, cudaStreamNonBlocking),
               "cudaStreamCreate");
    // order the plan after the caller's stream, then run the call once on
    // the capture stream: tables uploaded, the stream's scratch allocated
    if (c0.stream) {
      cudaEvent_t ev;
      cuda_check(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming),
                 "cudaEventCreate");
      cuda_check(cudaEventRecord(ev, c0.stream), "cudaEventRecord");
      cuda_check(cudaStreamWaitEvent(pl->cs, ev, 0), "cudaStreamWaitEvent");
      cuda_check(cudaEventDestroy(ev), "cudaEventDestroy");
    }
    Call c = c0;
    c.stream = pl->cs;
    c.sync = true;
    if (run(c) != C_SUCCESS)
      throw Fail(last_error());
    // capture the same call
    c.sync = false;
    cuda_check(cudaStreamBeginCapture(pl->cs, cudaStreamCaptureModeThreadLocal),
               "cudaStreamBeginCapture");
    g_capturing = true;
    const C_Status rs = run(c);
    g_capturing = false;
    const cudaError_t ec = cudaStreamEndCapture(pl->cs, &pl->graph);
    if (rs != C_SUCCESS)
      throw Fail(last_error());
    cuda_check(ec, "cudaStreamEndCapture");
    cuda_check(cudaGraphInstantiate(&pl->exec, pl->graph, 0),
               "cudaGraphInstantiate");
    // the plan owns the buffers its graph writes
    DeviceState &st = device_state(pl->dev);
    {
      std::lock_guard<std::mutex> lk(st.mu);
      auto it = st.per_stream.find(pl->cs);
      if (it != st.per_stream.end()) {
        pl->scratch = it->second.scratch;
        pl->frames = it->second.frames;
        if (it->second.last)
          cudaEventDestroy(it->second.last);
        st.per_stream.erase(it);
      }
    }
    *plan_out = pl;
    return C_SUCCESS;
  } catch (const std::exception &e) {
    g_capturing = false;
    set_last_error(e.what());
    if (pl)
      plan_destroy(pl);
    return C_FAILED;
  }
}

C_Status plan_execute(void *plan, cudaStream_t stream, bool sync) {
  try {
    check(plan != nullptr, "plan: handle is NULL");
    Plan *pl = static_cast<Plan *>(plan);
    cuda_check(cudaSetDevice(pl->dev), "cudaSetDevice");
    cudaStream_t s = stream ? stream : pl->cs;
    cuda_check(cudaGraphLaunch(pl->exec, s), "cudaGraphLaunch");
    g_launches += 1;
    if (sync)
      cuda_check(cudaStreamSynchronize(s), "cudaStreamSynchronize");
    return C_SUCCESS;
  } catch (const std::exception &e) {
    set_last_error(e.what());
    return C_FAILED;
  }
}

C_Status plan_destroy(void *plan) {
  if (!plan)
    return C_SUCCESS;
  Plan *pl = static_cast<Plan *>(plan);
  cudaSetDevice(pl->dev);
  // executions may have been queued on any stream: let the device finish
  // them before the buffers their kernels write are released
  cudaDeviceSynchronize();
  if (pl->exec)
    cudaGraphExecDestroy(pl->exec);
  if (pl->graph)
    cudaGraphDestroy(pl->graph);
  if (pl->cs) {
    if (pl->scratch.p)
      cudaFreeAsync(pl->scratch.p, pl->cs);
    if (pl->frames.p)
      cudaFreeAsync(pl->frames.p, pl->cs);
    cudaStreamSynchronize(pl->cs);
  }
  if (pl->cs) {
    DeviceState &st = device_state(pl->dev);
    std::lock_guard<std::mutex> lk(st.mu);
    auto it = st.per_stream.find(pl->cs);
    if (it != st.per_stream.end()) {
      if (it->second.last)
        cudaEventDestroy(it->second.last);
      st.per_stream.erase(it);
    }
    cudaStreamDestroy(pl->cs);
  }
  delete pl;
  return C_SUCCESS;
}

} // namespace ib200

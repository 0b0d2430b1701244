// plugin.cpp — the Insight device-plugin boundary of the B200 backend.
//
// InitPluginGPU fills the reference's C_DeviceInterface
// (include/insight/c_api/device_ext.h:156-768) for CUDA devices, as the
// reference CUDA plugin does (backends/cuda/device/cuda_device.cpp:769-862),
// and registers the fused spectral kernels under the op names "welch", "csd",
// "spectrogram" and "stft" for INSIGHT_DEVICE_GPU x {F32, F64}.  The kernels
// use the reference kernel signature (include/insight/c_api/kernel.h:21) and
// argument convention (backends/cpu/kernels/fft/fft_c2c.cpp:9-16); see
// include/insight_b200.h for each layout.  Errors are C_FAILED plus a
// thread-local message (cuda_device.cpp:25-38); C_FALLBACK is never
// returned, so the core's CPU fallback (src/core/kernel.cpp:37-142) is never
// taken for these ops.
#include "frontend.h"

#include <chrono>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

using ib200::set_last_error;

namespace {

C_Status cerr(cudaError_t e) {
  if (e == cudaSuccess)
    return C_SUCCESS;
  set_last_error(cudaGetErrorString(e));
  return C_FAILED;
}

// ---------------------------------------------------------------------------
// C_DeviceInterface
// ---------------------------------------------------------------------------
C_Status b_initialize(void) {
  int n = 0;
  return cerr(cudaGetDeviceCount(&n));
}
C_Status b_finalize(void) { return C_SUCCESS; }
C_Status b_init_device(C_Device d) { return d ? cerr(cudaSetDevice(d->id)) : C_FAILED; }
C_Status b_deinit_device(C_Device d) { return d ? C_SUCCESS : C_FAILED; }
C_Status b_set_device(C_Device d) { return d ? cerr(cudaSetDevice(d->id)) : C_FAILED; }
C_Status b_get_device(C_Device d) {
  if (!d)
    return C_FAILED;
  return cerr(cudaGetDevice(&d->id));
}
C_Status b_synchronize_device(C_Device d) {
  if (!d)
    return C_FAILED;
  C_Status s = cerr(cudaSetDevice(d->id));
  return s != C_SUCCESS ? s : cerr(cudaDeviceSynchronize());
}
C_Status b_get_device_count(size_t *count) {
  if (!count)
    return C_FAILED;
  int n = 0;
  C_Status s = cerr(cudaGetDeviceCount(&n));
  *count = (size_t)n;
  return s;
}
C_Status b_get_device_list(size_t *devices) {
  if (!devices)
    return C_FAILED;
  size_t n = 0;
  C_Status s = b_get_device_count(&n);
  for (size_t i = 0; i < n; ++i)
    devices[i] = i;
  return s;
}
C_Status b_device_memory_allocate(C_Device d, void **ptr, size_t size) {
  if (!d || !ptr)
    return C_FAILED;
  C_Status s = cerr(cudaSetDevice(d->id));
  if (s != C_SUCCESS)
    return s;
  if (size == 0) {
    *ptr = nullptr;
    return C_SUCCESS;
  }
  return cerr(cudaMalloc(ptr, size));
}
C_Status b_device_memory_deallocate(C_Device d, void *ptr, size_t) {
  if (!d)
    return C_FAILED;
  if (!ptr)
    return C_SUCCESS;
  C_Status s = cerr(cudaSetDevice(d->id));
  return s != C_SUCCESS ? s : cerr(cudaFree(ptr));
}
C_Status b_host_memory_allocate(C_Device, void **ptr, size_t size) {
  if (!ptr)
    return C_FAILED;
  return cerr(cudaMallocHost(ptr, size));
}
C_Status b_host_memory_deallocate(C_Device, void *ptr, size_t) {
  return ptr ? cerr(cudaFreeHost(ptr)) : C_SUCCESS;
}
C_Status copy_sync(C_Device d, void *dst, const void *src, size_t n,
                   cudaMemcpyKind k) {
  if (!d)
    return C_FAILED;
  C_Status s = cerr(cudaSetDevice(d->id));
  return s != C_SUCCESS ? s : cerr(cudaMemcpy(dst, src, n, k));
}
C_Status b_copy_h2d(C_Device d, void *dst, const void *src, size_t n) {
  return copy_sync(d, dst, src, n, cudaMemcpyHostToDevice);
}
C_Status b_copy_d2h(C_Device d, void *dst, const void *src, size_t n) {
  return copy_sync(d, dst, src, n, cudaMemcpyDeviceToHost);
}
C_Status b_copy_d2d(C_Device d, void *dst, const void *src, size_t n) {
  return copy_sync(d, dst, src, n, cudaMemcpyDeviceToDevice);
}
C_Status b_copy_p2p(C_Device dd, C_Device sd, void *dst, const void *src,
                    size_t n) {
  if (!dd || !sd)
    return C_FAILED;
  return cerr(cudaMemcpyPeer(dst, dd->id, src, sd->id, n));
}
C_Status b_memset(C_Device d, void *ptr, unsigned char v, size_t n) {
  if (!d)
    return C_FAILED;
  C_Status s = cerr(cudaSetDevice(d->id));
  return s != C_SUCCESS ? s : cerr(cudaMemset(ptr, v, n));
}
C_Status b_memory_stats(C_Device d, size_t *total, size_t *free_b) {
  if (!d || !total || !free_b)
    return C_FAILED;
  C_Status s = cerr(cudaSetDevice(d->id));
  return s != C_SUCCESS ? s : cerr(cudaMemGetInfo(free_b, total));
}
C_Status copy_async(C_Device d, C_Stream st, void *dst, const void *src,
                    size_t n, cudaMemcpyKind k) {
  if (!d)
    return C_FAILED;
  C_Status s = cerr(cudaSetDevice(d->id));
  return s != C_SUCCESS
             ? s
             : cerr(cudaMemcpyAsync(dst, src, n, k, (cudaStream_t)st));
}
C_Status b_acopy_h2d(C_Device d, C_Stream s, void *dst, const void *src, size_t n) {
  return copy_async(d, s, dst, src, n, cudaMemcpyHostToDevice);
}
C_Status b_acopy_d2h(C_Device d, C_Stream s, void *dst, const void *src, size_t n) {
  return copy_async(d, s, dst, src, n, cudaMemcpyDeviceToHost);
}
C_Status b_acopy_d2d(C_Device d, C_Stream s, void *dst, const void *src, size_t n) {
  return copy_async(d, s, dst, src, n, cudaMemcpyDeviceToDevice);
}
C_Status b_acopy_p2p(C_Device dd, C_Device sd, C_Stream s, void *dst,
                     const void *src, size_t n) {
  if (!dd || !sd)
    return C_FAILED;
  return cerr(cudaMemcpyPeerAsync(dst, dd->id, src, sd->id, n, (cudaStream_t)s));
}
C_Status b_create_stream(C_Device d, C_Stream *s) {
  if (!d || !s)
    return C_FAILED;
  C_Status r = cerr(cudaSetDevice(d->id));
  if (r != C_SUCCESS)
    return r;
  cudaStream_t cs = nullptr;
  r = cerr(cudaStreamCreateWithFlags(&cs, cudaStreamNonBlocking));
  *s = (C_Stream)cs;
  return r;
}
C_Status b_destroy_stream(C_Device, C_Stream s) {
  return cerr(cudaStreamDestroy((cudaStream_t)s));
}
C_Status b_query_stream(C_Device, C_Stream s) {
  cudaError_t e = cudaStreamQuery((cudaStream_t)s);
  if (e == cudaErrorNotReady)
    return C_FAILED;
  return cerr(e);
}
C_Status b_sync_stream(C_Device, C_Stream s) {
  return cerr(cudaStreamSynchronize((cudaStream_t)s));
}

struct CbData {
  void (*cb)(C_Device, C_Stream, void *, C_Status *);
  C_Device dev;
  C_Stream stream;
  void *user;
};
void host_cb(void *p) {
  CbData *d = (CbData *)p;
  C_Status st = C_SUCCESS;
  d->cb(d->dev, d->stream, d->user, &st);
  delete d;
}
C_Status b_stream_add_callback(C_Device d, C_Stream s,
                               void (*cb)(C_Device, C_Stream, void *, C_Status *),
                               void *user) {
  if (!cb)
    return C_FAILED;
  CbData *data = new CbData{cb, d, s, user};
  cudaError_t e = cudaLaunchHostFunc((cudaStream_t)s, host_cb, data);
  if (e != cudaSuccess)
    delete data;
  return cerr(e);
}
C_Status b_stream_wait_event(C_Device, C_Stream s, C_Event e) {
  return cerr(cudaStreamWaitEvent((cudaStream_t)s, (cudaEvent_t)e, 0));
}
C_Status b_create_event(C_Device d, C_Event *e) {
  if (!d || !e)
    return C_FAILED;
  C_Status r = cerr(cudaSetDevice(d->id));
  if (r != C_SUCCESS)
    return r;
  cudaEvent_t ce = nullptr;
  r = cerr(cudaEventCreate(&ce));
  *e = (C_Event)ce;
  return r;
}
C_Status b_destroy_event(C_Device, C_Event e) {
  return cerr(cudaEventDestroy((cudaEvent_t)e));
}
C_Status b_record_event(C_Device, C_Stream s, C_Event e) {
  return cerr(cudaEventRecord((cudaEvent_t)e, (cudaStream_t)s));
}
C_Status b_query_event(C_Device, C_Event e) {
  cudaError_t r = cudaEventQuery((cudaEvent_t)e);
  if (r == cudaErrorNotReady)
    return C_FAILED;
  return cerr(r);
}
C_Status b_sync_event(C_Device, C_Event e) {
  return cerr(cudaEventSynchronize((cudaEvent_t)e));
}
C_Status b_elapsed(C_Event a, C_Event b, float *ms) {
  if (!ms)
    return C_FAILED;
  return cerr(cudaEventElapsedTime(ms, (cudaEvent_t)a, (cudaEvent_t)b));
}
C_Status dev_attr(C_Device d, cudaDeviceAttr a, int *v) {
  if (!d || !v)
    return C_FAILED;
  return cerr(cudaDeviceGetAttribute(v, a, d->id));
}
C_Status b_capability(C_Device d, size_t *cap) {
  int ma = 0, mi = 0;
  if (!cap)
    return C_FAILED;
  C_Status s = dev_attr(d, cudaDevAttrComputeCapabilityMajor, &ma);
  if (s == C_SUCCESS)
    s = dev_attr(d, cudaDevAttrComputeCapabilityMinor, &mi);
  *cap = (size_t)(ma * 10 + mi);
  return s;
}
C_Status b_runtime_version(C_Device, size_t *v) {
  int r = 0;
  if (!v)
    return C_FAILED;
  C_Status s = cerr(cudaRuntimeGetVersion(&r));
  *v = (size_t)r;
  return s;
}
C_Status b_driver_version(C_Device, size_t *v) {
  int r = 0;
  if (!v)
    return C_FAILED;
  C_Status s = cerr(cudaDriverGetVersion(&r));
  *v = (size_t)r;
  return s;
}
C_Status attr_out(C_Device d, cudaDeviceAttr a, size_t *out) {
  int v = 0;
  if (!out)
    return C_FAILED;
  C_Status s = dev_attr(d, a, &v);
  *out = (size_t)v;
  return s;
}
C_Status b_multi_process(C_Device d, size_t *v) {
  return attr_out(d, cudaDevAttrMultiProcessorCount, v);
}
C_Status b_threads_per_mp(C_Device d, size_t *v) {
  return attr_out(d, cudaDevAttrMaxThreadsPerMultiProcessor, v);
}
C_Status b_threads_per_block(C_Device d, size_t *v) {
  return attr_out(d, cudaDevAttrMaxThreadsPerBlock, v);
}
C_Status b_grid_dims(C_Device d, size_t dims[3]) {
  if (!dims)
    return C_FAILED;
  C_Status s = attr_out(d, cudaDevAttrMaxGridDimX, &dims[0]);
  if (s == C_SUCCESS)
    s = attr_out(d, cudaDevAttrMaxGridDimY, &dims[1]);
  if (s == C_SUCCESS)
    s = attr_out(d, cudaDevAttrMaxGridDimZ, &dims[2]);
  return s;
}
C_Status b_device_name(C_Device d, char *buf, size_t n) {
  if (!d || !buf || n == 0)
    return C_FAILED;
  cudaDeviceProp prop;
  C_Status s = cerr(cudaGetDeviceProperties(&prop, d->id));
  if (s != C_SUCCESS)
    return s;
  std::strncpy(buf, prop.name, n - 1);
  buf[n - 1] = '\0';
  return C_SUCCESS;
}

// Named-event profiler: device time between CUDA events recorded on the
// legacy default stream after a device synchronisation, so the interval
// covers every stream's work between begin and end (the reference plugin
// measures host wall time around the same interval, cuda_device.cpp:632-762).
struct ProfEvent {
  std::string name;
  size_t calls = 0;
  double total = 0.0, mn = 1e300, mx = 0.0;
};
struct Profiler {
  std::string name;
  int dev = 0;
  bool running = false, in_event = false;
  std::string cur;
  cudaEvent_t a = nullptr, b = nullptr;
  std::unordered_map<std::string, ProfEvent> events;
  std::vector<C_ProfilerEvent> report;
};
void clear_report(Profiler *p) {
  for (auto &e : p->report)
    std::free(const_cast<char *>(e.name));
  p->report.clear();
}
C_Status b_prof_create(C_Profiler *prof, const char *name, int dev) {
  if (!prof)
    return C_FAILED;
  Profiler *p = new Profiler();
  p->name = name ? name : "";
  p->dev = dev;
  if (cudaSetDevice(dev) != cudaSuccess || cudaEventCreate(&p->a) != cudaSuccess ||
      cudaEventCreate(&p->b) != cudaSuccess) {
    delete p;
    set_last_error("profiler_create: CUDA event creation failed");
    return C_FAILED;
  }
  *prof = (C_Profiler)p;
  return C_SUCCESS;
}
C_Status b_prof_destroy(C_Profiler prof) {
  Profiler *p = (Profiler *)prof;
  if (!p)
    return C_FAILED;
  clear_report(p);
  cudaEventDestroy(p->a);
  cudaEventDestroy(p->b);
  delete p;
  return C_SUCCESS;
}
C_Status b_prof_start(C_Profiler prof) {
  if (!prof)
    return C_FAILED;
  ((Profiler *)prof)->running = true;
  return C_SUCCESS;
}
C_Status b_prof_stop(C_Profiler prof) {
  if (!prof)
    return C_FAILED;
  ((Profiler *)prof)->running = false;
  return C_SUCCESS;
}
C_Status b_prof_reset(C_Profiler prof) {
  Profiler *p = (Profiler *)prof;
  if (!p)
    return C_FAILED;
  p->events.clear();
  clear_report(p);
  return C_SUCCESS;
}
C_Status b_prof_begin(C_Profiler prof, const char *name) {
  Profiler *p = (Profiler *)prof;
  if (!p || !name)
    return C_FAILED;
  if (!p->running)
    return C_SUCCESS;
  cudaSetDevice(p->dev);
  cudaDeviceSynchronize();
  p->cur = name;
  p->in_event = true;
  return cerr(cudaEventRecord(p->a, 0));
}
C_Status b_prof_end(C_Profiler prof) {
  Profiler *p = (Profiler *)prof;
  if (!p)
    return C_FAILED;
  if (!p->running || !p->in_event)
    return C_SUCCESS;
  cudaSetDevice(p->dev);
  cudaDeviceSynchronize();
  C_Status s = cerr(cudaEventRecord(p->b, 0));
  if (s == C_SUCCESS)
    s = cerr(cudaEventSynchronize(p->b));
  float ms = 0.f;
  if (s == C_SUCCESS)
    s = cerr(cudaEventElapsedTime(&ms, p->a, p->b));
  p->in_event = false;
  if (s != C_SUCCESS)
    return s;
  ProfEvent &e = p->events[p->cur];
  e.name = p->cur;
  e.calls++;
  e.total += ms;
  e.mn = std::min(e.mn, (double)ms);
  e.mx = std::max(e.mx, (double)ms);
  return C_SUCCESS;
}
C_Status b_prof_events(C_Profiler prof, C_ProfilerEvent **events, size_t *count) {
  Profiler *p = (Profiler *)prof;
  if (!p || !events || !count)
    return C_FAILED;
  clear_report(p);
  for (auto &kv : p->events) {
    C_ProfilerEvent e;
    e.name = strdup(kv.second.name.c_str());
    e.calls = kv.second.calls;
    e.total_ms = (float)kv.second.total;
    e.min_ms = (float)(kv.second.mn < 1e299 ? kv.second.mn : 0.0);
    e.max_ms = (float)kv.second.mx;
    p->report.push_back(e);
  }
  *events = p->report.data();
  *count = p->report.size();
  return C_SUCCESS;
}

const char *b_last_error(void) { return ib200::last_error(); }

// ---------------------------------------------------------------------------
// Registered kernels
// ---------------------------------------------------------------------------
size_t count_args(void **a) {
  size_t n = 0;
  while (a && a[n])
    ++n;
  return n;
}

bool read_window(const InsightArray *w, std::vector<double> &out) {
  if (!w || w->dtype != INSIGHT_DTYPE_F64 || w->ndim != 1) {
    set_last_error("window must be a 1-D F64 array");
    return false;
  }
  const int64_t n = w->dims[0];
  out.resize(n);
  const double *base = reinterpret_cast<const double *>(w->data) + w->offset;
  const int64_t s = w->strides[0];
  if (w->device_type == INSIGHT_DEVICE_GPU) {
    std::vector<double> span(n > 0 ? (n - 1) * s + 1 : 0);
    if (!span.empty() &&
        cerr(cudaMemcpy(span.data(), base, span.size() * 8,
                        cudaMemcpyDeviceToHost)) != C_SUCCESS)
      return false;
    for (int64_t i = 0; i < n; ++i)
      out[i] = span[i * s];
  } else {
    for (int64_t i = 0; i < n; ++i)
      out[i] = base[i * s];
  }
  return true;
}

bool gpu_array(const InsightArray *a) {
  return a && a->device_type == INSIGHT_DEVICE_GPU;
}

C_Status accum_kernel(void **in, void **out, int op) {
  if (count_args(in) < 11 || count_args(out) < 1) {
    set_last_error("welch/csd kernel: expected 11 inputs and 1 output");
    return C_FAILED;
  }
  InsightArray *o = (InsightArray *)out[0];
  const InsightArray *x = (const InsightArray *)in[1];
  const InsightArray *y = (const InsightArray *)in[2];
  if (!gpu_array(o) || !gpu_array(x) || !gpu_array(y)) {
    set_last_error("welch/csd kernel: arrays must be GPU arrays");
    return C_FAILED;
  }
  std::vector<double> w;
  if (!read_window((const InsightArray *)in[3], w))
    return C_FAILED;
  ib200::Call c;
  c.op = op;
  c.x = x;
  c.y = op == INSIGHT_B200_OP_WELCH ? nullptr : y;
  c.out = o;
  c.window_values = &w;
  c.nperseg = *(int64_t *)in[4];
  c.noverlap = *(int64_t *)in[5];
  c.nfft = *(int64_t *)in[6];
  c.detrend_constant = *(int32_t *)in[7] == 1;
  c.detrend_linear = *(int32_t *)in[7] == 2;
  c.onesided = *(int32_t *)in[8] != 0;
  c.has_scale = true;
  c.scale = *(double *)in[9];
  c.axis = (int)*(int64_t *)in[10];
  c.sync = true;
  return ib200::run(c);
}

} // namespace

extern "C" {

const char *insight_b200_get_last_error(void) { return ib200::last_error(); }

int64_t insight_b200_launch_count(void) { return ib200::launch_count(); }

C_Status insight_b200_welch_kernel(void **inputs, void **outputs) {
  return accum_kernel(inputs, outputs, INSIGHT_B200_OP_WELCH);
}

C_Status insight_b200_csd_kernel(void **inputs, void **outputs) {
  return accum_kernel(inputs, outputs, INSIGHT_B200_OP_CSD);
}

C_Status insight_b200_coherence_kernel(void **inputs, void **outputs) {
  return accum_kernel(inputs, outputs, INSIGHT_B200_OP_COHERENCE);
}

C_Status insight_b200_istft_kernel(void **in, void **out) {
  if (count_args(in) < 6 || count_args(out) < 1) {
    set_last_error("istft kernel: expected 6 inputs and 1 output");
    return C_FAILED;
  }
  InsightArray *o = (InsightArray *)out[0];
  const InsightArray *z = (const InsightArray *)in[1];
  if (!gpu_array(o) || !gpu_array(z)) {
    set_last_error("istft kernel: arrays must be GPU arrays");
    return C_FAILED;
  }
  std::vector<double> w;
  if (!read_window((const InsightArray *)in[2], w))
    return C_FAILED;
  ib200::IstftCall c;
  c.z = z;
  c.out = o;
  c.window_values = &w;
  c.nperseg = *(int64_t *)in[3];
  c.noverlap = *(int64_t *)in[4];
  c.nfft = *(int64_t *)in[5];
  c.sync = true;
  return ib200::run_istft(c);
}

C_Status insight_b200_spectrogram_kernel(void **in, void **out) {
  if (count_args(in) < 11 || count_args(out) < 1) {
    set_last_error("spectrogram kernel: expected 11 inputs and 1 output");
    return C_FAILED;
  }
  InsightArray *o = (InsightArray *)out[0];
  const InsightArray *x = (const InsightArray *)in[1];
  if (!gpu_array(o) || !gpu_array(x)) {
    set_last_error("spectrogram kernel: arrays must be GPU arrays");
    return C_FAILED;
  }
  std::vector<double> w;
  if (!read_window((const InsightArray *)in[2], w))
    return C_FAILED;
  ib200::Call c;
  c.op = INSIGHT_B200_OP_SPECTROGRAM;
  c.x = x;
  c.out = o;
  c.window_values = &w;
  c.nperseg = *(int64_t *)in[3];
  c.noverlap = *(int64_t *)in[4];
  c.nfft = *(int64_t *)in[5];
  c.detrend_constant = *(int32_t *)in[6] == 1;
  c.detrend_linear = *(int32_t *)in[6] == 2;
  c.onesided = *(int32_t *)in[7] != 0;
  const int mode = *(int32_t *)in[8];
  c.mode = mode == 0 ? "psd" : mode == 1 ? "complex" : "magnitude";
  if (mode == 3 && !(o->dtype == INSIGHT_DTYPE_C32 || o->dtype == INSIGHT_DTYPE_C64)) {
    set_last_error("spectrogram kernel: mode 3 needs a C32/C64 output");
    return C_FAILED;
  }
  c.has_scale = true;
  c.scale = *(double *)in[9];
  c.axis = (int)*(int64_t *)in[10];
  c.sync = true;
  return ib200::run(c);
}

C_Status InitPluginGPU(CustomRuntimeParams *params) {
  if (!params || !params->interface)
    return C_ERROR;
  if (params->size != sizeof(CustomRuntimeParams) ||
      params->interface->size != sizeof(C_DeviceInterface))
    return C_ERROR;
  params->version.major = INSIGHT_CUSTOM_DEVICE_MAJOR_VERSION;
  params->version.minor = INSIGHT_CUSTOM_DEVICE_MINOR_VERSION;
  params->version.patch = INSIGHT_CUSTOM_DEVICE_PATCH_VERSION;

  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) {
    set_last_error("InitPluginGPU: no CUDA device visible");
    return C_FAILED;
  }
  int major = 0;
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, 0);
  if (major != 10) {
    set_last_error("InitPluginGPU: the B200 backend needs an sm_100 device");
    return C_FAILED;
  }

  C_DeviceInterface *f = params->interface;
  const size_t sz = f->size;
  std::memset(f, 0, sizeof(C_DeviceInterface));
  f->size = sz;
  f->initialize = b_initialize;
  f->finalize = b_finalize;
  f->init_device = b_init_device;
  f->deinit_device = b_deinit_device;
  f->set_device = b_set_device;
  f->get_device = b_get_device;
  f->synchronize_device = b_synchronize_device;
  f->get_device_count = b_get_device_count;
  f->get_device_list = b_get_device_list;
  f->device_memory_allocate = b_device_memory_allocate;
  f->device_memory_deallocate = b_device_memory_deallocate;
  f->host_memory_allocate = b_host_memory_allocate;
  f->host_memory_deallocate = b_host_memory_deallocate;
  f->memory_copy_h2d = b_copy_h2d;
  f->memory_copy_d2h = b_copy_d2h;
  f->memory_copy_d2d = b_copy_d2d;
  f->memory_copy_p2p = b_copy_p2p;
  f->device_memory_set = b_memset;
  f->device_memory_stats = b_memory_stats;
  f->async_memory_copy_h2d = b_acopy_h2d;
  f->async_memory_copy_d2h = b_acopy_d2h;
  f->async_memory_copy_d2d = b_acopy_d2d;
  f->async_memory_copy_p2p = b_acopy_p2p;
  f->create_stream = b_create_stream;
  f->destroy_stream = b_destroy_stream;
  f->query_stream = b_query_stream;
  f->synchronize_stream = b_sync_stream;
  f->stream_add_callback = b_stream_add_callback;
  f->stream_wait_event = b_stream_wait_event;
  f->create_event = b_create_event;
  f->destroy_event = b_destroy_event;
  f->record_event = b_record_event;
  f->query_event = b_query_event;
  f->synchronize_event = b_sync_event;
  f->elapsed_time = b_elapsed;
  f->get_compute_capability = b_capability;
  f->get_runtime_version = b_runtime_version;
  f->get_driver_version = b_driver_version;
  f->get_multi_process = b_multi_process;
  f->get_max_threads_per_mp = b_threads_per_mp;
  f->get_max_threads_per_block = b_threads_per_block;
  f->get_max_grid_dim_size = b_grid_dims;
  f->get_device_name = b_device_name;
  f->profiler_create = b_prof_create;
  f->profiler_destroy = b_prof_destroy;
  f->profiler_start = b_prof_start;
  f->profiler_stop = b_prof_stop;
  f->profiler_reset = b_prof_reset;
  f->profiler_begin_event = b_prof_begin;
  f->profiler_end_event = b_prof_end;
  f->profiler_get_events = b_prof_events;
  f->get_last_error = b_last_error;

  params->device_type = const_cast<char *>("b200");
  params->sub_device_type = const_cast<char *>("sm_100a");
  if (params->register_kernel) {
    const int32_t dts[2] = {INSIGHT_DTYPE_F32, INSIGHT_DTYPE_F64};
    for (int32_t dt : dts) {
      params->register_kernel("welch", INSIGHT_DEVICE_GPU, dt,
                              insight_b200_welch_kernel);
      params->register_kernel("csd", INSIGHT_DEVICE_GPU, dt,
                              insight_b200_csd_kernel);
      params->register_kernel("coherence", INSIGHT_DEVICE_GPU, dt,
                              insight_b200_coherence_kernel);
      params->register_kernel("spectrogram", INSIGHT_DEVICE_GPU, dt,
                              insight_b200_spectrogram_kernel);
      params->register_kernel("istft", INSIGHT_DEVICE_GPU,
                              dt == INSIGHT_DTYPE_F32 ? INSIGHT_DTYPE_C32
                                                      : INSIGHT_DTYPE_C64,
                              insight_b200_istft_kernel);
      params->register_kernel("stft", INSIGHT_DEVICE_GPU, dt,
                              insight_b200_spectrogram_kernel);
    }
  }
  return C_SUCCESS;
}

// ---------------------------------------------------------------------------
// Frontend entry points
// ---------------------------------------------------------------------------
static int current_device() {
  int d = 0;
  if (cudaGetDevice(&d) != cudaSuccess)
    d = 0;
  return d;
}

C_Status insight_b200_welch(const InsightArray *x, double fs, const char *window,
                            int64_t nperseg, int64_t noverlap, int64_t nfft,
                            const char *detrend, int return_onesided,
                            const char *scaling, InsightArray *f,
                            InsightArray *pxx) {
  ib200::Call c;
  c.op = INSIGHT_B200_OP_WELCH;
  c.x = x;
  c.out = pxx;
  c.f = f;
  c.fs = fs;
  c.window = window ? window : "hann";
  c.nperseg = nperseg;
  c.noverlap = noverlap;
  c.nfft = nfft;
  c.detrend_constant = detrend && std::string(detrend) == "constant";
  c.onesided = return_onesided != 0;
  c.scaling = scaling ? scaling : "density";
  c.default_device = current_device();
  return ib200::run(c);
}

C_Status insight_b200_csd(const InsightArray *x, const InsightArray *y,
                          double fs, const char *window, int64_t nperseg,
                          int64_t noverlap, int64_t nfft, const char *detrend,
                          int return_onesided, const char *scaling,
                          InsightArray *f, InsightArray *pxy) {
  ib200::Call c;
  c.op = INSIGHT_B200_OP_CSD;
  c.x = x;
  c.y = y;
  c.out = pxy;
  c.f = f;
  c.fs = fs;
  c.window = window ? window : "hann";
  c.nperseg = nperseg;
  c.noverlap = noverlap;
  c.nfft = nfft;
  c.detrend_constant = detrend && std::string(detrend) == "constant";
  c.onesided = return_onesided != 0;
  c.scaling = scaling ? scaling : "density";
  c.default_device = current_device();
  return ib200::run(c);
}

C_Status insight_b200_coherence(const InsightArray *x, const InsightArray *y,
                                double fs, const char *window, int64_t nperseg,
                                int64_t noverlap, int64_t nfft,
                                const char *detrend, InsightArray *f,
                                InsightArray *cxy) {
  ib200::Call c;
  c.op = INSIGHT_B200_OP_COHERENCE;
  c.x = x;
  c.y = y;
  c.out = cxy;
  c.f = f;
  c.fs = fs;
  c.window = window ? window : "hann";
  c.nperseg = nperseg;
  c.noverlap = noverlap;
  c.nfft = nfft;
  c.detrend_constant = detrend && std::string(detrend) == "constant";
  c.onesided = true;
  c.scaling = "density";
  c.default_device = current_device();
  return ib200::run(c);
}

C_Status insight_b200_periodogram(const InsightArray *x, double fs,
                                  const char *window, int64_t nfft,
                                  const char *detrend, int return_onesided,
                                  const char *scaling, InsightArray *f,
                                  InsightArray *pxx) {
  // periodogram = welch(x, fs, window, 256, 0, nfft, ...)
  // (spectral_analysis.cpp:189-193)
  return insight_b200_welch(x, fs, window ? window : "boxcar", 256, 0, nfft,
                            detrend, return_onesided, scaling, f, pxx);
}

C_Status insight_b200_istft_shape(const InsightArray *zxx, int64_t nperseg,
                                  int64_t noverlap, int64_t nfft,
                                  int64_t *n_channels, int64_t *n_total) {
  ib200::IstftCall c;
  c.z = zxx;
  c.nperseg = nperseg;
  c.noverlap = noverlap;
  c.nfft = nfft;
  return ib200::istft_shape(c, n_channels, n_total);
}

C_Status insight_b200_istft(const InsightArray *zxx, double fs,
                            const char *window, int64_t nperseg,
                            int64_t noverlap, int64_t nfft, InsightArray *out) {
  (void)fs; // the reference's istft does not use fs either
  ib200::IstftCall c;
  c.z = zxx;
  c.out = out;
  c.window = window ? window : "hann";
  c.nperseg = nperseg;
  c.noverlap = noverlap;
  c.nfft = nfft;
  c.default_device = current_device();
  return ib200::run_istft(c);
}

C_Status insight_b200_istft_async(const InsightArray *zxx, const char *window,
                                  int64_t nperseg, int64_t noverlap,
                                  int64_t nfft, InsightArray *out, void *stream,
                                  int sync) {
  ib200::IstftCall c;
  c.z = zxx;
  c.out = out;
  c.window = window ? window : "hann";
  c.nperseg = nperseg;
  c.noverlap = noverlap;
  c.nfft = nfft;
  c.default_device = current_device();
  c.stream = (cudaStream_t)stream;
  c.sync = sync != 0;
  return ib200::run_istft(c);
}

C_Status insight_b200_spectrogram(const InsightArray *x, double fs,
                                  const char *window, int64_t nperseg,
                                  int64_t noverlap, int64_t nfft,
                                  const char *detrend, int return_onesided,
                                  const char *mode, InsightArray *f,
                                  InsightArray *t, InsightArray *sxx) {
  ib200::Call c;
  c.op = INSIGHT_B200_OP_SPECTROGRAM;
  c.x = x;
  c.out = sxx;
  c.f = f;
  c.t = t;
  c.fs = fs;
  c.window = window ? window : "hann";
  c.nperseg = nperseg;
  c.noverlap = noverlap;
  c.nfft = nfft;
  c.detrend_constant = detrend && std::string(detrend) == "constant";
  c.onesided = return_onesided != 0;
  c.mode = mode ? mode : "psd";
  c.default_device = current_device();
  return ib200::run(c);
}

C_Status insight_b200_stft(const InsightArray *x, double fs, const char *window,
                           int64_t nperseg, int64_t noverlap, int64_t nfft,
                           InsightArray *f, InsightArray *t, InsightArray *zxx) {
  // stft = spectrogram(x, fs, window, nperseg, noverlap, nfft, "none", true,
  //                    "complex")  (spectral_analysis.cpp:330-334)
  ib200::Call c;
  c.op = INSIGHT_B200_OP_STFT;
  c.x = x;
  c.out = zxx;
  c.f = f;
  c.t = t;
  c.fs = fs;
  c.window = window ? window : "hann";
  c.nperseg = nperseg;
  c.noverlap = noverlap;
  c.nfft = nfft;
  c.detrend_constant = false;
  c.onesided = true;
  c.mode = "complex";
  c.default_device = current_device();
  return ib200::run(c);
}

static ib200::Call from_desc(const InsightB200SpectralDesc *d) {
  ib200::Call c;
  c.op = d->op;
  c.axis = d->axis;
  c.fs = d->fs;
  c.window = d->window ? d->window : "hann";
  c.nperseg = d->nperseg == 0 ? 256 : d->nperseg;
  c.noverlap = d->noverlap;
  c.nfft = d->nfft;
  const char *detrend = d->detrend ? d->detrend : "constant";
  c.detrend_constant = std::string(detrend) == "constant";
  // native option: least-squares line removal ('linear' stays the
  // reference's no-op)
  c.detrend_linear = std::string(detrend) == "linear_lsq";
  c.onesided = d->return_onesided != 0;
  c.scaling = d->scaling ? d->scaling : "density";
  c.mode = d->mode ? d->mode : "psd";
  if (d->op == INSIGHT_B200_OP_STFT) {
    c.detrend_constant = false;
    c.detrend_linear = false;
    c.onesided = true;
    c.mode = "complex";
  }
  c.seg_begin = d->seg_begin;
  c.seg_end = d->seg_end;
  c.raw_sums = d->raw_sums != 0;
  c.avg_segments = d->avg_segments;
  c.default_device = current_device();
  return c;
}

C_Status insight_b200_spectral_shape(const InsightB200SpectralDesc *desc,
                                     const InsightArray *x, int64_t *n_channels,
                                     int64_t *n_seg, int64_t *n_freq) {
  if (!desc) {
    set_last_error("spectral_shape: desc is NULL");
    return C_FAILED;
  }
  ib200::Call c = from_desc(desc);
  c.x = x;
  return ib200::shape(c, n_channels, n_seg, n_freq);
}

C_Status insight_b200_spectral(const InsightB200SpectralDesc *desc,
                               const InsightArray *x, const InsightArray *y,
                               InsightArray *out, InsightArray *f,
                               InsightArray *t, void *stream, int sync) {
  if (!desc) {
    set_last_error("spectral: desc is NULL");
    return C_FAILED;
  }
  ib200::Call c = from_desc(desc);
  c.x = x;
  c.y = y;
  c.out = out;
  c.f = f;
  c.t = t;
  c.stream = (cudaStream_t)stream;
  c.sync = sync != 0;
  return ib200::run(c);
}

C_Status insight_b200_plan_create(const InsightB200SpectralDesc *desc,
                                  const InsightArray *x, const InsightArray *y,
                                  InsightArray *out, void *stream,
                                  InsightB200Plan **plan) {
  if (!desc || !plan) {
    set_last_error("plan: desc or plan handle is NULL");
    return C_FAILED;
  }
  ib200::Call c = from_desc(desc);
  c.x = x;
  c.y = y;
  c.out = out;
  c.stream = (cudaStream_t)stream;
  void *p = nullptr;
  const C_Status s = ib200::plan_create(c, &p);
  *plan = static_cast<InsightB200Plan *>(p);
  return s;
}

C_Status insight_b200_plan_execute(InsightB200Plan *plan, void *stream, int sync) {
  return ib200::plan_execute(plan, (cudaStream_t)stream, sync != 0);
}

C_Status insight_b200_plan_destroy(InsightB200Plan *plan) {
  return ib200::plan_destroy(plan);
}

C_Status insight_b200_finalize_sums(const InsightB200SpectralDesc *desc,
                                    int64_t n_seg, int32_t x_dtype,
                                    InsightArray *sums, void *stream) {
  if (!desc) {
    set_last_error("finalize_sums: desc is NULL");
    return C_FAILED;
  }
  ib200::Call c = from_desc(desc);
  c.x_dtype = x_dtype;
  c.stream = (cudaStream_t)stream;
  c.sync = stream == nullptr;
  return ib200::finalize_sums(c, n_seg, sums);
}

} // extern "C"

/* insight_b200.h — C ABI of the B200 spectral-estimation backend.
 *
 * libinsight_b200_backend.so is a drop-in Insight GPU device plugin for the
 * spectral-estimation ops (welch, csd, spectrogram, stft).  It exposes:
 *
 *  1. The plugin factory InitPluginGPU (replaces
 *     backends/cuda/device/cuda_device.cpp:769 InitPluginGPU; declared in
 *     include/insight/c_api/device_ext.h:905).  It fills C_DeviceInterface
 *     (device_ext.h:156-768) and registers the kernels "welch", "csd",
 *     "spectrogram" and "stft" for INSIGHT_DEVICE_GPU x {F32, F64} through
 *     params->register_kernel (device_ext.h:847).
 *
 *  2. The registered kernels, with the reference kernel signature
 *     C_Status fn(void **inputs, void **outputs)  (include/insight/c_api/kernel.h:21),
 *     also exported by name so a host can bind them without the registry.
 *
 *  3. Host entry points with the argument meaning, defaults and error
 *     behaviour of the reference frontend
 *     ins::signal::{welch, csd, spectrogram, stft}
 *     (include/insight/ops/signal/spectral_analysis.h:40-96,
 *      src/ops/signal/spectral_analysis.cpp:104-334),
 *     taking InsightArray descriptors (include/insight/c_api/array.h:19-31)
 *     in host or device memory, plus a batched native entry point.
 *
 * The ABI types below have the exact layout of the reference's c_api types.
 * A translation unit that already includes the reference's headers defines
 * INSIGHT_B200_USE_INSIGHT_HEADERS before including this file and the
 * reference definitions are used instead.
 */
#ifndef INSIGHT_B200_H
#define INSIGHT_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(INSIGHT_B200_USE_INSIGHT_HEADERS)
#include "insight/c_api/array.h"
#include "insight/c_api/device_ext.h"
#include "insight/c_api/place.h"
#else

/* include/insight/c_api/dtype.h:10-39 */
typedef enum {
  C_SUCCESS = 0,
  C_WARNING,
  C_FAILED,
  C_ERROR,
  C_INTERNAL_ERROR,
  C_FALLBACK
} C_Status;

typedef enum {
  INSIGHT_DTYPE_UNKNOWN = 0,
  INSIGHT_DTYPE_BOOL,
  INSIGHT_DTYPE_U8,
  INSIGHT_DTYPE_I8,
  INSIGHT_DTYPE_I16,
  INSIGHT_DTYPE_I32,
  INSIGHT_DTYPE_I64,
  INSIGHT_DTYPE_F16,
  INSIGHT_DTYPE_BF16,
  INSIGHT_DTYPE_F32,
  INSIGHT_DTYPE_F64,
  INSIGHT_DTYPE_C32, /* complex64  */
  INSIGHT_DTYPE_C64, /* complex128 */
  INSIGHT_DTYPE_F8_E4M3,
  INSIGHT_DTYPE_F8_E5M2,
  INSIGHT_DTYPE_U16,
  INSIGHT_DTYPE_U32,
  INSIGHT_DTYPE_U64,
  INSIGHT_DTYPE_COUNT
} InsightDType;

/* include/insight/c_api/place.h:10-13 */
typedef enum { INSIGHT_DEVICE_CPU = 0, INSIGHT_DEVICE_GPU = 1 } InsightDeviceType;

/* include/insight/c_api/array.h:10-31: data is the storage base, offset and
 * strides are in elements. */
#define INSIGHT_MAX_NDIM 10
typedef struct {
  void *data;
  int64_t dims[INSIGHT_MAX_NDIM];
  int64_t strides[INSIGHT_MAX_NDIM];
  int32_t ndim;
  int64_t numel;
  int32_t dtype;
  int32_t device_type;
  int32_t device_id;
  int64_t offset;
  int32_t is_view;
  int32_t *ref_count;
} InsightArray;

/* include/insight/c_api/kernel.h:21 */
typedef C_Status (*InsightKernel)(void **inputs, void **outputs);

/* include/insight/c_api/device_ext.h:66-768 */
#define INSIGHT_CUSTOM_DEVICE_MAJOR_VERSION 1
#define INSIGHT_CUSTOM_DEVICE_MINOR_VERSION 0
#define INSIGHT_CUSTOM_DEVICE_PATCH_VERSION 0

typedef struct C_Device_st *C_Device;
typedef struct C_Stream_st *C_Stream;
typedef struct C_Event_st *C_Event;
typedef struct C_Profiler_st *C_Profiler;

typedef struct C_ProfilerEvent {
  const char *name;
  size_t calls;
  float total_ms;
  float min_ms;
  float max_ms;
} C_ProfilerEvent;

struct C_Device_st {
  int id;
};

typedef struct C_DeviceInterface {
  size_t size;
  C_Status (*initialize)(void);
  C_Status (*finalize)(void);
  C_Status (*init_device)(C_Device device);
  C_Status (*deinit_device)(C_Device device);
  C_Status (*set_device)(C_Device device);
  C_Status (*get_device)(C_Device device);
  C_Status (*synchronize_device)(C_Device device);
  C_Status (*get_device_count)(size_t *count);
  C_Status (*get_device_list)(size_t *devices);
  C_Status (*device_memory_allocate)(C_Device device, void **ptr, size_t size);
  C_Status (*device_memory_deallocate)(C_Device device, void *ptr, size_t size);
  C_Status (*host_memory_allocate)(C_Device device, void **ptr, size_t size);
  C_Status (*host_memory_deallocate)(C_Device device, void *ptr, size_t size);
  C_Status (*memory_copy_h2d)(C_Device device, void *dst, const void *src,
                              size_t size);
  C_Status (*memory_copy_d2h)(C_Device device, void *dst, const void *src,
                              size_t size);
  C_Status (*memory_copy_d2d)(C_Device device, void *dst, const void *src,
                              size_t size);
  C_Status (*memory_copy_p2p)(C_Device dst_device, C_Device src_device,
                              void *dst, const void *src, size_t size);
  C_Status (*device_memory_set)(C_Device device, void *ptr, unsigned char value,
                                size_t size);
  C_Status (*device_memory_stats)(C_Device device, size_t *total_memory,
                                  size_t *free_memory);
  C_Status (*async_memory_copy_h2d)(C_Device device, C_Stream stream, void *dst,
                                    const void *src, size_t size);
  C_Status (*async_memory_copy_d2h)(C_Device device, C_Stream stream, void *dst,
                                    const void *src, size_t size);
  C_Status (*async_memory_copy_d2d)(C_Device device, C_Stream stream, void *dst,
                                    const void *src, size_t size);
  C_Status (*async_memory_copy_p2p)(C_Device dst_device, C_Device src_device,
                                    C_Stream stream, void *dst, const void *src,
                                    size_t size);
  C_Status (*create_stream)(C_Device device, C_Stream *stream);
  C_Status (*destroy_stream)(C_Device device, C_Stream stream);
  C_Status (*query_stream)(C_Device device, C_Stream stream);
  C_Status (*synchronize_stream)(C_Device device, C_Stream stream);
  C_Status (*stream_add_callback)(C_Device device, C_Stream stream,
                                  void (*callback)(C_Device device,
                                                   C_Stream stream,
                                                   void *user_data,
                                                   C_Status *status),
                                  void *user_data);
  C_Status (*stream_wait_event)(C_Device device, C_Stream stream,
                                C_Event event);
  C_Status (*create_event)(C_Device device, C_Event *event);
  C_Status (*destroy_event)(C_Device device, C_Event event);
  C_Status (*record_event)(C_Device device, C_Stream stream, C_Event event);
  C_Status (*query_event)(C_Device device, C_Event event);
  C_Status (*synchronize_event)(C_Device device, C_Event event);
  C_Status (*elapsed_time)(C_Event start, C_Event end, float *ms);
  C_Status (*get_compute_capability)(C_Device device, size_t *capability);
  C_Status (*get_runtime_version)(C_Device device, size_t *version);
  C_Status (*get_driver_version)(C_Device device, size_t *version);
  C_Status (*get_multi_process)(C_Device device, size_t *multi_process);
  C_Status (*get_max_threads_per_mp)(C_Device device, size_t *threads);
  C_Status (*get_max_threads_per_block)(C_Device device, size_t *threads);
  C_Status (*get_max_grid_dim_size)(C_Device device, size_t dims[3]);
  C_Status (*get_device_name)(C_Device device, char *buf, size_t buf_size);
  C_Status (*profiler_create)(C_Profiler *prof, const char *name,
                              int device_id);
  C_Status (*profiler_destroy)(C_Profiler prof);
  C_Status (*profiler_start)(C_Profiler prof);
  C_Status (*profiler_stop)(C_Profiler prof);
  C_Status (*profiler_reset)(C_Profiler prof);
  C_Status (*profiler_begin_event)(C_Profiler prof, const char *name);
  C_Status (*profiler_end_event)(C_Profiler prof);
  C_Status (*profiler_get_events)(C_Profiler prof, C_ProfilerEvent **events,
                                  size_t *count);
  const char *(*get_last_error)(void);
  void *reserved[8];
} C_DeviceInterface;

typedef struct CustomRuntimeVersion {
  size_t major;
  size_t minor;
  size_t patch;
} CustomRuntimeVersion;

typedef struct CustomRuntimeParams {
  size_t size;
  C_DeviceInterface *interface;
  CustomRuntimeVersion version;
  char *device_type;
  char *sub_device_type;
  C_Status (*register_kernel)(const char *op_name, int32_t device_type,
                              int32_t dtype, InsightKernel kernel);
  char reserved[32];
} CustomRuntimeParams;

#endif /* INSIGHT_B200_USE_INSIGHT_HEADERS */

#if defined(__GNUC__)
#define INSIGHT_B200_API __attribute__((visibility("default")))
#else
#define INSIGHT_B200_API
#endif

/* ------------------------------------------------------------------------ */
/* 1. Plugin factory                                                         */
/* ------------------------------------------------------------------------ */

/* Replaces InitPluginGPU (backends/cuda/device/cuda_device.cpp:769-862).
 * Checks params->size / params->interface->size like
 * INSIGHT_CHECK_CUSTOM_DEVICE_VERSION (device_ext.h:873-882), fills the
 * version, every C_DeviceInterface slot the core calls, device_type "b200",
 * and registers the kernels below.  Returns C_ERROR on a size mismatch and
 * C_FAILED when no sm_100 device is visible. */
INSIGHT_B200_API C_Status InitPluginGPU(CustomRuntimeParams *params);

/* Thread-local message of the last failing call (C_DeviceInterface
 * get_last_error, cuda_device.cpp:25-38). */
INSIGHT_B200_API const char *insight_b200_get_last_error(void);

/* ------------------------------------------------------------------------ */
/* 2. Registered kernels (reference kernel signature, kernel.h:21)           */
/* ------------------------------------------------------------------------ */
/* Argument convention follows the reference's FFT kernel
 * (backends/cpu/kernels/fft/fft_c2c.cpp:9-16): inputs[0] is the output
 * array, then the input arrays, then pointers to host scalars; both lists
 * are NULL-terminated; outputs[0] is the result.  All arrays must be GPU
 * arrays (device_type INSIGHT_DEVICE_GPU, device_id honoured); strides and
 * offset are honoured.  Calls are synchronous.  A kernel never returns
 * C_FALLBACK: failures are C_FAILED with insight_b200_get_last_error().
 *
 * "welch" / "csd"   (ops registered for F32 and F64 inputs)
 *   inputs = { out     F64 [n_freq] or [C, n_freq] (C64 allowed: complex Pxy),
 *              x       F32/F64 [n] or 2-D (sample axis = *axis),
 *              y       same shape/dtype as x (pass x again for welch),
 *              window  F64 [nperseg], CPU or GPU (get_window(window, nperseg,
 *                      false) of the frontend, spectral_analysis.cpp:39-41),
 *              int64_t *nperseg, int64_t *noverlap (resolved, > 0),
 *              int64_t *nfft (resolved, >= nperseg),
 *              int32_t *detrend   (0 none, 1 constant; 'linear' -> 0 as the
 *                                  reference, spectral_analysis.cpp:79;
 *                                  2 = least-squares line removal after the
 *                                  window, an extension with no reference
 *                                  counterpart),
 *              int32_t *onesided,
 *              double  *scale     (compute_psd_scale, spectral_analysis.cpp:57-67),
 *              int64_t *axis,
 *              NULL }
 *   outputs = { out, NULL }
 *   out[c, k] = scale / n_seg * m[k] * sum_s Re(conj(X_s[k]) Y_s[k]),
 *   m = 2 on bins 1..n_freq-2 when onesided.
 *
 * "spectrogram" / "stft"
 *   inputs = { out     F64 (n_freq, n_seg) contiguous per channel, or
 *                      [C, n_freq, n_seg]; C32/C64 for the complex STFT,
 *              x, window F64 [nperseg],
 *              int64_t *nperseg, int64_t *noverlap (resolved, > 0),
 *              int64_t *nfft, int32_t *detrend, int32_t *onesided,
 *              int32_t *mode (0 psd, 1 complex = Re(X), 2 magnitude,
 *                             3 complex spectrum X itself),
 *              double  *scale (psd mode), int64_t *axis, NULL }
 *   The (n_freq, n_seg) buffer is what the reference builds before returning
 *   its transposed (n_seg, n_freq) view (spectral_analysis.cpp:256,321).
 */
INSIGHT_B200_API C_Status insight_b200_welch_kernel(void **inputs,
                                                    void **outputs);
INSIGHT_B200_API C_Status insight_b200_csd_kernel(void **inputs,
                                                  void **outputs);
INSIGHT_B200_API C_Status insight_b200_spectrogram_kernel(void **inputs,
                                                          void **outputs);
/* "coherence" (F32 / F64): inputs as "csd" with out F64 [n_freq] or
 * [C, n_freq]; onesided must be 1 (the reference's coherence is one-sided). */
INSIGHT_B200_API C_Status insight_b200_coherence_kernel(void **inputs,
                                                        void **outputs);
/* "istft" (registered for C32 and C64 Zxx):
 *   inputs = { out F64 [n_total] or [C, n_total], Zxx, window F64 [nperseg],
 *              int64_t *nperseg, int64_t *noverlap, int64_t *nfft (each 0 ->
 *              the reference default), NULL }
 *   outputs = { out, NULL } */
INSIGHT_B200_API C_Status insight_b200_istft_kernel(void **inputs,
                                                    void **outputs);

/* ------------------------------------------------------------------------ */
/* 3. Host entry points                                                      */
/* ------------------------------------------------------------------------ */

/* Frontend functions with the reference's argument meaning and defaults
 * (spectral_analysis.h:40-96; bindings/python/insight_py.cpp:1585-1610):
 *   noverlap == 0 -> nperseg/2 (welch, csd) or nperseg/8 (spectrogram, stft),
 *   nfft == 0 -> nperseg, window by name (symmetric, get_window(.., false)),
 *   detrend "constant" subtracts the mean after windowing, any other string
 *   (including "linear") does not detrend, scaling "density" -> fs/sum(w^2),
 *   otherwise 1/sum(w^2).
 * x (and y) may be CPU or GPU arrays, 1-D (the reference) or 2-D (a batch of
 * channels; the sample axis is the last one unless the array is a
 * transposed view with unit sample stride along axis 0).  Results are
 * written into caller-allocated arrays f [n_freq] (F64), pxx [n_freq] or
 * [C, n_freq] (F64; C32/C64 requests the complex cross spectrum), t [n_seg]
 * (F64), sxx (F64 [n_seg, n_freq] or a C32/C64 [C, n_freq, n_seg] complex
 * STFT); each may live on the CPU or the GPU.  f and t may be NULL.
 * Use insight_b200_spectral_shape first to size the outputs. */
INSIGHT_B200_API C_Status insight_b200_welch(
    const InsightArray *x, double fs, const char *window, int64_t nperseg,
    int64_t noverlap, int64_t nfft, const char *detrend, int return_onesided,
    const char *scaling, InsightArray *f, InsightArray *pxx);

INSIGHT_B200_API C_Status insight_b200_csd(
    const InsightArray *x, const InsightArray *y, double fs, const char *window,
    int64_t nperseg, int64_t noverlap, int64_t nfft, const char *detrend,
    int return_onesided, const char *scaling, InsightArray *f,
    InsightArray *pxy);

INSIGHT_B200_API C_Status insight_b200_spectrogram(
    const InsightArray *x, double fs, const char *window, int64_t nperseg,
    int64_t noverlap, int64_t nfft, const char *detrend, int return_onesided,
    const char *mode, InsightArray *f, InsightArray *t, InsightArray *sxx);

INSIGHT_B200_API C_Status insight_b200_stft(const InsightArray *x, double fs,
                                            const char *window, int64_t nperseg,
                                            int64_t noverlap, int64_t nfft,
                                            InsightArray *f, InsightArray *t,
                                            InsightArray *zxx);

/* Replaces ins::signal::coherence (spectral_analysis.h:76-82,
 * spectral_analysis.cpp:199-221): Cxy = Pxy^2 / max(Pxx Pyy, 1e-30) (0 where
 * Pxx Pyy <= 1e-30) with Pxx, Pyy from welch and Pxy the real part that the
 * reference's csd returns, all one-sided with 'density' scaling, as the
 * reference composes them.  Computed in one pass over x and y.  cxy is F64
 * [n_freq] or [C, n_freq]. */
INSIGHT_B200_API C_Status insight_b200_coherence(
    const InsightArray *x, const InsightArray *y, double fs, const char *window,
    int64_t nperseg, int64_t noverlap, int64_t nfft, const char *detrend,
    InsightArray *f, InsightArray *cxy);

/* Replaces ins::signal::periodogram (spectral_analysis.h:66-74,
 * spectral_analysis.cpp:189-193), which is welch with nperseg 256 and the
 * default overlap (128); the window defaults to "boxcar" there.  pxx as in
 * insight_b200_welch. */
INSIGHT_B200_API C_Status insight_b200_periodogram(
    const InsightArray *x, double fs, const char *window, int64_t nfft,
    const char *detrend, int return_onesided, const char *scaling,
    InsightArray *f, InsightArray *pxx);

/* Replaces ins::signal::istft (spectral_analysis.h:110-113,
 * spectral_analysis.cpp:340-457): overlap-add inverse of a one-sided (or
 * full) complex STFT Zxx (n_freq, n_frames), C32 or C64 (the reference reads
 * C64), 2-D or a 3-D [C, n_freq, n_frames] batch, any strides; defaults
 * nfft = 2 (n_freq - 1), nperseg = nfft, noverlap = nperseg / 2; fs is
 * unused, as in the reference.  out is F64 [n_total] (or [C, n_total]),
 * n_total = (n_frames - 1) * (nperseg - noverlap) + nperseg; use
 * insight_b200_istft_shape to size it. */
INSIGHT_B200_API C_Status insight_b200_istft_shape(const InsightArray *zxx,
                                                   int64_t nperseg,
                                                   int64_t noverlap,
                                                   int64_t nfft,
                                                   int64_t *n_channels,
                                                   int64_t *n_total);
INSIGHT_B200_API C_Status insight_b200_istft(const InsightArray *zxx, double fs,
                                             const char *window, int64_t nperseg,
                                             int64_t noverlap, int64_t nfft,
                                             InsightArray *out);
/* insight_b200_istft on a caller stream (cudaStream_t of Zxx's device, NULL
 * -> the backend's own); returns after enqueueing when sync == 0 and Zxx and
 * out are GPU arrays. */
INSIGHT_B200_API C_Status insight_b200_istft_async(
    const InsightArray *zxx, const char *window, int64_t nperseg,
    int64_t noverlap, int64_t nfft, InsightArray *out, void *stream, int sync);

/* Operation codes of the native entry point. */
enum {
  INSIGHT_B200_OP_WELCH = 0,
  INSIGHT_B200_OP_CSD = 1,
  INSIGHT_B200_OP_SPECTROGRAM = 2,
  INSIGHT_B200_OP_STFT = 3,
  INSIGHT_B200_OP_COHERENCE = 4
};

/* Native description of one spectral call (strings as in the frontend). */
typedef struct InsightB200SpectralDesc {
  int32_t op;               /* INSIGHT_B200_OP_*                            */
  int32_t axis;             /* sample axis of x / y; -1 = last              */
  double fs;
  const char *window;       /* NULL -> "hann"                               */
  int64_t nperseg;          /* 0 -> 256                                     */
  int64_t noverlap;         /* 0 -> reference default for the op            */
  int64_t nfft;             /* 0 -> nperseg                                 */
  const char *detrend;      /* NULL -> "constant"; "linear_lsq" removes the */
                            /* least-squares line after the window (the     */
                            /* reference's "linear" does not detrend)       */
  int32_t return_onesided;
  const char *scaling;      /* welch/csd; NULL -> "density"                 */
  const char *mode;         /* spectrogram; NULL -> "psd"                   */
  int64_t seg_begin;        /* segment range [seg_begin, seg_end) of this   */
  int64_t seg_end;          /* call; seg_end <= 0 -> all segments           */
  int32_t raw_sums;         /* welch/csd: write unscaled F64 sums (for a    */
                            /* cross-device reduction) instead of the PSD   */
  int64_t avg_segments;     /* welch/csd: average over this many segments   */
                            /* instead of the call's own count (0 -> own).  */
                            /* A shard that holds only its segment range of */
                            /* a longer signal passes the whole signal's    */
                            /* count: the shards' outputs then sum to the   */
                            /* PSD, so a plain all-reduce is the last step  */
} InsightB200SpectralDesc;

/* Output geometry of a call: channels, segments (of the whole signal), bins. */
INSIGHT_B200_API C_Status insight_b200_spectral_shape(
    const InsightB200SpectralDesc *desc, const InsightArray *x,
    int64_t *n_channels, int64_t *n_seg, int64_t *n_freq);

/* Run one call.  stream is a cudaStream_t of x's device (NULL -> the
 * backend's own stream for that device); the call returns after the work is
 * enqueued when sync == 0 and all inputs and outputs are GPU arrays,
 * otherwise it returns with the results in place. */
INSIGHT_B200_API C_Status insight_b200_spectral(
    const InsightB200SpectralDesc *desc, const InsightArray *x,
    const InsightArray *y, InsightArray *out, InsightArray *f, InsightArray *t,
    void *stream, int sync);

/* A plan: one insight_b200_spectral call captured into a CUDA graph.  No
 * counterpart in the reference (its spectral ops are per-call composites).
 * For callers that repeat the same call on the same GPU arrays and are
 * bound by launch and host overhead (short signals, tight loops): executing
 * a plan is one graph launch instead of the call's host-side planning and
 * kernel launches.
 * plan_create takes the arguments of insight_b200_spectral (x, y, out must
 * be GPU arrays; no f / t axes), runs the call once on the plan's own
 * stream (ordered after `stream`, NULL: none), then captures it.  The plan
 * keeps the arrays' device addresses: each execution recomputes out from
 * the current contents of x (and y).  It owns its working buffers, so
 * executions of one plan must not overlap on the GPU (different plans may).
 * plan_execute launches the graph on `stream` (NULL: the plan's stream) and
 * returns at once (sync == 0) or after the stream has finished (sync != 0).
 * plan_destroy waits for the device, then releases the plan. */
typedef struct InsightB200Plan InsightB200Plan;
INSIGHT_B200_API C_Status insight_b200_plan_create(
    const InsightB200SpectralDesc *desc, const InsightArray *x,
    const InsightArray *y, InsightArray *out, void *stream,
    InsightB200Plan **plan);
INSIGHT_B200_API C_Status insight_b200_plan_execute(InsightB200Plan *plan,
                                                    void *stream, int sync);
INSIGHT_B200_API C_Status insight_b200_plan_destroy(InsightB200Plan *plan);

/* Scale and mask F64 raw sums of welch/csd (raw_sums = 1) in place after
 * they were reduced across devices: out = sums * scale / n_seg * m[k].
 * sums is a GPU array [n_freq] or [C, n_freq] (F64, or C64 for complex
 * sums).  n_seg is the segment count of the whole signal. */
INSIGHT_B200_API C_Status insight_b200_finalize_sums(
    const InsightB200SpectralDesc *desc, int64_t n_seg, int32_t x_dtype,
    InsightArray *sums, void *stream);

/* Welch PSD without any device allocation.  No counterpart in the
 * reference: it exists for callers that cannot let a library allocate device
 * memory, such as a host framework that hands out every GPU buffer from its
 * own pool, or a latency-critical path that must not pay the implicit device
 * synchronisation of cudaMalloc / cudaFree.
 * x is a device pointer (current device) to sample 0 of channel 0, with
 * element strides channel_stride / sample_stride; pxx is a device pointer to
 * an F64 [n_channels, n_freq] contiguous result.  Arguments mean what they
 * mean in insight_b200_welch.  The working memory (twiddles, window, partial
 * sums) is an 8 MiB file-scope device array that every GPU loading this
 * library holds until exit; calls needing more (n_channels * (nfft/2+1) * 8
 * bytes beyond ~8 MiB) and constant detrend with nfft > nperseg are rejected
 * with C_FAILED.  The first call on a device looks up the array's device
 * address (cudaGetSymbolAddress); make that first call before any stream
 * capture.  All calls on a device share the array, so calls that overlap on
 * the GPU race.  stream is a cudaStream_t (NULL: legacy default stream); the
 * call returns after the stream has finished the work. */
INSIGHT_B200_API C_Status insight_b200_welch_noalloc(
    const void *x, int32_t dtype, int64_t n_channels, int64_t n_samples,
    int64_t channel_stride, int64_t sample_stride, double fs,
    const char *window, int64_t nperseg, int64_t noverlap, int64_t nfft,
    const char *detrend, int32_t return_onesided, const char *scaling,
    double *pxx, void *stream);

/* Kernel launches issued by this process so far (all devices). */
INSIGHT_B200_API int64_t insight_b200_launch_count(void);

#ifdef __cplusplus
}
#endif

#endif /* INSIGHT_B200_H */

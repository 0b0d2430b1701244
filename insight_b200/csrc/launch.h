// launch.h — device-side launch interface shared by the frontend and the
// per-dtype kernel translation units.
#pragma once
#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

namespace ib200 {

// LK_COH: magnitude-squared coherence of x and y (one pass: Sxx, Syy, Sxy).
enum LaunchKind { LK_PSD = 0, LK_CSD = 1, LK_STORE = 2, LK_COH = 3 };

// What the kernels write.
enum OutKindK {
  OUT_C64_K = 0,      // complex64 (store kernel: complex of the compute dtype)
  OUT_REAL_F64_K = 1, // Re(.) as double: reference csd/welch value, stft
  OUT_PSD_F64_K = 2,  // |X|^2 * scale * mask as double (spectrogram 'psd')
  OUT_MAG_F64_K = 3,  // |X| as double (spectrogram 'magnitude')
  OUT_RAW_F64_K = 4,  // unscaled sums (welch: double, csd: double2)
  OUT_C128_K = 5,     // complex128
};

struct LaunchDesc {
  int kind = LK_PSD;
  bool f64 = false;       // compute dtype: false f32, true f64
  int64_t nfft = 0;       // transform length L (power of two, 16..8192)
  int64_t nperseg = 0, step = 0;
  int64_t C = 1;          // channels
  int64_t seg0 = 0;       // first segment handled by this launch
  int64_t S = 0;          // segments handled by this launch, per channel
  const void *x = nullptr, *y = nullptr; // sample 0 of channel 0
  int64_t x_cs = 0, x_ss = 1, y_cs = 0, y_ss = 1;
  const void *win = nullptr;  // [nfft] window in compute dtype
  const void *tw = nullptr;   // [nfft] twiddles in compute dtype
  const void *dtab = nullptr; // [nfft] detrend correction table
  int dc_mode = 0; // 0 none, 1 DC bin, 2 zero-padded mean, 3 least-squares line
  int64_t F = 0;              // bins written
  bool onesided_mask = false;
  // welch / csd result
  double avg_scale = 1.0;
  int out_kind = 0;           // OutKindK
  void *out = nullptr;
  int64_t o_cs = 0, o_rs = 0, o_ts = 0; // elements
  double psd_scale = 1.0;     // spectrogram 'psd'
  int64_t max_units = 0;      // welch / csd: cap on work units (0 = none)
};

// Bytes of scratch the launch needs (welch / csd unit partials).
// Transforms per channel: segment pairs, except csd / coherence with f64
// nfft = 8192 (one segment per transform, x_s and y_s packed; packs_xy in
// spectral_kernels.cuh).
inline int64_t tasks_per_channel(const LaunchDesc &d) {
  const bool two = d.kind == LK_CSD || d.kind == LK_COH;
  return (two && d.f64 && d.nfft >= 8192) ? d.S : (d.S + 1) / 2;
}

// Upper bound on resident CTAs per SM used by the flat welch / csd split
// (its scratch holds grid + channels - 1 partial slots).
constexpr int kFlatMaxBlocksPerSm = 8;

size_t scratch_bytes(const LaunchDesc &d, int num_sms);

// Enqueue the kernels on `stream`.  scratch must hold scratch_bytes(d).
cudaError_t launch(const LaunchDesc &d, void *scratch, int num_sms,
                   cudaStream_t stream, int64_t *launches);

bool nfft_supported(int64_t nfft);

// Inverse STFT (overlap-add) of a complex [C, F, S] array.
struct IstftDesc {
  bool f64 = false;         // complex128 input (else complex64)
  int64_t C = 1, F = 0, S = 0;
  int64_t nfft = 0, nperseg = 0, hop = 0, n_total = 0;
  bool pack = true;         // F == nfft/2 + 1: Hermitian frame pairs
  const void *z = nullptr;  // element (c, k, i) at z[c*z_cs + k*z_fs + i*z_ts]
  int64_t z_cs = 0, z_fs = 0, z_ts = 0;
  const void *win = nullptr;    // [nperseg] window (f64: the transform dtype)
  const double *win64 = nullptr; // [nperseg] window, f64 (normalisation)
  const void *tw = nullptr;     // [nfft] f64 twiddles
  void *frames = nullptr;       // scratch [C][S][nperseg], input precision
  double *out = nullptr;        // element (c, m) at out[c*o_cs + m*o_ss]
  int64_t o_cs = 0, o_ss = 1;
};
cudaError_t launch_istft(const IstftDesc &d, int num_sms, cudaStream_t stream,
                         int64_t *launches);

// Per-dtype entry points (one translation unit each).
cudaError_t launch_f32(const LaunchDesc &d, void *scratch, int num_sms,
                       cudaStream_t stream, int64_t *launches);
cudaError_t launch_f64(const LaunchDesc &d, void *scratch, int num_sms,
                       cudaStream_t stream, int64_t *launches);

// Work split of the welch / csd kernels.
struct AccSplit {
  int64_t Tc, Qt, nq, U;
  int grid;
};
AccSplit acc_split(const LaunchDesc &d, int num_sms, int blocks_per_sm);

// f[i] = i * df (F values) and t[i] = (i * step + half) / fs (S values) on the
// device, bit-identical to the same double expressions on the host; a null
// pointer skips that axis.
cudaError_t write_axes_device(double *f, int64_t F, double df, double *t,
                              int64_t S, int64_t step, double half, double fs,
                              cudaStream_t stream);

// sums[c, k] *= factor * (mask && 1 <= k <= F-2 ? 2 : 1); complex sums are
// interleaved double pairs.
cudaError_t scale_sums(double *sums, int64_t C, int64_t F, bool complex_sums,
                       double factor, bool mask, cudaStream_t stream);

} // namespace ib200

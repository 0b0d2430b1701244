// frontend.h — host planner of the B200 spectral backend (C++ side of the
// C ABI in include/insight_b200.h).
#pragma once
#include "insight_b200.h"

#include <cuda_runtime.h>
#include <cstdint>
#include <string>
#include <vector>

namespace ib200 {

// One spectral call, with the reference frontend's arguments.
struct Call {
  int op = INSIGHT_B200_OP_WELCH;
  const InsightArray *x = nullptr;
  const InsightArray *y = nullptr;
  InsightArray *out = nullptr; // Pxx / Pxy / Sxx / Zxx
  InsightArray *f = nullptr;   // optional
  InsightArray *t = nullptr;   // optional
  int axis = -1;
  double fs = 1.0;
  std::string window = "hann";
  const std::vector<double> *window_values = nullptr; // registry kernels
  int64_t nperseg = 256, noverlap = 0, nfft = 0;
  bool detrend_constant = true;
  bool detrend_linear = false; // least-squares line removal (native option)
  bool onesided = true;
  std::string scaling = "density";
  std::string mode = "psd";
  bool has_scale = false; // registry kernels pass the frontend's scale
  double scale = 1.0;
  int64_t seg_begin = 0, seg_end = 0;
  bool raw_sums = false;
  int64_t avg_segments = 0; // welch/csd: averaging count (0 -> the call's own)
  int32_t x_dtype = 0;    // finalize_sums only
  int default_device = 0; // device for CPU inputs
  cudaStream_t stream = nullptr;
  bool sync = true;
};

// One inverse STFT (reference ins::signal::istft), see spectral_istft.cuh.
struct IstftCall {
  const InsightArray *z = nullptr; // complex [F, S] or [C, F, S]
  InsightArray *out = nullptr;     // F64 [n_total] or [C, n_total]
  std::string window = "hann";
  const std::vector<double> *window_values = nullptr; // registry kernel
  int64_t nperseg = 0, noverlap = 0, nfft = 0;       // 0 -> reference defaults
  int default_device = 0;
  cudaStream_t stream = nullptr;
  bool sync = true;
};

C_Status run(const Call &c);
C_Status run_istft(const IstftCall &c);
C_Status istft_shape(const IstftCall &c, int64_t *n_channels, int64_t *n_total);
C_Status shape(const Call &c, int64_t *n_channels, int64_t *n_seg,
               int64_t *n_freq);
C_Status finalize_sums(const Call &c, int64_t S_total, InsightArray *sums);

// One call (GPU arrays only) captured into a CUDA graph; executing the plan
// replays the call's kernels on the arrays it was made with.
C_Status plan_create(const Call &c, void **plan);
C_Status plan_execute(void *plan, cudaStream_t stream, bool sync);
C_Status plan_destroy(void *plan);

void set_last_error(const std::string &msg);
const char *last_error();
int64_t launch_count();
void add_launches(int64_t n);

} // namespace ib200

// launch.cpp — work split and dtype dispatch of the fused spectral kernels.
#include "launch.h"

#include <algorithm>

namespace ib200 {

bool nfft_supported(int64_t nfft) {
  return nfft >= 16 && nfft <= 8192 && (nfft & (nfft - 1)) == 0;
}

// welch / csd work units: (channel, contiguous range of Qt transforms).  The
// unit count targets 16 units per SM so the grid-stride loop balances, and
// every unit keeps at least 16 transforms so the per-unit partial written to
// scratch (F values) stays a small fraction of the unit's input.
AccSplit acc_split(const LaunchDesc &d, int num_sms, int blocks_per_sm) {
  AccSplit s{};
  s.Tc = tasks_per_channel(d);
  const int64_t total = d.C * s.Tc;
  const int64_t target = (int64_t)std::max(num_sms, 1) * 16;
  int64_t q0 = (total + target - 1) / target;
  q0 = std::max<int64_t>(q0, std::min<int64_t>(s.Tc, 16));
  q0 = std::max<int64_t>(q0, 1);
  s.nq = (s.Tc + q0 - 1) / q0;
  if (d.max_units > 0 && d.C * s.nq > d.max_units)
    s.nq = std::max<int64_t>(1, d.max_units / std::max<int64_t>(d.C, 1));
  s.Qt = (s.Tc + s.nq - 1) / s.nq;
  s.U = d.C * s.nq;
  const int64_t gmax = (int64_t)std::max(num_sms, 1) * std::max(blocks_per_sm, 1);
  s.grid = (int)std::max<int64_t>(1, std::min<int64_t>(s.U, gmax));
  return s;
}

size_t scratch_bytes(const LaunchDesc &d, int num_sms) {
  if (d.kind == LK_STORE)
    return 0;
  AccSplit s = acc_split(d, num_sms, 1);
  const size_t per = d.kind == LK_COH ? 32 : (d.kind == LK_CSD ? 16 : 8);
  // unit split (generic kernel) or flat split (fast kernel), whichever needs more
  const int64_t T_all = d.C * s.Tc;
  int64_t flat = std::min<int64_t>(T_all, (int64_t)std::max(num_sms, 1) *
                                              kFlatMaxBlocksPerSm) +
                 d.C - 1;
  if (d.max_units > 0)
    flat = std::min<int64_t>(flat, d.max_units);
  const int64_t slots = std::max<int64_t>(s.U, flat);
  return (size_t)slots * (size_t)(d.nfft / 2 + 1) * per;
}

cudaError_t launch(const LaunchDesc &d, void *scratch, int num_sms,
                   cudaStream_t stream, int64_t *launches) {
  if (!nfft_supported(d.nfft))
    return cudaErrorInvalidValue;
  return d.f64 ? launch_f64(d, scratch, num_sms, stream, launches)
               : launch_f32(d, scratch, num_sms, stream, launches);
}

} // namespace ib200

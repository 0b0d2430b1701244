// spectral_dispatch.cuh — instantiation of the fused kernels for one compute
// dtype and every supported transform length, plus their launch logic.
#pragma once
#include "launch.h"
#include "spectral_kernels.cuh"

#include <algorithm>

namespace ib200 {

// Values per thread: 16 (f32) / 8 (f64) for long transforms; short
// transforms keep at least 32 threads per group where possible.
template <typename T> __host__ __device__ constexpr int values_per_thread(int L) {
  const int big = std::is_same<T, float>::value ? 16 : 8;
  const int minE = 2;
  int e = L / 32;
  if (e > big)
    e = big;
  if (e < minE)
    e = minE;
  return e;
}

// Transform groups per CTA of the store kernel: about 16K (f32) / 8K (f64)
// staged values, at most 8 groups, 1024 threads, and one group when a group
// is smaller than a warp (named barriers count whole warps).
template <typename T> __host__ __device__ constexpr int store_groups(int L) {
  constexpr int budget = std::is_same<T, float>::value ? 16384 : 8192;
  const int E = values_per_thread<T>(L);
  const int P = L / E;
  int g = budget / L;
  if (g > 8)
    g = 8;
  while (g > 1 && g * P > 1024)
    --g;
  if (g < 1 || (P % 32) != 0)
    g = 1;
  return g;
}

template <typename T>
SpecArgs<T> make_args(const LaunchDesc &d, void *scratch) {
  using V = typename V2T<T>::type;
  SpecArgs<T> a{};
  a.x = reinterpret_cast<const T *>(d.x);
  a.y = reinterpret_cast<const T *>(d.y ? d.y : d.x);
  a.x_cs = d.x_cs;
  a.x_ss = d.x_ss;
  a.y_cs = d.y ? d.y_cs : d.x_cs;
  a.y_ss = d.y ? d.y_ss : d.x_ss;
  a.C = d.C;
  a.nperseg = d.nperseg;
  a.step = d.step;
  a.seg0 = d.seg0;
  a.S = d.S;
  a.win = reinterpret_cast<const T *>(d.win);
  a.tw = reinterpret_cast<const V *>(d.tw);
  a.dtab = reinterpret_cast<const V *>(d.dtab);
  a.dc_mode = d.dc_mode;
  a.Tc = (d.kind == LK_CSD) ? d.S : (d.S + 1) / 2;
  a.scratch = reinterpret_cast<double *>(scratch);
  a.F = d.F;
  a.out = d.out;
  a.o_cs = d.o_cs;
  a.o_rs = d.o_rs;
  a.o_ts = d.o_ts;
  a.out_kind = d.out_kind;
  a.psd_scale = d.psd_scale;
  a.onesided_mask = d.onesided_mask ? 1 : 0;
  return a;
}

template <typename T, int L, int MODE>
cudaError_t run_accum(const LaunchDesc &d, void *scratch, int num_sms,
                      cudaStream_t stream, int64_t *launches) {
  using V = typename V2T<T>::type;
  constexpr int E = values_per_thread<T>(L);
  constexpr int P = L / E;
  auto kern = spectral_accum_kernel<T, L, E, MODE>;
  const size_t smem = sizeof(V) * spad_size(L);
  static int blocks_per_sm = -1; // per instantiation; same on every B200
  if (blocks_per_sm < 0) {
    cudaError_t e = cudaFuncSetAttribute(
        kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess)
      return e;
    int nb = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, kern, P, smem);
    if (e != cudaSuccess)
      return e;
    blocks_per_sm = std::max(nb, 1);
  }
  SpecArgs<T> a = make_args<T>(d, scratch);
  AccSplit sp = acc_split(d, num_sms, blocks_per_sm);
  a.nq = sp.nq;
  a.Qt = sp.Qt;
  a.U = sp.U;
  kern<<<sp.grid, P, smem, stream>>>(a);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess)
    return e;
  const int64_t n = d.C * d.F;
  const int threads = 256;
  const int64_t blocks = (n + threads - 1) / threads;
  spectral_finalize_kernel<MODE><<<(unsigned)blocks, threads, 0, stream>>>(
      a.scratch, d.C, sp.nq, d.nfft, d.F, d.avg_scale, d.onesided_mask ? 1 : 0,
      d.out, d.o_cs, d.out_kind);
  if (launches)
    *launches += 2;
  return cudaGetLastError();
}

template <typename T, int L>
cudaError_t run_store(const LaunchDesc &d, int num_sms, cudaStream_t stream,
                      int64_t *launches) {
  using V = typename V2T<T>::type;
  constexpr int E = values_per_thread<T>(L);
  constexpr int P = L / E;
  constexpr int G = store_groups<T>(L);
  auto kern = spectral_store_kernel<T, L, E, G>;
  const size_t smem = sizeof(V) * (size_t)G * (spad_size(L) + 2);
  static int blocks_per_sm = -1;
  if (blocks_per_sm < 0) {
    cudaError_t e = cudaFuncSetAttribute(
        kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess)
      return e;
    int nb = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, kern, G * P, smem);
    if (e != cudaSuccess)
      return e;
    blocks_per_sm = std::max(nb, 1);
  }
  SpecArgs<T> a = make_args<T>(d, nullptr);
  const int64_t tiles = d.C * ((a.Tc + G - 1) / G);
  const int64_t grid =
      std::max<int64_t>(1, std::min<int64_t>(tiles, (int64_t)num_sms * blocks_per_sm));
  kern<<<(unsigned)grid, G * P, smem, stream>>>(a);
  if (launches)
    *launches += 1;
  return cudaGetLastError();
}

template <typename T, int L>
cudaError_t run_len(const LaunchDesc &d, void *scratch, int num_sms,
                    cudaStream_t stream, int64_t *launches) {
  switch (d.kind) {
  case LK_PSD:
    return run_accum<T, L, ACC_PSD>(d, scratch, num_sms, stream, launches);
  case LK_CSD:
    return run_accum<T, L, ACC_CSD>(d, scratch, num_sms, stream, launches);
  default:
    return run_store<T, L>(d, num_sms, stream, launches);
  }
}

template <typename T>
cudaError_t launch_t(const LaunchDesc &d, void *scratch, int num_sms,
                     cudaStream_t stream, int64_t *launches) {
  switch (d.nfft) {
  case 16: return run_len<T, 16>(d, scratch, num_sms, stream, launches);
  case 32: return run_len<T, 32>(d, scratch, num_sms, stream, launches);
  case 64: return run_len<T, 64>(d, scratch, num_sms, stream, launches);
  case 128: return run_len<T, 128>(d, scratch, num_sms, stream, launches);
  case 256: return run_len<T, 256>(d, scratch, num_sms, stream, launches);
  case 512: return run_len<T, 512>(d, scratch, num_sms, stream, launches);
  case 1024: return run_len<T, 1024>(d, scratch, num_sms, stream, launches);
  case 2048: return run_len<T, 2048>(d, scratch, num_sms, stream, launches);
  case 4096: return run_len<T, 4096>(d, scratch, num_sms, stream, launches);
  case 8192: return run_len<T, 8192>(d, scratch, num_sms, stream, launches);
  default: return cudaErrorInvalidValue;
  }
}

} // namespace ib200

// spectral_dispatch.cuh — instantiation of the fused kernels for one compute
// dtype and every supported transform length, plus their launch logic.
#pragma once
#include "launch.h"
#include "spectral_kernels.cuh"
#include "spectral_accum_fast.cuh"
#include "spectral_stft_ws.cuh"
#include "spectral_stft_tma.cuh"

#include <cudaTypedefs.h>
#include <algorithm>
#include <type_traits>

namespace ib200 {


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

// Shared-memory budget of one CTA of the STFT fast path.
#ifndef IB200_STFT_SMEM_BUDGET
#define IB200_STFT_SMEM_BUDGET 225280
#endif

// Fast-path shape: G transform groups per CTA, M interleaved transforms per
// thread, and whether the per-thread twiddle rows fit in shared memory.  The
// preferred shape is IB200_STFT_PAIRS segment pairs per tile (8 pairs give
// 16-segment, 128-byte complex64 runs per bin row) with IB200_STFT_INTERLEAVE
// transforms per thread.
template <typename T> struct FastShape {
  int G, M;
  bool tws;
};

#ifndef IB200_STFT_PAIRS
#define IB200_STFT_PAIRS 8
#endif
#ifndef IB200_STFT_INTERLEAVE
#define IB200_STFT_INTERLEAVE 1
#endif

template <typename T, int L>
constexpr size_t fast_smem_bytes(int G, int M, bool tws) {
  constexpr int E = values_per_thread<T>(L);
  constexpr int P = L / E;
  constexpr int SEC = 32 / (2 * (int)sizeof(T));
  size_t b = (size_t)G * M * (spad_size(L) + 2) * 2 * sizeof(T) +
             (size_t)P * (E + 16 / sizeof(T)) * sizeof(T) +
             ((size_t)(L / 2 + 1) * (SEC - 1) * 2 * sizeof(T) + 15) / 16 * 16;
  if (tws)
    b += (size_t)P * ThreadTw<T, L, E>::stride() * 2 * sizeof(T);
  return b;
}

template <typename T, int L> constexpr FastShape<T> fast_shape_any() {
  constexpr int E = values_per_thread<T>(L);
  constexpr int P = L / E;
  if (P % 32 != 0)
    return {0, 0, false};
  // interleaved: Q pairs as Q/M groups of M transforms, twiddle rows required
  for (int q = IB200_STFT_PAIRS; q >= 4; q /= 2) {
    const int m = IB200_STFT_INTERLEAVE;
    const int g = q / m;
    if (g >= 1 && g * P <= 1024 && (g * P) / (2 * q) >= 16 &&
        ((g * P) / (2 * q)) % 16 == 0 &&
        fast_smem_bytes<T, L>(g, m, true) <= IB200_STFT_SMEM_BUDGET)
      return {g, m, true};
  }
  // one transform per thread
  for (int pass = 0; pass < 2; ++pass) {
    const bool tws = pass == 0;
    int g = 8;
    while (g > 1 && (fast_smem_bytes<T, L>(g, 1, tws) > IB200_STFT_SMEM_BUDGET ||
                     g * P > 1024))
      g /= 2;
    if (fast_smem_bytes<T, L>(g, 1, tws) <= IB200_STFT_SMEM_BUDGET &&
        (g >= 4 || !tws) && P / 2 >= 16)
      return {g, 1, tws};
  }
  return {0, 0, false};
}

// The sector-aligned store needs tile rows of whole 32-byte sectors.
template <typename T, int L> constexpr FastShape<T> fast_shape() {
  constexpr FastShape<T> s = fast_shape_any<T, L>();
  constexpr int sec = 32 / (2 * (int)sizeof(T));
  if (s.G == 0 || 2 * s.G * s.M < sec || (2 * s.G * s.M) % sec != 0)
    return {0, 0, false};
  return s;
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
  a.Tc = tasks_per_channel(d);
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
  const size_t smem =
      sizeof(V) * spad_size(L) * (MODE != ACC_PSD && !packs_xy<T, L>() ? 2 : 1);
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
  e = launch_finalize<MODE>(a.scratch, d.C, sp.nq, 0, d.nfft, d.F, d.avg_scale,
                            d.onesided_mask ? 1 : 0, d.out, d.o_cs, d.out_kind,
                            stream);
  if (launches)
    *launches += 2;
  return e;
}

// Overlap shift of the fast path: hop = SH * L/R0 with SH in {R0/4, R0/2}
// (75% / 50% overlap) reuses registers; other hops load both segments.
template <typename T, int L> int fast_shift(int64_t step) {
  constexpr int E = values_per_thread<T>(L);
  constexpr int R0 = Plan<L, E>::radix(0);
  constexpr int Q = L / R0;
  if (step % Q != 0)
    return 0;
  const int64_t sh = step / Q;
  if (R0 >= 4 && sh == R0 / 4)
    return R0 / 4;
  if (R0 >= 2 && sh == R0 / 2)
    return R0 / 2;
  return 0;
}

template <typename T, int L, int SH>
cudaError_t run_stft_fast_sh(const LaunchDesc &d, int num_sms,
                             cudaStream_t stream, int64_t *launches) {
  constexpr int E = values_per_thread<T>(L);
  constexpr int P = L / E;
  constexpr FastShape<T> FS = fast_shape<T, L>();
  constexpr int G = FS.G;
  constexpr int M = FS.M;
  auto kern = stft_fast_kernel<T, L, E, G, M, SH, FS.tws>;
  const size_t smem = fast_smem_bytes<T, L>(G, M, FS.tws);
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
  // Units of nsub consecutive tiles per CTA: long enough that the partial
  // sectors at unit ends are a few percent of the writes, short enough for
  // about eight units per resident CTA.
  const int64_t tpc = (a.Tc + G * M - 1) / (G * M);
  const int64_t ctas = (int64_t)num_sms * blocks_per_sm;
  int nsub = (int)std::max<int64_t>(
      1, std::min<int64_t>(16, (d.C * tpc) / std::max<int64_t>(1, 8 * ctas)));
  const int64_t units = d.C * ((tpc + nsub - 1) / nsub);
  const int64_t grid = std::max<int64_t>(1, std::min<int64_t>(units, ctas));
  kern<<<(unsigned)grid, G * P, smem, stream>>>(a, nsub);
  if (launches)
    *launches += 1;
  return cudaGetLastError();
}

// Warp-specialised variant (spectral_stft_ws.cuh) where its shape fits.
#ifndef IB200_STFT_WS
#define IB200_STFT_WS 1
#endif
#ifndef IB200_STFT_WS_TWM
#define IB200_STFT_WS_TWM 1
#endif
// 0: not usable; else 1 + the twiddle mode of the warp-specialised kernel
// (IB200_STFT_WS_TWM or less, whichever fits the shared-memory budget)
template <typename T, int L> constexpr int stft_ws_mode() {
  using SS = StftWsShape<T, L>;
  if constexpr (!IB200_STFT_WS || !SS::ok) {
    return 0;
  } else {
    for (int twm = IB200_STFT_WS_TWM; twm >= 0; --twm)
      if (SS::smem(twm) <= IB200_STFT_SMEM_BUDGET)
        return 1 + twm;
    return 0;
  }
}

template <typename T, int L, int SH>
cudaError_t run_stft_ws_sh(const LaunchDesc &d, int num_sms, cudaStream_t stream,
                           int64_t *launches) {
  using SS = StftWsShape<T, L>;
  constexpr int TWM = stft_ws_mode<T, L>() - 1;
  auto kern = stft_ws_kernel<T, L, SH, TWM>;
  const size_t smem = SS::smem(TWM);
  static bool attr = false;
  if (!attr) {
    cudaError_t e = cudaFuncSetAttribute(
        kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess)
      return e;
    attr = true;
  }
  SpecArgs<T> a = make_args<T>(d, nullptr);
  // units of nsub consecutive tiles per CTA (one CTA per SM), as in
  // run_stft_fast_sh
  const int64_t tpc = (a.Tc + SS::Q - 1) / SS::Q;
  const int64_t ctas = num_sms;
  int nsub = (int)std::max<int64_t>(
      1, std::min<int64_t>(32, (d.C * tpc) / std::max<int64_t>(1, 8 * ctas)));
  const int64_t units = d.C * ((tpc + nsub - 1) / nsub);
  const int64_t grid = std::max<int64_t>(1, std::min<int64_t>(units, ctas));
  kern<<<(unsigned)grid, SS::NT, smem, stream>>>(a, nsub);
  if (launches)
    *launches += 1;
  return cudaGetLastError();
}

// TMA-store variant (spectral_stft_tma.cuh): f32, nperseg = nfft = 2048,
// contiguous bin rows, 32-byte-aligned output.
#ifndef IB200_STFT_TMA
#define IB200_STFT_TMA 1
#endif

// cuTensorMapEncodeTiled from the driver, looked up once per process.
inline PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static const PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
    void *ptr = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault,
                                &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      ptr = nullptr;
    return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }();
  return fn;
}

inline bool stft_tma_eligible(const LaunchDesc &d) {
  return IB200_STFT_TMA && !d.f64 && d.nfft == StftTma::L && d.S >= 1 &&
         d.C >= 1 && d.o_ts == 1 && d.o_rs >= d.S &&
         d.o_cs == StftTma::F * d.o_rs &&
         (reinterpret_cast<uintptr_t>(d.out) & 31) == 0 &&
         d.C * StftTma::F / 4 + StftTma::ROWS < (int64_t(1) << 31) &&
         2 * (d.S + 4) < (int64_t(1) << 31) &&
         d.C * ((d.S + 1) / 2 / StftTma::Q + 1) < (int64_t(1) << 31) &&
         32 * d.o_rs < (int64_t(1) << 40) && tensor_map_encoder() != nullptr;
}

// Tensor map of the rows R = c*F + k with R mod 4 == m: their sector-aligned
// origin (d_m = (m * o_rs) mod 4 elements before row m's first column), a
// stride of 4 rows, S + d_m complex columns as 2 (S + d_m) floats, boxes of
// 8 columns x 256 rows with the 64-byte swizzle.
inline cudaError_t encode_stft_map(CUtensorMap *tm, const LaunchDesc &d, int m) {
  const int64_t dm = (m * (d.o_rs & 3)) & 3;
  float2 *base = reinterpret_cast<float2 *>(d.out) + (m * d.o_rs - dm);
  const cuuint64_t dims[2] = {(cuuint64_t)(2 * (d.S + dm)),
                              (cuuint64_t)((d.C * StftTma::F - m + 3) / 4)};
  const cuuint64_t strides[1] = {(cuuint64_t)(32 * d.o_rs)};
  const cuuint32_t box[2] = {2 * StftTma::W, StftTma::ROWS};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = tensor_map_encoder()(
      tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, base, dims, strides, box, estr,
      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B,
      CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

template <int SH>
cudaError_t run_stft_tma_sh(const LaunchDesc &d, int num_sms, cudaStream_t stream,
                            int64_t *launches) {
  using K = StftTma;
  auto kern = stft_tma_kernel<SH>;
  static const cudaError_t attr = cudaFuncSetAttribute(
      kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)K::SMEM);
  if (attr != cudaSuccess)
    return attr;
  StftTmaArgs a{};
  a.x = reinterpret_cast<const float *>(d.x);
  a.x_cs = d.x_cs;
  a.step = d.step;
  a.seg0 = d.seg0;
  a.S = (int)d.S;
  a.tpc = (int)(((d.S + 1) / 2 + K::Q - 1) / K::Q);
  a.ntiles = (int)(d.C * a.tpc);
  a.win = reinterpret_cast<const float *>(d.win);
  a.tw = reinterpret_cast<const float2 *>(d.tw);
  a.out = reinterpret_cast<float2 *>(d.out);
  a.o_cs = d.o_cs;
  a.o_rs = d.o_rs;
  a.dc_mode = d.dc_mode;
  CUtensorMap tm[4];
  for (int m = 0; m < 4; ++m) {
    cudaError_t e = encode_stft_map(&tm[m], d, m);
    if (e != cudaSuccess)
      return e;
  }
  const int64_t grid = std::max<int64_t>(1, std::min<int64_t>(a.ntiles, num_sms));
  kern<<<(unsigned)grid, K::NT, K::SMEM, stream>>>(a, tm[0], tm[1], tm[2], tm[3]);
  if (launches)
    *launches += 1;
  return cudaGetLastError();
}

inline cudaError_t run_stft_tma(const LaunchDesc &d, int num_sms,
                                cudaStream_t stream, int64_t *launches) {
  const int sh = fast_shift<float, StftTma::L>(d.step);
  if (sh == 4)
    return run_stft_tma_sh<4>(d, num_sms, stream, launches);
  if (sh == 8)
    return run_stft_tma_sh<8>(d, num_sms, stream, launches);
  return run_stft_tma_sh<0>(d, num_sms, stream, launches);
}

template <typename T, int L>
cudaError_t run_stft_fast(const LaunchDesc &d, int num_sms, cudaStream_t stream,
                          int64_t *launches) {
  if constexpr (std::is_same<T, float>::value && L == StftTma::L) {
    if (stft_tma_eligible(d))
      return run_stft_tma(d, num_sms, stream, launches);
  }
  if constexpr (stft_ws_mode<T, L>() > 0) {
    constexpr int E = values_per_thread<T>(L);
    constexpr int R0 = Plan<L, E>::radix(0);
    const int sh = fast_shift<T, L>(d.step);
    if constexpr (R0 >= 4) {
      if (sh == R0 / 4)
        return run_stft_ws_sh<T, L, R0 / 4>(d, num_sms, stream, launches);
    }
    if constexpr (R0 >= 2) {
      if (sh == R0 / 2)
        return run_stft_ws_sh<T, L, R0 / 2>(d, num_sms, stream, launches);
    }
    return run_stft_ws_sh<T, L, 0>(d, num_sms, stream, launches);
  }
  constexpr int E = values_per_thread<T>(L);
  constexpr int R0 = Plan<L, E>::radix(0);
  const int sh = fast_shift<T, L>(d.step);
  if constexpr (R0 >= 4) {
    if (sh == R0 / 4)
      return run_stft_fast_sh<T, L, R0 / 4>(d, num_sms, stream, launches);
  }
  if constexpr (R0 >= 2) {
    if (sh == R0 / 2)
      return run_stft_fast_sh<T, L, R0 / 2>(d, num_sms, stream, launches);
  }
  return run_stft_fast_sh<T, L, 0>(d, num_sms, stream, launches);
}

template <typename T, int L>
cudaError_t run_store(const LaunchDesc &d, int num_sms, cudaStream_t stream,
                      int64_t *launches) {
  using V = typename V2T<T>::type;
  constexpr int EE = values_per_thread<T>(L);
  if constexpr (fast_shape<T, L>().G > 0 && Plan<L, EE>::passes() >= 2) {
    const bool want = std::is_same<T, float>::value ? d.out_kind == OUT_C64_K
                                                    : d.out_kind == OUT_C128_K;
    if (want && d.x_ss == 1 && d.nperseg == d.nfft && d.dc_mode <= 1 &&
        d.o_ts == 1 && d.F == d.nfft / 2 + 1)
      return run_stft_fast<T, L>(d, num_sms, stream, launches);
  }
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

// welch / csd fast path shape: G transform groups (at most 512 threads, a
// 128-register budget for the f64 accumulators) and whether the per-thread
// twiddle rows fit next to the transform buffers.
struct AccShape {
  int G;
  int twm; // 0 global twiddle table, 1 first-twiddle rows, 2 full rows
};

template <typename T, int L>
constexpr size_t acc_fast_smem(int G, int twm, bool stg, int mode) {
  constexpr int E = values_per_thread<T>(L);
  constexpr int P = L / E;
  constexpr int GS = (spad_size(L) + 1) / 2 * 2;
  const int nbuf = mode == ACC_PSD ? 1 : 2; // csd, coherence: x and y spectra
  size_t b = (size_t)G * nbuf * GS * 2 * sizeof(T) +
             (size_t)P * (E + 16 / sizeof(T)) * sizeof(T);
  if (stg)
    b += (size_t)G * nbuf * 2 * L * sizeof(T);
  if (twm == 2)
    b += (size_t)P * ThreadTw<T, L, E>::stride() * 2 * sizeof(T);
  else if (twm == 1)
    b += (size_t)P * ThreadTw1<T, L, E>::stride() * 2 * sizeof(T);
  if (acc_prefetch<T, L, E>(mode, twm, stg)) // f64 totals, 2 (E/2 + 1) a thread
    b += (size_t)G * P * 2 * (E / 2 + 1) * sizeof(double);
  if (acc_prefetch_psd<T, L, E>(mode, twm, stg)) // f64 totals, E a thread
    b += (size_t)G * P * E * sizeof(double);
  return b;
}

// MAXT: threads per CTA (coherence keeps three accumulators per bin and uses
// at most 256 threads, i.e. up to 255 registers each).  csd and coherence
// are never shaped for f64 L = 8192 (two spectra do not fit; see packs_xy).
#ifndef IB200_ACC_TWM
#define IB200_ACC_TWM 2
#endif
template <typename T, int L, bool STG, int MODE>
constexpr AccShape acc_fast_shape() {
  constexpr int MAXT = MODE == ACC_COH ? 256 : 512;
  constexpr int E = values_per_thread<T>(L);
  constexpr int P = L / E;
  // the prefetching csd shape holds its f64 totals in shared memory too
  constexpr size_t budget =
      acc_prefetch<T, L, E>(MODE, 1, STG) ? 227 * 1024 : 220 * 1024;
  int g = 8;
  while (g > 1 && g * P > MAXT)
    --g;
  if (P % 32 != 0)
    g = 1;
  while (g > 1 && (g & (g - 1)) != 0)
    --g;
  // csd / coherence: first-twiddle rows, for the mirrored last pass
  constexpr int TW0 =
      acc_mirrored<T, L, E>(MODE, 1) ? 1 : IB200_ACC_TWM;
  for (; g >= 1; g /= 2)
    for (int twm = TW0; twm >= 0; --twm)
      if (acc_fast_smem<T, L>(g, twm, STG, MODE) <= budget)
        return {g, twm};
  return {0, 0};
}

// Resident CTAs per SM of one fast accumulate instantiation (sets its
// dynamic shared-memory limit on first use; 0 on error).
template <typename T, int L, int MODE, int SH, bool STG>
int acc_fast_blocks_per_sm() {
  constexpr int E = values_per_thread<T>(L);
  constexpr int P = L / E;
  constexpr AccShape AS = acc_fast_shape<T, L, STG, MODE>();
  auto kern = accum_fast_kernel<T, L, E, AS.G, SH, AS.twm, MODE, STG>;
  const size_t smem = acc_fast_smem<T, L>(AS.G, AS.twm, STG, MODE);
  static int blocks_per_sm = -1;
  if (blocks_per_sm < 0) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)smem) != cudaSuccess)
      return 0;
    int nb = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, kern, AS.G * P,
                                                      smem) != cudaSuccess)
      return 0;
    blocks_per_sm = std::max(nb, 1);
  }
  return blocks_per_sm;
}

template <typename T, int L, int MODE, int SH, bool STG>
cudaError_t run_accum_fast_sh(const LaunchDesc &d, void *scratch, int num_sms,
                              cudaStream_t stream, int64_t *launches) {
  constexpr int E = values_per_thread<T>(L);
  constexpr int P = L / E;
  constexpr AccShape AS = acc_fast_shape<T, L, STG, MODE>();
  constexpr int G = AS.G;
  auto kern = accum_fast_kernel<T, L, E, G, SH, AS.twm, MODE, STG>;
  const size_t smem = acc_fast_smem<T, L>(G, AS.twm, STG, MODE);
  const int blocks_per_sm = acc_fast_blocks_per_sm<T, L, MODE, SH, STG>();
  if (blocks_per_sm == 0)
    return cudaGetLastError() != cudaSuccess ? cudaErrorInvalidValue
                                             : cudaErrorInvalidConfiguration;
  SpecArgs<T> a = make_args<T>(d, scratch);
  // Flat split: one CTA per resident slot, each with the same number of
  // transforms (to within one); CTA b's partial of channel c is slot b + c.
  const int64_t T_all = d.C * a.Tc;
  int64_t grid = std::min<int64_t>(
      T_all, (int64_t)num_sms * std::min(blocks_per_sm, kFlatMaxBlocksPerSm));
  // small problems: at least G transforms a CTA, so no transform group idles
  // and the finalize reads fewer partial slots
  grid = std::min<int64_t>(grid, std::max<int64_t>(1, T_all / G));
  if (d.max_units > 0) {
    if (d.max_units < d.C)
      return cudaErrorInvalidValue;
    grid = std::min<int64_t>(grid, d.max_units - d.C + 1);
  }
  grid = std::max<int64_t>(grid, 1);
  kern<<<(unsigned)grid, G * P, smem, stream>>>(a);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess)
    return e;
  e = launch_finalize<MODE>(a.scratch, d.C, grid, T_all, d.nfft, d.F, d.avg_scale,
                            d.onesided_mask ? 1 : 0, d.out, d.o_cs, d.out_kind,
                            stream);
  if (launches)
    *launches += 2;
  return e;
}

// Every segment start 16-byte aligned (the cp.async staging condition).
template <typename T, int MODE>
bool segments_aligned16(const LaunchDesc &d, int L) {
  const int64_t sz = sizeof(T);
  auto al = [](const void *q) {
    return (reinterpret_cast<uintptr_t>(q) & 15u) == 0;
  };
  bool ok = al(d.x) && (d.step * sz) % 16 == 0 && (L * sz) % 16 == 0 &&
            (d.C == 1 || (d.x_cs * sz) % 16 == 0);
  if (MODE != ACC_PSD)
    ok = ok && d.y != nullptr && al(d.y) && (d.C == 1 || (d.y_cs * sz) % 16 == 0);
  return ok;
}

// cp.async staging where the segments are 16-byte aligned and it keeps as
// many resident threads per SM as the unstaged kernel (its buffers can cost
// a CTA per SM, e.g. coherence at 256 threads).
template <typename T, int L, int MODE, int SH>
cudaError_t run_accum_fast_pick(const LaunchDesc &d, void *scratch, int num_sms,
                                cudaStream_t stream, int64_t *launches) {
  constexpr AccShape S0 = acc_fast_shape<T, L, false, MODE>();
  constexpr AccShape S1 = acc_fast_shape<T, L, true, MODE>();
  constexpr int E = values_per_thread<T>(L);
  if constexpr (S0.G > 0 && acc_prefetch_psd<T, L, E>(MODE, S0.twm, false)) {
    // welch with the register prefetch: no staging
    return run_accum_fast_sh<T, L, MODE, SH, false>(d, scratch, num_sms, stream,
                                                    launches);
  } else if constexpr (S1.G > 0 && S1.G >= S0.G) {
    if (segments_aligned16<T, MODE>(d, L)) {
      const int b1 = acc_fast_blocks_per_sm<T, L, MODE, SH, true>();
      const int b0 = acc_fast_blocks_per_sm<T, L, MODE, SH, false>();
      if (b1 > 0 && b1 * S1.G >= b0 * S0.G)
        return run_accum_fast_sh<T, L, MODE, SH, true>(d, scratch, num_sms,
                                                       stream, launches);
    }
  }
  return run_accum_fast_sh<T, L, MODE, SH, false>(d, scratch, num_sms, stream,
                                                  launches);
}

template <typename T, int L, int MODE>
cudaError_t run_accum_any(const LaunchDesc &d, void *scratch, int num_sms,
                          cudaStream_t stream, int64_t *launches) {
  constexpr int E = values_per_thread<T>(L);
  constexpr int R0 = Plan<L, E>::radix(0);
  constexpr AccShape S0 = acc_fast_shape<T, L, false, MODE>();
  if constexpr (S0.G > 0 && !(MODE != ACC_PSD && packs_xy<T, L>())) {
    const bool ok = d.x_ss == 1 && (MODE == ACC_PSD || d.y_ss == 1) &&
                    d.nperseg == d.nfft && d.dc_mode <= 1;
    if (ok) {
      // overlap reuse: hop = SH * L/R0 lets segment b take samples from a
      constexpr int Q = L / R0;
      const int64_t v = d.step % Q == 0 ? d.step / Q : -1;
      if constexpr (R0 >= 4) {
        if (v == R0 / 4)
          return run_accum_fast_pick<T, L, MODE, R0 / 4>(d, scratch, num_sms,
                                                         stream, launches);
      }
      if constexpr (R0 >= 2) {
        if (v == R0 / 2)
          return run_accum_fast_pick<T, L, MODE, R0 / 2>(d, scratch, num_sms,
                                                         stream, launches);
      }
      return run_accum_fast_pick<T, L, MODE, 0>(d, scratch, num_sms, stream,
                                                launches);
    }
  }
  return run_accum<T, L, MODE>(d, scratch, num_sms, stream, launches);
}

template <typename T, int L>
cudaError_t run_len(const LaunchDesc &d, void *scratch, int num_sms,
                    cudaStream_t stream, int64_t *launches) {
  switch (d.kind) {
  case LK_PSD:
    return run_accum_any<T, L, ACC_PSD>(d, scratch, num_sms, stream, launches);
  case LK_CSD:
    return run_accum_any<T, L, ACC_CSD>(d, scratch, num_sms, stream, launches);
  case LK_COH:
    return run_accum_any<T, L, ACC_COH>(d, scratch, num_sms, stream, launches);
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

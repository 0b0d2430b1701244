// spectral_istft.cuh — inverse STFT (overlap-add), reference
// ins::signal::istft (src/ops/signal/spectral_analysis.cpp:340-457).
//
// Per frame the reference rebuilds the full spectrum from the one-sided
// column (bins 1..F-2 mirrored as conjugates) when n_freq == nfft/2 + 1 and
// nfft > 2, takes Re(ifft(full, nfft)) (1/nfft scaling), truncates it to
// nperseg samples and multiplies by the window; the frames are overlap-added
// with hop = nperseg - noverlap and divided by the overlap-added squared
// window wherever that exceeds 1e-10.
//
// istft_frames_kernel: one task per pair of frames a, b (one-sided input):
// the Hermitian spectra A, B (imaginary parts of the DC and Nyquist bins
// dropped, which is what taking the real part does) are packed as Z = A + iB,
// so one complex inverse transform gives both real frames,
// IFFT(Z) = a + i b.  The inverse runs on the forward kernels:
// IFFT(Z) = conj(FFT(conj Z)) / nfft.  Other inputs (n_freq != nfft/2 + 1)
// take one frame per task and Re(IFFT(Z)) of the zero-padded / truncated
// column.  Windowed frames go to a frame buffer [C][S][nperseg] in the
// input's precision (f32 for complex64).  istft_ws_kernel is the same
// computation for frame pairs with unit frame stride, fed by coalesced row
// reads.
// The transforms run in f64 for complex64 input too: the overlap-add divides
// by the summed squared window, which is tiny where the window ends, so an
// f32 transform's rounding would be amplified there far above 1e-5.
// istft_ola_kernel: every output sample sums its frames in frame order and
// divides by the summed squared window (f64, as the reference).
#pragma once
#include "launch.h"
#include "spectral_kernels.cuh"

namespace ib200 {

template <typename T, typename TZ> struct IstftArgs {
  using VZ = typename V2T<TZ>::type;
  using V = typename V2T<T>::type;
  const VZ *z;           // Zxx, element (c, k, i) at z[c*z_cs + k*z_fs + i*z_ts]
  int64_t z_cs, z_fs, z_ts;
  int64_t C, F, S;       // channels, bins, frames
  int64_t nperseg;
  int pack;              // 1: Hermitian frame pairs, 0: one frame per task
  int64_t Tc;            // tasks per channel
  const T *win;          // [nperseg] window in T
  const V *tw;           // [L] W_L^m
  void *frames;          // [C][S][nperseg] of TF (f32 for complex64 input)
};

template <typename T, typename TZ, typename TF, int L, int E, int G>
__global__ void __launch_bounds__(G *(L / E))
    istft_frames_kernel(const IstftArgs<T, TZ> p) {
  using V = typename V2T<T>::type;
  constexpr int P = L / E;
  constexpr int GS = spad_size(L);
  extern __shared__ __align__(16) unsigned char smem_raw[];
  V *buf = reinterpret_cast<V *>(smem_raw) + (threadIdx.x / P) * GS;
  const int g = threadIdx.x / P;
  const int t = threadIdx.x - g * P;
  const int64_t tpc = (p.Tc + G - 1) / G;
  const int64_t ntiles = p.C * tpc;
  const T inv = T(1) / T(L);

  for (int64_t tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
    const int64_t c = tile / tpc;
    const int64_t task = (tile - c * tpc) * G + g;
    if (task >= p.Tc)
      continue; // the whole group idles (no CTA-wide barrier below)
    const int64_t ia = p.pack ? 2 * task : task;
    const bool hasb = p.pack && ia + 1 < p.S;
    const auto *za = p.z + c * p.z_cs + ia * p.z_ts;
    auto ld = [&](int64_t i) -> V {
      const auto q = za[i];
      return V{(T)q.x, (T)q.y};
    };
    V v[E];
    static_for<0, E>([&](auto eIC) {
      constexpr int e = decltype(eIC)::value;
      const int k = in_index<L, E, P>(t, e);
      V zc;
      if (p.pack) {
        const bool mirror = k > L / 2;
        const int kk = mirror ? L - k : k;
        V a = ld(kk * p.z_fs);
        V b = hasb ? ld(kk * p.z_fs + p.z_ts) : V{T(0), T(0)};
        if (kk == 0 || kk == L / 2) {
          a.y = T(0);
          b.y = T(0);
        }
        if (mirror) {
          a.y = -a.y;
          b.y = -b.y;
        }
        zc = {a.x - b.y, -(a.y + b.x)}; // conj(A + iB)
      } else {
        zc = k < p.F ? ld(k * p.z_fs) : V{T(0), T(0)};
        zc.y = -zc.y;
      }
      v[e] = zc;
    });
    fft_group<T, L, E, P, G>(v, buf, t, g, p.tw);
    TF *fa = static_cast<TF *>(p.frames) + (c * p.S + ia) * p.nperseg;
    static_for<0, E>([&](auto eIC) {
      constexpr int e = decltype(eIC)::value;
      const int n = out_bin<L, E, P>(t, e);
      if (n < p.nperseg) {
        const T w = p.win[n];
        fa[n] = (TF)(v[e].x * inv * w);
        if (hasb)
          fa[p.nperseg + n] = (TF)(-v[e].y * inv * w);
      }
    });
  }
}

// Warp-specialised frame kernel for Hermitian frame pairs with unit frame
// stride.  The frames of a tile (Q pairs, 2Q consecutive columns of every
// bin row) are read by NLD loader threads as row runs of 2Q values (64 bytes
// or more) with asynchronous copies (cp.async, no registers held) into one
// of two staging buffers, [pair][bin] with the two frames of a pair side by
// side; GF transform groups take the pairs of a full buffer (PPG each), so
// the loads of tile n+1 are in flight while tile n is transformed.  The
// roles meet at named barriers FULL(b) / EMPTY(b) as in stft_ws_kernel.
template <typename TZ, int L, int E_> struct IstftWsShape {
  static constexpr int E = E_; // f64 transforms, E values per thread
  static constexpr int P = L / E;
  static constexpr int NLD = 64;
  // transform threads: up to 512 at E = 8; at E = 16 (about 128 registers a
  // thread) the whole CTA stays within 512 threads
  static constexpr int NFTMAX = E == 16 ? 512 - NLD : 512;
  static constexpr int GF = (NFTMAX / P < 8 ? NFTMAX / P : 8);
  static constexpr int NFT = GF * P;
  static constexpr int NT = NFT + NLD;
  static constexpr int ZB = 2 * (int)sizeof(TZ); // bytes of one input value
  // pairs per tile: row runs of at least 32 bytes
  static constexpr int GF1 = GF > 0 ? GF : 1;
  static constexpr int PPG =
      2 * GF1 * ZB >= 32 ? 1 : (64 + 2 * GF1 * ZB - 1) / (2 * GF1 * ZB);
  static constexpr int Q = GF * PPG;
  static constexpr int FH = L / 2 + 1;
  // pair stride in (frame a, frame b) entries: = 2 mod 8 keeps the loaders'
  // 8- or 16-byte writes of a row run on distinct banks
  static constexpr int FHS = (FH + 5) / 8 * 8 + 2;
  static constexpr int GS = spad_size(L);
  // per-thread first-twiddle rows of the passes after the first
  static constexpr int TWS = ThreadTw1<double, L, E>::stride();
  static constexpr size_t smem0 = (size_t)GF * GS * 16 +
                                  (size_t)2 * Q * FHS * 2 * ZB +
                                  (size_t)P * TWS * 16;
  // the f64 window in shared memory too where it fits (the opt-in maximum
  // of a CTA is 227 KB), else read through the L1 cache
  static constexpr bool WSM = smem0 + (size_t)L * 8 <= 232448;
  static constexpr size_t smem = smem0 + (WSM ? (size_t)L * 8 : 0);
  static constexpr bool ok = GF >= 2 && P % 32 == 0 && GF + 5 <= 16 &&
                             NLD >= 2 * Q && smem0 <= 225280;
};

template <typename TZ, typename TF, int L, int E_>
__global__ void __launch_bounds__(IstftWsShape<TZ, L, E_>::NT)
    istft_ws_kernel(const IstftArgs<double, TZ> p) {
  using T = double;
  using V = double2;
  using VZ = typename V2T<TZ>::type;
  using SS = IstftWsShape<TZ, L, E_>;
  constexpr int E = SS::E, P = SS::P, GF = SS::GF, NFT = SS::NFT, NT = SS::NT;
  constexpr int NLD = SS::NLD, Q = SS::Q, PPG = SS::PPG, FH = SS::FH;
  constexpr int FHS = SS::FHS, GS = SS::GS;
  constexpr int FULL0 = GF + 1, EMPTY0 = GF + 3;
  static_assert(SS::ok, "shape");
  extern __shared__ __align__(16) unsigned char smem_raw[];
  V *scratch = reinterpret_cast<V *>(smem_raw);                // [GF][GS]
  VZ *stage = reinterpret_cast<VZ *>(scratch + GF * GS);       // [2][Q][FHS][2]
  V *tws = reinterpret_cast<V *>(stage + 2 * Q * FHS * 2);     // [P][TWS]
  T *wsm = reinterpret_cast<T *>(tws + P * SS::TWS);            // [nperseg]
  fill_thread_w1<T, L, E, P>(tws, p.tw, threadIdx.x, NT);
  if constexpr (SS::WSM)
    fill_batched<8>(
        threadIdx.x, (int)p.nperseg, NT, [&](int i) { return p.win[i]; },
        [&](int i, T v) { wsm[i] = v; });
  __syncthreads();
  const int64_t tpc = (p.Tc + Q - 1) / Q;
  const int64_t ntiles = p.C * tpc;
  const int64_t mine = ntiles > blockIdx.x
                           ? (ntiles - blockIdx.x + gridDim.x - 1) / gridDim.x
                           : 0; // tiles of this CTA

  if (threadIdx.x >= NFT) {
    // ---------------------------------------------------------------- loads
    constexpr int CPR = 2 * Q;         // columns per row run
    constexpr int RPW = NLD / CPR;     // rows per loader round
    const int lt = threadIdx.x - NFT;
    const int col = lt % CPR;
    const int kr0 = lt / CPR;
    const int kend = lt < RPW * CPR ? FH : 0; // spare loader threads copy nothing
    for (int64_t n = 0; n < mine; ++n) {
      const int64_t tile = blockIdx.x + n * gridDim.x;
      const int b = (int)(n & 1);
      const int64_t c = tile / tpc;
      const int64_t f = (tile - c * tpc) * (2 * Q) + col; // frame of this column
      const bool valid = f < p.S;
      const VZ *src = p.z + c * p.z_cs + (valid ? f : 0);
      VZ *dst = stage + ((size_t)(b * Q + (col >> 1)) * FHS) * 2 + (col & 1);
      if (n >= 2)
        named_sync(EMPTY0 + b, NT); // the transforms released buffer b
      for (int k = kr0; k < kend; k += RPW) {
        const unsigned d =
            static_cast<unsigned>(__cvta_generic_to_shared(dst + 2 * k));
        const VZ *sk = src + k * p.z_fs;
        if constexpr (sizeof(VZ) == 16)
          asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(d),
                       "l"(sk), "r"(valid ? 16 : 0)
                       : "memory");
        else
          asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;\n" ::"r"(d),
                       "l"(sk), "r"(valid ? 8 : 0)
                       : "memory");
      }
      cp_async_commit();
      if (n >= 1) {
        asm volatile("cp.async.wait_group 1;\n" ::: "memory");
        named_arrive(FULL0 + (b ^ 1), NT); // tile n-1 has landed
      }
    }
    if (mine >= 1) {
      cp_async_wait_all();
      named_arrive(FULL0 + (int)((mine - 1) & 1), NT);
    }
    // wait for the last releases so every barrier phase completes
    for (int64_t k = mine >= 2 ? mine - 2 : 0; k < mine; ++k)
      named_sync(EMPTY0 + (int)(k & 1), NT);
    return;
  }

  // ------------------------------------------------------------ transforms
  const int g = threadIdx.x / P;
  const int t = threadIdx.x - g * P;
  V *buf = scratch + g * GS;
  const T inv = T(1) / T(L);
  for (int64_t n = 0; n < mine; ++n) {
    const int64_t tile = blockIdx.x + n * gridDim.x;
    const int b = (int)(n & 1);
    const int64_t c = tile / tpc;
    named_sync(FULL0 + b, NT); // the loaders filled buffer b
#pragma unroll 1
    for (int pp = 0; pp < PPG; ++pp) {
      const int q = g * PPG + pp;
      const int64_t task = (tile - c * tpc) * Q + q;
      const bool act = task < p.Tc; // uniform over the group
      const int64_t ia = 2 * task;
      const bool hasb = ia + 1 < p.S;
      V v[E];
      if (act) {
        const VZ *ent = stage + ((size_t)(b * Q + q) * FHS) * 2;
        static_for<0, E>([&](auto eIC) {
          constexpr int e = decltype(eIC)::value;
          const int k = in_index<L, E, P>(t, e);
          const bool mirror = k > L / 2;
          const int kk = mirror ? L - k : k;
          const VZ za = ent[2 * kk], zb = ent[2 * kk + 1];
          V a{(T)za.x, (T)za.y}, bb{(T)zb.x, (T)zb.y};
          if (kk == 0 || kk == L / 2) {
            a.y = T(0);
            bb.y = T(0);
          }
          if (mirror) {
            a.y = -a.y;
            bb.y = -bb.y;
          }
          v[e] = V{a.x - bb.y, -(a.y + bb.x)}; // conj(A + iB)
        });
      }
      if (pp == PPG - 1)
        named_arrive(EMPTY0 + b, NT); // this thread is done with buffer b
      if (act) {
        fft_group_w1<T, L, E, P, GF>(v, buf, t, g, tws + t * SS::TWS);
        TF *fa = static_cast<TF *>(p.frames) + (c * p.S + ia) * p.nperseg;
        static_for<0, E>([&](auto eIC) {
          constexpr int e = decltype(eIC)::value;
          const int nn = out_bin<L, E, P>(t, e);
          if (nn < p.nperseg) {
            const T w = SS::WSM ? wsm[nn] : __ldg(p.win + nn);
            fa[nn] = (TF)(v[e].x * inv * w);
            if (hasb)
              fa[p.nperseg + nn] = (TF)(-v[e].y * inv * w);
          }
        });
      }
    }
  }
}

// out[c, m] = sum_i frames[c, i, m - i*hop] / sum_i w[m - i*hop]^2 over the
// frames i covering m (unchanged where the squared-window sum is <= 1e-10).
// With m = q*hop + r the covering frames are i = q - back(r) .. q, clipped
// to 0 .. S-1, where back(r) = (nperseg-1-r)/hop; both sums run in frame
// order.  A CTA takes channel blockIdx.y and NQ consecutive q; its threads
// take VEC consecutive offsets r each (one 16-byte load per frame when hop
// and nperseg are multiples of VEC, which also makes back() the same for
// the VEC offsets), so every frame read and output write is a contiguous
// run, and the squared-window sums of the unclipped case are formed once.
template <typename TF, int VEC> struct alignas(sizeof(TF) * VEC) FrameVec {
  TF v[VEC];
};

template <typename TF, int VEC>
__global__ void __launch_bounds__(256)
    istft_ola_kernel(const TF *__restrict__ frames, int64_t C, int64_t S,
                     int64_t nperseg, int64_t hop, int64_t n_total,
                     const double *__restrict__ win, double *__restrict__ out,
                     int64_t o_cs, int64_t o_ss, int64_t nq) {
  using FV = FrameVec<TF, VEC>;
  const int64_t nqt = (n_total + hop - 1) / hop;
  const int64_t q0 = blockIdx.x * nq;
  const int64_t q1 = q0 + nq < nqt ? q0 + nq : nqt;
  for (int64_t c = blockIdx.y; c < C; c += gridDim.y) {
    const TF *fc = frames + c * S * nperseg;
    double *oc = out + c * o_cs;
    for (int r = threadIdx.x * VEC; r < hop; r += blockDim.x * VEC) {
      const int back = (int)((nperseg - 1 - r) / hop);
      double nrm_full[VEC];
#pragma unroll
      for (int u = 0; u < VEC; ++u) {
        nrm_full[u] = 0.0;
        for (int j = back; j >= 0; --j) {
          const double w = win[r + u + j * hop];
          nrm_full[u] += w * w;
        }
      }
      for (int64_t q = q0; q < q1; ++q) {
        const int64_t m = q * hop + r;
        if (m >= n_total)
          break;
        const int64_t i0 = q - back > 0 ? q - back : 0;
        const int64_t i1 = q < S - 1 ? q : S - 1;
        const bool clipped = i0 != q - back || i1 != q;
        const TF *f = fc + i0 * nperseg + (m - i0 * hop);
        const int64_t nf = i1 - i0 + 1;
        double sum[VEC];
#pragma unroll
        for (int u = 0; u < VEC; ++u)
          sum[u] = 0.0;
        constexpr int KM = VEC > 1 ? 4 : 8; // frames loaded at once
        if (nf <= KM) {
          // all loads first, then the frame-order sums
          FV fv[KM];
#pragma unroll
          for (int j = 0; j < KM; ++j)
            if (j < nf)
              fv[j] = *reinterpret_cast<const FV *>(f + j * (nperseg - hop));
#pragma unroll
          for (int j = 0; j < KM; ++j)
            if (j < nf) {
#pragma unroll
              for (int u = 0; u < VEC; ++u)
                sum[u] += (double)fv[j].v[u];
            }
        } else {
          for (int64_t i = i0; i <= i1; ++i, f += nperseg - hop) {
            const FV x = *reinterpret_cast<const FV *>(f);
#pragma unroll
            for (int u = 0; u < VEC; ++u)
              sum[u] += (double)x.v[u];
          }
        }
#pragma unroll
        for (int u = 0; u < VEC; ++u) {
          double nrm = nrm_full[u];
          if (clipped) {
            nrm = 0.0;
            for (int64_t i = i0; i <= i1; ++i) {
              const double w = win[m + u - i * hop];
              nrm += w * w;
            }
          }
          double v = sum[u];
          if (fabs(nrm) > 1e-10)
            v /= nrm;
          oc[(m + u) * o_ss] = v;
        }
      }
    }
  }
}

// Frames are kept in the input's precision: a complex64 spectrum's frames
// (computed in f64) are rounded once to f32, a relative error that the
// overlap-add's division by the squared-window sum does not amplify.
template <typename TZ> using FrameT = TZ;

template <typename TZ, int L, int E>
cudaError_t run_istft_ws(const IstftArgs<double, TZ> &a, int num_sms,
                         cudaStream_t stream) {
  using SS = IstftWsShape<TZ, L, E>;
  auto kern = istft_ws_kernel<TZ, FrameT<TZ>, L, E>;
  static bool attr = false;
  if (!attr) {
    cudaError_t e = cudaFuncSetAttribute(
        kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SS::smem);
    if (e != cudaSuccess)
      return e;
    attr = true;
  }
  const int64_t tiles = a.C * ((a.Tc + SS::Q - 1) / SS::Q);
  const int64_t grid = std::max<int64_t>(1, std::min<int64_t>(tiles, num_sms));
  kern<<<(unsigned)grid, SS::NT, SS::smem, stream>>>(a);
  return cudaGetLastError();
}

#ifndef IB200_ISTFT_WS
#define IB200_ISTFT_WS 1
#endif

template <typename T, typename TZ, int L>
cudaError_t run_istft_len(const IstftDesc &d, int num_sms, cudaStream_t stream,
                          int64_t *launches) {
  using V = typename V2T<T>::type;
  using VZ = typename V2T<TZ>::type;
  using TF = FrameT<TZ>;
  constexpr int E = values_per_thread<T>(L);
  constexpr int P = L / E;
  constexpr int G = (P >= 32 && P <= 256) ? 256 / P : 1;
  auto kern = istft_frames_kernel<T, TZ, TF, L, E, G>;
  const size_t smem = (size_t)G * spad_size(L) * sizeof(V);
  static bool attr = false;
  if (!attr) {
    cudaError_t e = cudaFuncSetAttribute(
        kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess)
      return e;
    attr = true;
  }
  IstftArgs<T, TZ> a{};
  a.z = reinterpret_cast<const VZ *>(d.z);
  a.z_cs = d.z_cs;
  a.z_fs = d.z_fs;
  a.z_ts = d.z_ts;
  a.C = d.C;
  a.F = d.F;
  a.S = d.S;
  a.nperseg = d.nperseg;
  a.pack = d.pack ? 1 : 0;
  a.Tc = d.pack ? (d.S + 1) / 2 : d.S;
  a.win = reinterpret_cast<const T *>(d.win);
  a.tw = reinterpret_cast<const V *>(d.tw);
  a.frames = d.frames;
  cudaError_t e = cudaSuccess;
  bool ws = false;
  // 8 values a thread where that shape fits (at length 2048: 18 warps a
  // CTA at 96 registers and the window in shared memory, against 14 warps at
  // 128 registers with 16 values), else the transforms' own width
  constexpr int EW = IstftWsShape<TZ, L, 8>::ok ? 8 : E;
  if constexpr (std::is_same<T, double>::value &&
                IstftWsShape<TZ, L, EW>::ok && IB200_ISTFT_WS) {
    // unit frame stride and an element-aligned base: cp.async row runs
    ws = d.pack && d.z_ts == 1 &&
         reinterpret_cast<uintptr_t>(d.z) % sizeof(VZ) == 0;
    if (ws)
      e = run_istft_ws<TZ, L, EW>(a, num_sms, stream);
  }
  if (!ws) {
    const int64_t tiles = d.C * ((a.Tc + G - 1) / G);
    const int64_t grid = std::max<int64_t>(
        1, std::min<int64_t>(tiles, (int64_t)num_sms * 8));
    kern<<<(unsigned)grid, G * P, smem, stream>>>(a);
    e = cudaGetLastError();
  }
  if (e != cudaSuccess)
    return e;
  // threads over the offsets within a hop (VEC each), NQ hops per CTA
  // (about 8K outputs), channels on grid.y
  constexpr int VEC = 16 / (int)sizeof(TF);
  const bool vec = d.hop % VEC == 0 && d.nperseg % VEC == 0;
  const int per = vec ? VEC : 1;
  const int threads =
      (int)std::min<int64_t>(256, (d.hop / per + 31) / 32 * 32);
  const int64_t nqt = (d.n_total + d.hop - 1) / d.hop;
  const int64_t nq = std::max<int64_t>(1, 8192 / d.hop);
  const dim3 ogrid((unsigned)((nqt + nq - 1) / nq),
                   (unsigned)std::min<int64_t>(d.C, 65535));
  const TF *fr = static_cast<const TF *>(d.frames);
  if (vec)
    istft_ola_kernel<TF, VEC><<<ogrid, threads, 0, stream>>>(
        fr, d.C, d.S, d.nperseg, d.hop, d.n_total, d.win64, d.out, d.o_cs,
        d.o_ss, nq);
  else
    istft_ola_kernel<TF, 1><<<ogrid, threads, 0, stream>>>(
        fr, d.C, d.S, d.nperseg, d.hop, d.n_total, d.win64, d.out, d.o_cs,
        d.o_ss, nq);
  if (launches)
    *launches += 2;
  return cudaGetLastError();
}

template <typename T, typename TZ>
cudaError_t run_istft_t(const IstftDesc &d, int num_sms, cudaStream_t stream,
                        int64_t *launches) {
  switch (d.nfft) {
  case 16: return run_istft_len<T, TZ, 16>(d, num_sms, stream, launches);
  case 32: return run_istft_len<T, TZ, 32>(d, num_sms, stream, launches);
  case 64: return run_istft_len<T, TZ, 64>(d, num_sms, stream, launches);
  case 128: return run_istft_len<T, TZ, 128>(d, num_sms, stream, launches);
  case 256: return run_istft_len<T, TZ, 256>(d, num_sms, stream, launches);
  case 512: return run_istft_len<T, TZ, 512>(d, num_sms, stream, launches);
  case 1024: return run_istft_len<T, TZ, 1024>(d, num_sms, stream, launches);
  case 2048: return run_istft_len<T, TZ, 2048>(d, num_sms, stream, launches);
  case 4096: return run_istft_len<T, TZ, 4096>(d, num_sms, stream, launches);
  case 8192: return run_istft_len<T, TZ, 8192>(d, num_sms, stream, launches);
  default: return cudaErrorInvalidValue;
  }
}

} // namespace ib200

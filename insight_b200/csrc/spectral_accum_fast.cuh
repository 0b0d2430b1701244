// spectral_accum_fast.cuh — welch / csd fast path (contiguous channels,
// nperseg == nfft, no detrend or DC-only detrend).
//
// CTA b owns the transforms [b*T/n, (b+1)*T/n) of the flattened
// (channel, transform) space (T = channels * transforms per channel, n CTAs),
// so every CTA gets the same work to within one transform.  It runs G
// transform groups of P threads; within each channel of its range group g
// takes the transforms g, g + G, ...  Per transform, as the generic accumulate kernel
// (spectral_kernels.cuh): welch pairs consecutive segments and accumulates
// |Z[k]|^2 of the bins each thread owns, csd pairs x_s with y_s and
// accumulates conj(A[k]) B[k] from Z[k], Z[L-k] staged in shared memory.
// Differences: the window rows and (TWS) the per-thread Stockham twiddles
// are in shared memory, overlapping samples of welch's two segments are read
// once (hop = SH * L/R0), and f32 inputs accumulate in f32 for FL transforms
// before each f64 update, instead of converting and adding in f64 every
// transform (FL = 16 terms of f32 rounding, far below the 1e-5 parity bar).
// At the end of each channel of its range the groups' f64 partials are
// combined in shared memory and written to the slot b + c of the scratch
// array (slots are distinct because the ranges are ordered);
// spectral_finalize_flat_kernel sums the slots of a channel in a fixed
// order (no atomics).
#pragma once
#include "spectral_kernels.cuh"

namespace ib200 {

// 16-byte asynchronous global -> shared copies (cp.async, L2 only), and the
// wait for all of this thread's outstanding copies.  cp.async.wait_group is a
// hardware wait on the thread's own copies, not a spin loop.
__device__ __forceinline__ void cp_async16(void *smem_dst, const void *gsrc) {
  const unsigned d = static_cast<unsigned>(__cvta_generic_to_shared(smem_dst));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(d), "l"(gsrc)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;\n" ::: "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.wait_group 0;\n" ::: "memory");
}

// n contiguous elements (n * sizeof(T) a multiple of 16, both ends 16-byte
// aligned) from src to dst, spread over the P threads of a group.
template <typename T, int P>
__device__ __forceinline__ void stage_copy(T *dst, const T *src, int64_t n,
                                           int t) {
  constexpr int PER = 16 / (int)sizeof(T);
  const int nch = (int)(n / PER);
  for (int j = t; j < nch; j += P)
    cp_async16(dst + j * PER, src + j * PER);
}

// STG: segment samples are staged in shared memory by cp.async one transform
// ahead (the copy for a group's next transform is in flight during this
// transform's FFT); requires 16-byte aligned segment starts.  Without STG
// the samples are loaded straight into registers.
// TWM: Stockham twiddles from the global table (0), from per-thread rows of
// the first twiddle of each butterfly (1), or from full per-thread rows (2).
template <typename T, int L, int E, int G, int SH, int TWM, int MODE, bool STG>
__global__ void __launch_bounds__(G *(L / E))
    accum_fast_kernel(const SpecArgs<T> p) {
  using V = typename V2T<T>::type;
  using PL = Plan<L, E>;
  using TT = ThreadTw<T, L, E>;
  constexpr int P = L / E;
  constexpr int NT = G * P;
  constexpr int R0 = PL::radix(0);
  constexpr int FH = L / 2 + 1;
  constexpr int NB = (FH + P - 1) / P;        // csd bins per thread
  constexpr int GS = (spad_size(L) + 1) / 2 * 2;
  constexpr int WS = E + 16 / (int)sizeof(T);
  constexpr int NACC = MODE == ACC_PSD ? E : 2 * NB;
  constexpr int FL = sizeof(T) == 4 ? 16 : 1; // transforms per f32 partial
  static_assert(SH >= 0 && SH < R0, "overlap shift");
  extern __shared__ __align__(16) unsigned char smem_raw[];
  V *bufs = reinterpret_cast<V *>(smem_raw);               // [G][GS]
  T *raws = reinterpret_cast<T *>(bufs + G * GS);          // [G][2L] (STG)
  V *tws = reinterpret_cast<V *>(raws + (STG ? G * 2 * L : 0)); // [P][stride]
  constexpr int TWROW = TWM == 2 ? TT::stride()
                                 : (TWM == 1 ? ThreadTw1<T, L, E>::stride() : 0);
  T *wsm = reinterpret_cast<T *>(tws + P * TWROW);                // [P][WS]
  const int g = threadIdx.x / P;
  const int t = threadIdx.x - g * P;
  V *buf = bufs + g * GS;
  T *raw = raws + g * 2 * L;

  for (int i = threadIdx.x; i < P * E; i += NT) {
    const int tt = i / E, e = i - tt * E;
    wsm[tt * WS + e] = p.win[in_index<L, E, P>(tt, e)];
  }
  if constexpr (TWM == 2)
    fill_thread_twiddles<T, L, E, P>(tws, p.tw, threadIdx.x, NT);
  else if constexpr (TWM == 1)
    fill_thread_w1<T, L, E, P>(tws, p.tw, threadIdx.x, NT);
  __syncthreads();
  const V *row = tws + t * TWROW;

  T wv[E];
  static_for<0, E>([&](auto eIC) {
    constexpr int e = decltype(eIC)::value;
    wv[e] = wsm[t * WS + e];
  });

  // This CTA's share of the flattened (channel, transform) index space.
  const int64_t T_all = p.C * p.Tc;
  const int64_t f0 = flat_start(blockIdx.x, T_all, gridDim.x);
  const int64_t f1 = flat_start(blockIdx.x + 1, T_all, gridDim.x);
  for (int64_t c = f0 / p.Tc; f0 < f1 && c < p.C && c * p.Tc < f1; ++c) {
    const int64_t task0 = max(f0, c * p.Tc) - c * p.Tc;
    const int64_t task1 = min(f1, (c + 1) * p.Tc) - c * p.Tc;
    const int64_t u = blockIdx.x + c; // partial-sum slot of (CTA, channel)
    const T *xc = p.x + c * p.x_cs + t;
    const T *yc = p.y + c * p.y_cs + t;

    double acc[NACC];
    T accf[NACC];
#pragma unroll
    for (int i = 0; i < NACC; ++i) {
      acc[i] = 0.0;
      accf[i] = T(0);
    }
    int nf = 0;

    // STG: welch copies the pair's span [s*step, (s+1)*step + L) when the
    // segments overlap (b starts at raw + step), else a at raw, b at raw + L;
    // csd copies x_s to raw and y_s to raw + L.
    auto issue = [&](int64_t task) {
      if constexpr (MODE == ACC_PSD) {
        const T *xa = p.x + c * p.x_cs + (p.seg0 + 2 * task) * p.step;
        const bool hasb = (2 * task + 1) < p.S;
        if (hasb && p.step < L) {
          stage_copy<T, P>(raw, xa, p.step + L, t);
        } else {
          stage_copy<T, P>(raw, xa, L, t);
          if (hasb)
            stage_copy<T, P>(raw + L, xa + p.step, L, t);
        }
      } else {
        const int64_t off = (p.seg0 + task) * p.step;
        stage_copy<T, P>(raw, p.x + c * p.x_cs + off, L, t);
        stage_copy<T, P>(raw + L, p.y + c * p.y_cs + off, L, t);
      }
      cp_async_commit();
    };
    if constexpr (STG) {
      if (task0 + g < task1)
        issue(task0 + g);
    }

    for (int64_t task = task0 + g; task < task1; task += G) {
      V vv[1][E];
      V(&v)[E] = vv[0];
      if constexpr (STG) {
        cp_async_wait_all();
        group_sync<G, P>(g); // every thread's copies of this transform landed
        const T *rt = raw + t;
        if constexpr (MODE == ACC_PSD) {
          const bool hasb = (2 * task + 1) < p.S;
          const int64_t boff = p.step < L ? p.step : L;
          T ra[E];
          static_for<0, E>([&](auto eIC) {
            constexpr int e = decltype(eIC)::value;
            ra[e] = rt[in_index<L, E, P>(0, e)];
          });
          if (hasb) {
            static_for<0, E>([&](auto eIC) {
              constexpr int e = decltype(eIC)::value;
              constexpr int r = e % R0;
              T b;
              if constexpr (SH > 0 && r + SH < R0)
                b = ra[e + SH];
              else
                b = rt[boff + in_index<L, E, P>(0, e)];
              v[e] = {ra[e] * wv[e], b * wv[e]};
            });
          } else {
            static_for<0, E>([&](auto eIC) {
              constexpr int e = decltype(eIC)::value;
              v[e] = {ra[e] * wv[e], T(0)};
            });
          }
        } else {
          static_for<0, E>([&](auto eIC) {
            constexpr int e = decltype(eIC)::value;
            constexpr int n = in_index<L, E, P>(0, e);
            v[e] = {rt[n] * wv[e], rt[L + n] * wv[e]};
          });
        }
        group_sync<G, P>(g); // the staging buffer is free again
        if (task + G < task1)
          issue(task + G);
      } else if constexpr (MODE == ACC_PSD) {
        const int64_t s = p.seg0 + 2 * task;
        const bool hasb = (2 * task + 1) < p.S;
        const T *xa = xc + s * p.step;
        T ra[E];
        static_for<0, E>([&](auto eIC) {
          constexpr int e = decltype(eIC)::value;
          ra[e] = __ldg(xa + in_index<L, E, P>(0, e));
        });
        if (hasb) {
          static_for<0, E>([&](auto eIC) {
            constexpr int e = decltype(eIC)::value;
            constexpr int r = e % R0;
            T b;
            if constexpr (SH > 0 && r + SH < R0)
              b = ra[e + SH];
            else
              b = __ldg(xa + p.step + in_index<L, E, P>(0, e));
            v[e] = {ra[e] * wv[e], b * wv[e]};
          });
        } else {
          static_for<0, E>([&](auto eIC) {
            constexpr int e = decltype(eIC)::value;
            v[e] = {ra[e] * wv[e], T(0)};
          });
        }
      } else {
        const int64_t s = p.seg0 + task;
        const T *xa = xc + s * p.step;
        const T *yb = yc + s * p.step;
        static_for<0, E>([&](auto eIC) {
          constexpr int e = decltype(eIC)::value;
          constexpr int n = in_index<L, E, P>(0, e);
          v[e] = {__ldg(xa + n) * wv[e], __ldg(yb + n) * wv[e]};
        });
      }
      if constexpr (TWM == 2)
        fft_group_tw_m<T, L, E, P, G, 1>(vv, buf, GS, t, g, row);
      else if constexpr (TWM == 1)
        fft_group_w1<T, L, E, P, G>(v, buf, t, g, row);
      else
        fft_group<T, L, E, P, G>(v, buf, t, g, p.tw);
      if (p.dc_mode == 1 && t == 0)
        v[0] = {T(0), T(0)}; // register 0 of thread 0 holds bin 0

      if constexpr (MODE == ACC_PSD) {
#pragma unroll
        for (int e = 0; e < E; ++e)
          accf[e] = fma(v[e].x, v[e].x, fma(v[e].y, v[e].y, accf[e]));
      } else {
        store_bins<L, E, P>(v, buf, t);
        group_sync<G, P>(g);
#pragma unroll
        for (int i = 0; i < NB; ++i) {
          const int k = t + i * P;
          if (k < FH) {
            const V zk = buf[spad(k)];
            const V zm = buf[spad((L - k) & (L - 1))];
            // conj(A) B = Im(Z[L-k] Z[k]) / 2 - i (|Z[k]|^2 - |Z[L-k]|^2) / 4
            accf[2 * i] = fma(T(0.5), fma(zm.x, zk.y, zm.y * zk.x), accf[2 * i]);
            accf[2 * i + 1] =
                fma(T(0.25),
                    fma(zm.x, zm.x, zm.y * zm.y) - fma(zk.x, zk.x, zk.y * zk.y),
                    accf[2 * i + 1]);
          }
        }
        group_sync<G, P>(g);
      }
      if (++nf == FL) {
#pragma unroll
        for (int i = 0; i < NACC; ++i) {
          acc[i] += (double)accf[i];
          accf[i] = T(0);
        }
        nf = 0;
      }
    }
#pragma unroll
    for (int i = 0; i < NACC; ++i)
      acc[i] += (double)accf[i];

    // Combine the groups and fold into the unit's scratch slot.
    __syncthreads(); // every group is done with its transform buffer
    if constexpr (MODE == ACC_PSD) {
      double *sm = reinterpret_cast<double *>(buf);
#pragma unroll
      for (int e = 0; e < E; ++e)
        sm[out_bin<L, E, P>(t, e)] = acc[e];
    } else {
      double2 *sm = reinterpret_cast<double2 *>(buf);
#pragma unroll
      for (int i = 0; i < NB; ++i) {
        const int k = t + i * P;
        if (k < FH)
          sm[k] = make_double2(acc[2 * i], acc[2 * i + 1]);
      }
    }
    __syncthreads();
    for (int k = threadIdx.x; k < FH; k += NT) {
      if constexpr (MODE == ACC_PSD) {
        double s = 0.0;
        for (int gg = 0; gg < G; ++gg) {
          const double *sm = reinterpret_cast<const double *>(bufs + gg * GS);
          s += sm[k] + sm[(L - k) & (L - 1)];
        }
        p.scratch[u * FH + k] = s;
      } else {
        double2 s = make_double2(0.0, 0.0);
        for (int gg = 0; gg < G; ++gg) {
          const double2 v2 = reinterpret_cast<const double2 *>(bufs + gg * GS)[k];
          s.x += v2.x;
          s.y += v2.y;
        }
        reinterpret_cast<double2 *>(p.scratch)[u * FH + k] = s;
      }
    }
    __syncthreads();
  }
}

} // namespace ib200

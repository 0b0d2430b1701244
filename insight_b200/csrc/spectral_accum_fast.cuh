// spectral_accum_fast.cuh — welch / csd / coherence fast path (unit sample
// stride, nperseg == nfft, no detrend or DC-only detrend).
//
// CTA b owns the tasks [b*T/n, (b+1)*T/n) of the flattened (channel, task)
// space (T = channels * tasks per channel, n CTAs), so every CTA gets the
// same work to within one task.  It runs G transform groups of P threads;
// within each channel of its range group g takes the tasks g, g + G, ...
// A task is a pair of consecutive segments a = 2 task, b = 2 task + 1,
// transformed together as Z = FFT(w a + i w b) (two real sequences per
// complex transform):
//   welch     accumulates |Z[k]|^2 of the bins each thread owns
//             (|A|^2 + |B|^2 follow from the k and L-k terms at the end);
//   csd       transforms the x pair and the y pair, stages both spectra in
//             shared memory and accumulates conj(Xa) Ya + conj(Xb) Yb from
//             Zx[k], Zx[L-k], Zy[k], Zy[L-k];
//   coherence as csd, plus |Xa|^2 + |Xb|^2 and |Ya|^2 + |Yb|^2.
// Pairing segments of the same signal (rather than x_s with y_s) keeps the
// unpacking error of each spectrum relative to that signal's own power, so a
// quiet y next to a loud x (or y = 0) stays exact to rounding.
// The window rows and the per-thread Stockham twiddles (TWM) are in shared
// memory; overlapping samples of a and b are read once (hop = SH * L/R0);
// with STG the next task's samples are staged by cp.async during this task's
// transforms; welch on f32 inputs accumulates in f32 for FL tasks before each
// f64 update (FL = 16 terms of f32 rounding, far below the 1e-5 parity bar);
// csd and coherence, which hold more accumulators, add into f64 directly.
// At the end of each channel of its range the groups' f64 partials are
// combined in shared memory and written to the slot b + c of the scratch
// array (slots are distinct because the ranges are ordered);
// spectral_finalize_kernel sums the slots of a channel in a fixed order
// (no atomics).
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
// Coherence CTAs (256 threads) are register-capped at 128 so that two fit
// on an SM next to each other.
// MIR (csd, coherence with first-twiddle rows): the last pass runs on
// mirrored butterflies (pair_j), so every thread holds Z[k] and Z[L-k] of
// its bins in registers; x's transform is parked in the thread's own column
// of its buffer while y is transformed, and the cross products need no
// staged spectra, no shared-memory gathers of Z[k], Z[L-k] and one group
// barrier fewer per task.
#ifndef IB200_ACC_MIR
#define IB200_ACC_MIR 1
#endif
// SHF (welch with first-twiddle rows whose transform ends in a radix-2 pass
// after a radix-E pass, in groups of whole warps; with the shapes chosen in
// spectral_dispatch.cuh that is f32 nperseg 8192): the last pass runs on warp
// shuffles (fft_group_w1_lastshfl), one shared-memory exchange and one group
// barrier fewer per transform.
#ifndef IB200_ACC_SHFL
#define IB200_ACC_SHFL 1
#endif
#ifndef IB200_ACC_PF
#define IB200_ACC_PF 1
#endif
// csd and coherence (the mirrored path) run their butterflies on packed f32
// adds (vadd_k / vsub_k in fft_core.cuh): csd 5.27 -> 4.85 ms.
#ifndef IB200_ACC_PACKED
#define IB200_ACC_PACKED 1
#endif
template <typename T, int L, int E>
__host__ __device__ constexpr bool acc_shfl(int mode, int twm) {
  return IB200_ACC_SHFL && mode == ACC_PSD && twm == 1 &&
         LastShfl<L, E>::ok && (L / E) % 32 == 0;
}
template <typename T, int L, int E>
__host__ __device__ constexpr bool acc_mirrored(int mode, int twm) {
  return IB200_ACC_MIR && mode != ACC_PSD && twm == 1 &&
         Plan<L, E>::passes() >= 2 &&
         E / Plan<L, E>::radix(Plan<L, E>::passes() - 1) >= 2;
}

template <typename T, int L, int E>
__host__ __device__ constexpr bool acc_prefetch(int mode, int twm, bool stg) {
  return IB200_ACC_PF && mode == ACC_CSD && !stg && acc_mirrored<T, L, E>(mode, twm);
}
// PFW: the same for welch on the shuffle-last-pass shape (f32 nperseg 8192):
// the next task's samples in registers instead of cp.async staging (two CTA
// barriers a transform fewer), f64 totals in shared memory.
#ifndef IB200_ACC_PFW
#define IB200_ACC_PFW 1
#endif
#ifndef IB200_ACC_L2P
#define IB200_ACC_L2P 1
#endif
template <typename T, int L, int E>
__host__ __device__ constexpr bool acc_prefetch_psd(int mode, int twm, bool stg) {
  return IB200_ACC_PFW && mode == ACC_PSD && !stg && sizeof(T) == 4 &&
         acc_shfl<T, L, E>(mode, twm);
}

template <typename T, int L, int E, int G, int SH, int TWM, int MODE, bool STG>
__global__ void __launch_bounds__(G *(L / E), MODE == ACC_COH ? 2 : 1)
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
  constexpr int NACC = MODE == ACC_PSD ? E : (MODE == ACC_CSD ? 2 : 3) * NB;
  constexpr int FL = sizeof(T) == 4 ? 16 : 1; // transforms per f32 partial
  constexpr int NF = MODE == ACC_PSD ? NACC : 1; // f32 partial accumulators
  static_assert(SH >= 0 && SH < R0, "overlap shift");
  constexpr bool MIR = acc_mirrored<T, L, E>(MODE, TWM);
  constexpr bool SHF = acc_shfl<T, L, E>(MODE, TWM);
  constexpr int RL = PL::radix(PL::passes() - 1); // last-pass radix
  constexpr int NSL = L / RL;
  constexpr int HB = E / RL / 2; // mirrored butterfly pairs per thread
  static_assert(!MIR || NB == E / 2 + 1, "mirrored bins: E/2 + Nyquist");
  // PF (csd on the mirrored path, samples from global memory): the cross
  // products accumulate in f32 for FL tasks and then into f64 totals kept in
  // shared memory, and the registers this frees hold the next transform's
  // samples, loaded during the current transform (y during x's, the next
  // task's x during y's)
  constexpr bool PF = acc_prefetch<T, L, E>(MODE, TWM, STG);
  constexpr bool PFW = acc_prefetch_psd<T, L, E>(MODE, TWM, STG);
  // L2P (f64 welch, samples from global memory): the next task's span is
  // prefetched into L2 by one bulk prefetch a group and task
  constexpr bool L2P = IB200_ACC_L2P && MODE == ACC_PSD && !STG && !PFW &&
                       sizeof(T) == 8;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  // welch: one transform buffer and a 2L staging span per group; csd and
  // coherence: x and y buffers, x and y staging spans.
  constexpr int NBUF = MODE == ACC_PSD ? 1 : 2;
  constexpr int RAWN = NBUF * 2 * L;
  V *bufs = reinterpret_cast<V *>(smem_raw);               // [G][NBUF][GS]
  T *raws = reinterpret_cast<T *>(bufs + G * NBUF * GS);   // [G][RAWN] (STG)
  V *tws = reinterpret_cast<V *>(raws + (STG ? G * RAWN : 0)); // [P][stride]
  constexpr int TWROW = TWM == 2 ? TT::stride()
                                 : (TWM == 1 ? ThreadTw1<T, L, E>::stride() : 0);
  T *wsm = reinterpret_cast<T *>(tws + P * TWROW);                // [P][WS]
  double *acc64 = reinterpret_cast<double *>(wsm + P * WS); // PF: [2NB][NT], PFW: [E][NT]
  const int g = threadIdx.x / P;
  const int t = threadIdx.x - g * P;
  V *buf = bufs + g * NBUF * GS;
  V *buf2 = buf + (NBUF - 1) * GS;
  T *raw = raws + g * RAWN;

  // This CTA's share of the flattened (channel, transform) index space.
  const int64_t T_all = p.C * p.Tc;
  const int64_t f0 = flat_start(blockIdx.x, T_all, gridDim.x);
  const int64_t f1 = flat_start(blockIdx.x + 1, T_all, gridDim.x);
  const int64_t c_first = f0 / p.Tc;

  // STG: the pair's span [s*step, (s+1)*step + L) when the segments
  // overlap (b at + step), else a at + 0 and b at + L; x at raw, y at
  // raw + 2L.
  auto issue_one = [&](T *dst, const T *src, bool hasb) {
    if (hasb && p.step < L) {
      stage_copy<T, P>(dst, src, p.step + L, t);
    } else {
      stage_copy<T, P>(dst, src, L, t);
      if (hasb)
        stage_copy<T, P>(dst + L, src + p.step, L, t);
    }
  };
  auto issue_c = [&](int64_t c, int64_t task) {
    const int64_t off = (p.seg0 + 2 * task) * p.step;
    const bool hasb = (2 * task + 1) < p.S;
    issue_one(raw, p.x + c * p.x_cs + off, hasb);
    if constexpr (MODE != ACC_PSD)
      issue_one(raw + 2 * L, p.y + c * p.y_cs + off, hasb);
    cp_async_commit();
  };
  if constexpr (STG) {
    // the first task's samples are in flight while the tables are filled
    if (f0 < f1 && c_first < p.C) {
      const int64_t task0 = f0 - c_first * p.Tc;
      const int64_t task1 = min(f1, (c_first + 1) * p.Tc) - c_first * p.Tc;
      if (task0 + g < task1)
        issue_c(c_first, task0 + g);
    }
  }

  fill_batched<8>(
      threadIdx.x, P * E, NT,
      [&](int i) { return p.win[in_index<L, E, P>(i / E, i % E)]; },
      [&](int i, T v) { wsm[(i / E) * WS + i % E] = v; });
  if constexpr (TWM == 2)
    fill_thread_twiddles<T, L, E, P>(tws, p.tw, threadIdx.x, NT);
  else if constexpr (TWM == 1)
    fill_thread_w1<T, L, E, P, V, MIR, SHF>(tws, p.tw, threadIdx.x, NT);
  __syncthreads();
  const V *row = tws + t * TWROW;
  // MIR: bin of accumulator slot s (s < E/2: butterfly pair h = s / RL,
  // element r = (s % RL) / 2, the mirror half when s is odd; slot E/2 is the
  // Nyquist bin of thread 0)
  auto mir_bin = [&](int s) -> int {
    if (s == E / 2)
      return L / 2;
    const int h = s / RL, r = (s % RL) / 2;
    return pair_j<L, E, P>(t, h + (s & 1) * HB) + NSL * r;
  };

  // welch keeps the window values in registers when they are few (f32 and
  // short f64 rows); csd, coherence and long f64 rows reread them from the
  // shared-memory row per load.
  constexpr bool WREG = MODE == ACC_PSD && E * sizeof(T) <= 64;
  constexpr int NW = WREG ? E : 1;
  T wreg[NW];
  static_for<0, NW>([&](auto eIC) {
    constexpr int e = decltype(eIC)::value;
    wreg[e] = wsm[t * WS + e];
  });
  const T *wrow = wsm + t * WS;

  // Windowed pair a + i b of the segments 2 task, 2 task + 1 of one signal:
  // src points at this thread's first sample of a (shared staging or global
  // memory), b starts boff samples later; with SH > 0 the samples b shares
  // with a come from a's registers.
  auto load_v = [&](V(&v)[E], const T *src, int64_t boff, bool hasb) {
    T wv[E];
    static_for<0, E>([&](auto eIC) {
      constexpr int e = decltype(eIC)::value;
      if constexpr (WREG)
        wv[e] = wreg[e];
      else
        wv[e] = wrow[e];
    });
    T ra[E];
    static_for<0, E>([&](auto eIC) {
      constexpr int e = decltype(eIC)::value;
      if constexpr (STG)
        ra[e] = src[in_index<L, E, P>(0, e)];
      else
        ra[e] = __ldg(src + in_index<L, E, P>(0, e));
    });
    if (hasb) {
      static_for<0, E>([&](auto eIC) {
        constexpr int e = decltype(eIC)::value;
        constexpr int r = e % R0;
        T b;
        if constexpr (SH > 0 && r + SH < R0)
          b = ra[e + SH];
        else if constexpr (STG)
          b = src[boff + in_index<L, E, P>(0, e)];
        else
          b = __ldg(src + boff + in_index<L, E, P>(0, e));
        v[e] = {ra[e] * wv[e], b * wv[e]};
      });
    } else {
      static_for<0, E>([&](auto eIC) {
        constexpr int e = decltype(eIC)::value;
        v[e] = {ra[e] * wv[e], T(0)};
      });
    }
  };
  auto fft = [&](V(&v)[E], V *b) {
    if constexpr (MIR)
      fft_group_w1_pairs<T, L, E, P, G, IB200_ACC_PACKED>(v, b, t, g, row);
    else if constexpr (SHF)
      fft_group_w1_lastshfl<T, L, E, P, G>(v, b, t, g, row);
    else if constexpr (TWM == 2)
      fft_group_tw_m<T, L, E, P, G, 1>(&v, b, GS, t, g, row);
    else if constexpr (TWM == 1)
      fft_group_w1<T, L, E, P, G>(v, b, t, g, row);
    else
      fft_group<T, L, E, P, G>(v, b, t, g, p.tw);
    if (p.dc_mode == 1 && t == 0)
      v[0] = {T(0), T(0)}; // register 0 of thread 0 holds bin 0
  };

  for (int64_t c = c_first; f0 < f1 && c < p.C && c * p.Tc < f1; ++c) {
    const int64_t task0 = max(f0, c * p.Tc) - c * p.Tc;
    const int64_t task1 = min(f1, (c + 1) * p.Tc) - c * p.Tc;
    const int64_t u = blockIdx.x + c; // partial-sum slot of (CTA, channel)
    const T *xc = p.x + c * p.x_cs;
    const T *yc = p.y + c * p.y_cs;

    double acc[NACC];
    T accf[NF];
#pragma unroll
    for (int i = 0; i < NACC; ++i)
      acc[i] = 0.0;
#pragma unroll
    for (int i = 0; i < NF; ++i)
      accf[i] = T(0);
    int nf = 0;

    auto issue = [&](int64_t task) { issue_c(c, task); };
    if constexpr (STG) {
      // the first channel's first task was requested before the prologue
      if (c != c_first && task0 + g < task1)
        issue(task0 + g);
    }

    if constexpr (PFW) {
      // welch: f32 partials (FL tasks) over f64 totals in shared memory, the
      // next task's samples loaded into registers during this transform
#pragma unroll
      for (int i = 0; i < E; ++i)
        acc64[i * NT + threadIdx.x] = 0.0;
      constexpr int NBO = [] {
        int n = 0;
        for (int e = 0; e < E; ++e)
          if (!(SH > 0 && (e % R0) + SH < R0))
            ++n;
        return n;
      }();
      T ra[E], rb[NBO > 0 ? NBO : 1];
      auto load_raw = [&](const T *src, int64_t task) {
        const bool hb = (2 * task + 1) < p.S;
        static_for<0, E>([&](auto eIC) {
          constexpr int e = decltype(eIC)::value;
          ra[e] = __ldg(src + in_index<L, E, P>(0, e));
        });
        int j = 0;
        static_for<0, E>([&](auto eIC) {
          constexpr int e = decltype(eIC)::value;
          if constexpr (!(SH > 0 && (e % R0) + SH < R0)) {
            rb[j] = hb ? __ldg(src + p.step + in_index<L, E, P>(0, e)) : T(0);
            ++j;
          }
        });
      };
      auto soff = [&](int64_t task) { return (p.seg0 + 2 * task) * p.step + t; };
      if (task0 + g < task1)
        load_raw(xc + soff(task0 + g), task0 + g);
      int nfl = 0;
      for (int64_t task = task0 + g; task < task1; task += G) {
        const bool hasb = (2 * task + 1) < p.S;
        V v[E];
        int j = 0;
        static_for<0, E>([&](auto eIC) {
          constexpr int e = decltype(eIC)::value;
          const T w = wreg[WREG ? e : 0];
          T b;
          if constexpr (SH > 0 && (e % R0) + SH < R0)
            b = ra[e + SH];
          else
            b = rb[j++];
          v[e] = {ra[e] * w, hasb ? b * w : T(0)};
        });
        if (task + G < task1)
          load_raw(xc + soff(task + G), task + G);
        fft(v, buf);
#pragma unroll
        for (int e = 0; e < E; ++e)
          accf[e] = fma(v[e].x, v[e].x, fma(v[e].y, v[e].y, accf[e]));
        if (++nfl == FL) {
#pragma unroll
          for (int i = 0; i < E; ++i) {
            acc64[i * NT + threadIdx.x] += (double)accf[i];
            accf[i] = T(0);
          }
          nfl = 0;
        }
      }
#pragma unroll
      for (int i = 0; i < E; ++i) {
        acc[i] = acc64[i * NT + threadIdx.x] + (double)accf[i];
        accf[i] = T(0); // already folded in
      }
    } else if constexpr (PF) {
      // f32 partials (FL tasks) over f64 totals in shared memory
      T accp[2 * NB];
#pragma unroll
      for (int i = 0; i < 2 * NB; ++i) {
        accp[i] = T(0);
        acc64[i * NT + threadIdx.x] = 0.0;
      }
      // samples of one transform: a (E values) and b's own (the rest share
      // a's registers through the overlap shift)
      constexpr int NBO = [] {
        int n = 0;
        for (int e = 0; e < E; ++e)
          if (!(SH > 0 && (e % R0) + SH < R0))
            ++n;
        return n;
      }();
      T ra[E], rb[NBO > 0 ? NBO : 1];
      auto load_raw = [&](const T *src, int64_t task) {
        const bool hb = (2 * task + 1) < p.S;
        static_for<0, E>([&](auto eIC) {
          constexpr int e = decltype(eIC)::value;
          ra[e] = __ldg(src + in_index<L, E, P>(0, e));
        });
        int j = 0;
        static_for<0, E>([&](auto eIC) {
          constexpr int e = decltype(eIC)::value;
          if constexpr (!(SH > 0 && (e % R0) + SH < R0)) {
            rb[j] = hb ? __ldg(src + p.step + in_index<L, E, P>(0, e)) : T(0);
            ++j;
          }
        });
      };
      auto form = [&](V(&v)[E], bool hb) {
        int j = 0;
        static_for<0, E>([&](auto eIC) {
          constexpr int e = decltype(eIC)::value;
          const T w = wrow[e];
          T b;
          if constexpr (SH > 0 && (e % R0) + SH < R0)
            b = ra[e + SH];
          else
            b = rb[j++];
          v[e] = {ra[e] * w, hb ? b * w : T(0)};
        });
      };
      auto soff = [&](int64_t task) { return (p.seg0 + 2 * task) * p.step + t; };
      if (task0 + g < task1)
        load_raw(xc + soff(task0 + g), task0 + g);
      int nfl = 0;
      for (int64_t task = task0 + g; task < task1; task += G) {
        const bool hasb = (2 * task + 1) < p.S;
        V v[E];
        form(v, hasb);                       // x
        load_raw(yc + soff(task), task);     // y, during x's transform
        fft(v, buf);
        // park x's registers in this thread's column of buf: every read of
        // buf by the transform ended at its last group barrier
#pragma unroll
        for (int e = 0; e < E; ++e)
          buf[e * P + t] = v[e];
        form(v, hasb);                       // y
        if (task + G < task1)                // the next x, during y's transform
          load_raw(xc + soff(task + G), task + G);
        fft(v, buf2);
        // 4 (conj(Xa) Ya + conj(Xb) Yb) = 2 (conj(Zx[k]) Zy[k] +
        // Zx[L-k] conj(Zy[L-k])): the segment spectra need not be unpacked
        auto bin = [&](auto sIC, V xk, V xm, V yk, V ym) {
          constexpr int sb = decltype(sIC)::value;
          const T re = fma(xk.x, yk.x, fma(xk.y, yk.y, fma(xm.x, ym.x, xm.y * ym.y)));
          const T im = fma(xk.x, yk.y, fma(-xk.y, yk.x, fma(xm.y, ym.x, -xm.x * ym.y)));
          accp[2 * sb] = fma(T(2), re, accp[2 * sb]);
          accp[2 * sb + 1] = fma(T(2), im, accp[2 * sb + 1]);
        };
        auto px = [&](int e) { return buf[e * P + t]; };
        const bool j0 = t == 0; // butterflies 0 and NS/2 mirror themselves
        static_for<0, HB>([&](auto hIC) {
          constexpr int h = decltype(hIC)::value;
          static_for<0, RL / 2>([&](auto rIC) {
            constexpr int r = decltype(rIC)::value;
            constexpr int ea = h * RL + bitrev<RL>(r);
            constexpr int eam = (h + HB) * RL + bitrev<RL>(RL - 1 - r);
            constexpr int eself = h * RL + bitrev<RL>((RL - r) % RL);
            constexpr int ec = (h + HB) * RL + bitrev<RL>(r);
            constexpr int ecm = h * RL + bitrev<RL>(RL - 1 - r);
            const bool self = h == 0 && j0;
            bin(std::integral_constant<int, h * RL + 2 * r>{}, px(ea),
                px(self ? eself : eam), v[ea], self ? v[eself] : v[eam]);
            bin(std::integral_constant<int, h * RL + 2 * r + 1>{}, px(ec),
                px(self ? eam : ecm), v[ec], self ? v[eam] : v[ecm]);
          });
        });
        if (j0) {
          constexpr int en = bitrev<RL>(RL / 2);
          bin(std::integral_constant<int, E / 2>{}, px(en), px(en), v[en], v[en]);
        }
        group_sync<G, P>(g); // the parked column is read before buf is reused
        if (++nfl == FL) {
#pragma unroll
          for (int i = 0; i < 2 * NB; ++i) {
            acc64[i * NT + threadIdx.x] += (double)accp[i];
            accp[i] = T(0);
          }
          nfl = 0;
        }
      }
#pragma unroll
      for (int i = 0; i < 2 * NB; ++i)
        acc[i] = acc64[i * NT + threadIdx.x] + (double)accp[i];
    } else
    for (int64_t task = task0 + g; task < task1; task += G) {
      const bool hasb = (2 * task + 1) < p.S;
      const int64_t off = (p.seg0 + 2 * task) * p.step;
      const int64_t boff = STG ? ((hasb && p.step < L) ? p.step : L) : p.step;
      V v[E];
      if constexpr (STG) {
        cp_async_wait_all();
        group_sync<G, P>(g); // every thread's copies of this task landed
      }
      if constexpr (L2P) {
        // the group's next task span [off', off' + step + L) (just L without
        // its segment b) into L2 while this task's samples are used
        if (t == 0 && task + G < task1) {
          const int64_t tn = task + G;
          const int64_t n = ((2 * tn + 1) < p.S ? p.step : 0) + L;
          const T *src = xc + (p.seg0 + 2 * tn) * p.step;
          const uint64_t bytes = (uint64_t)n * sizeof(T);
          // a bulk prefetch needs a 16-byte aligned start and size
          if ((reinterpret_cast<uintptr_t>(src) & 15) == 0 && (bytes & 15) == 0)
            asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src),
                         "r"((unsigned)bytes)
                         : "memory");
        }
      }
      load_v(v, STG ? raw + t : xc + off + t, boff, hasb);
      if constexpr (MODE == ACC_PSD) {
        if constexpr (STG) {
          group_sync<G, P>(g); // the staging span is free again
          if (task + G < task1)
            issue(task + G);
        }
        fft(v, buf);
#pragma unroll
        for (int e = 0; e < E; ++e)
          accf[e] = fma(v[e].x, v[e].x, fma(v[e].y, v[e].y, accf[e]));
      } else if constexpr (MIR) {
        fft(v, buf);
        // park x's registers in this thread's column of buf: every read of
        // buf by the transform ended at its last group barrier
#pragma unroll
        for (int e = 0; e < E; ++e)
          buf[e * P + t] = v[e];
        load_v(v, STG ? raw + 2 * L + t : yc + off + t, boff, hasb);
        if constexpr (STG) {
          group_sync<G, P>(g); // the staging spans are free again
          if (task + G < task1)
            issue(task + G);
        }
        fft(v, buf2);
        // Zx = Xa + i Xb, Zy = Ya + i Yb: as in the staged epilogue below,
        // from registers (y) and the parked column (x)
        // 4 (conj(Xa) Ya + conj(Xb) Yb) = 2 (conj(Zx[k]) Zy[k] +
        // Zx[L-k] conj(Zy[L-k])) and 4 (|Xa|^2 + |Xb|^2) =
        // 2 (|Zx[k]|^2 + |Zx[L-k]|^2): the segment spectra need not be
        // unpacked
        auto bin = [&](auto sIC, V xk, V xm, V yk, V ym) {
          constexpr int s = decltype(sIC)::value;
          const T re = T(2) * fma(xk.x, yk.x, fma(xk.y, yk.y, fma(xm.x, ym.x, xm.y * ym.y)));
          if constexpr (MODE == ACC_COH) {
            acc[3 * s] += (double)(T(2) * fma(xk.x, xk.x, fma(xk.y, xk.y,
                                                 fma(xm.x, xm.x, xm.y * xm.y))));
            acc[3 * s + 1] += (double)(T(2) * fma(yk.x, yk.x, fma(yk.y, yk.y,
                                                     fma(ym.x, ym.x, ym.y * ym.y))));
            acc[3 * s + 2] += (double)re;
          } else {
            const T im = T(2) * fma(xk.x, yk.y, fma(-xk.y, yk.x, fma(xm.y, ym.x, -xm.x * ym.y)));
            acc[2 * s] += (double)re;
            acc[2 * s + 1] += (double)im;
          }
        };
        auto px = [&](int e) { return buf[e * P + t]; };
        const bool j0 = t == 0; // butterflies 0 and NS/2 mirror themselves
        static_for<0, HB>([&](auto hIC) {
          constexpr int h = decltype(hIC)::value;
          static_for<0, RL / 2>([&](auto rIC) {
            constexpr int r = decltype(rIC)::value;
            constexpr int ea = h * RL + bitrev<RL>(r);
            constexpr int eam = (h + HB) * RL + bitrev<RL>(RL - 1 - r);
            constexpr int eself = h * RL + bitrev<RL>((RL - r) % RL);
            constexpr int ec = (h + HB) * RL + bitrev<RL>(r);
            constexpr int ecm = h * RL + bitrev<RL>(RL - 1 - r);
            const bool self = h == 0 && j0;
            bin(std::integral_constant<int, h * RL + 2 * r>{}, px(ea),
                px(self ? eself : eam), v[ea], self ? v[eself] : v[eam]);
            bin(std::integral_constant<int, h * RL + 2 * r + 1>{}, px(ec),
                px(self ? eam : ecm), v[ec], self ? v[eam] : v[ecm]);
          });
        });
        if (j0) {
          constexpr int en = bitrev<RL>(RL / 2);
          bin(std::integral_constant<int, E / 2>{}, px(en), px(en), v[en], v[en]);
        }
        group_sync<G, P>(g); // the parked column is read before buf is reused
      } else {
        fft(v, buf);
        store_bins<L, E, P>(v, buf, t);
        load_v(v, STG ? raw + 2 * L + t : yc + off + t, boff, hasb);
        if constexpr (STG) {
          group_sync<G, P>(g); // the staging spans are free again
          if (task + G < task1)
            issue(task + G);
        }
        fft(v, buf2);
        store_bins<L, E, P>(v, buf2, t);
        group_sync<G, P>(g);
        // Zx = Xa + i Xb, Zy = Ya + i Yb (segments a, b of x and of y):
        // 2 Xa = Zx[k] + conj Zx[L-k], 2 Xb = -i (Zx[k] - conj Zx[L-k]).
        // Partials are 4 (conj(Xa) Ya + conj(Xb) Yb) (and 4 |X|^2, 4 |Y|^2).
#pragma unroll
        for (int i = 0; i < NB; ++i) {
          const int k = t + i * P;
          if (k < FH) {
            const int m = (L - k) & (L - 1);
            const V xk = buf[spad(k)], xm = buf[spad(m)];
            const V yk = buf2[spad(k)], ym = buf2[spad(m)];
            const T xar = xk.x + xm.x, xai = xk.y - xm.y;
            const T xbr = xk.y + xm.y, xbi = xm.x - xk.x;
            const T yar = yk.x + ym.x, yai = yk.y - ym.y;
            const T ybr = yk.y + ym.y, ybi = ym.x - yk.x;
            const T re = fma(xar, yar, fma(xai, yai, fma(xbr, ybr, xbi * ybi)));
            if constexpr (MODE == ACC_COH) {
              acc[3 * i] +=
                  (double)fma(xar, xar, fma(xai, xai, fma(xbr, xbr, xbi * xbi)));
              acc[3 * i + 1] +=
                  (double)fma(yar, yar, fma(yai, yai, fma(ybr, ybr, ybi * ybi)));
              acc[3 * i + 2] += (double)re;
            } else {
              const T im = fma(xar, yai, fma(-xai, yar, fma(xbr, ybi, -xbi * ybr)));
              acc[2 * i] += (double)re;
              acc[2 * i + 1] += (double)im;
            }
          }
        }
        group_sync<G, P>(g);
      }
      if constexpr (MODE == ACC_PSD) {
        if (++nf == FL) {
#pragma unroll
          for (int i = 0; i < NF; ++i) {
            acc[i] += (double)accf[i];
            accf[i] = T(0);
          }
          nf = 0;
        }
      }
    }
    if constexpr (MODE == ACC_PSD) {
#pragma unroll
      for (int i = 0; i < NF; ++i)
        acc[i] += (double)accf[i];
    }

    // Combine the groups and fold into the unit's scratch slot.
    __syncthreads(); // every group is done with its transform buffer
    if constexpr (MODE == ACC_PSD) {
      double *sm = reinterpret_cast<double *>(buf);
#pragma unroll
      for (int e = 0; e < E; ++e)
        sm[SHF ? shfl_bin<L, E>(t, e) : out_bin<L, E, P>(t, e)] = acc[e];
      __syncthreads();
      for (int k = threadIdx.x; k < FH; k += NT) {
        double s = 0.0;
        for (int gg = 0; gg < G; ++gg) {
          const double *sm =
              reinterpret_cast<const double *>(bufs + gg * NBUF * GS);
          s += sm[k] + sm[(L - k) & (L - 1)];
        }
        p.scratch[u * FH + k] = s;
      }
      __syncthreads();
    } else {
      // csd: one round of (re, im); coherence: rounds (Sxx, Syy), (Sxy, 0)
      constexpr int ROUNDS = MODE == ACC_CSD ? 1 : 2;
      constexpr int W = MODE == ACC_CSD ? 2 : 3;
      static_for<0, ROUNDS>([&](auto rIC) {
        constexpr int r = decltype(rIC)::value;
        double2 *sm = reinterpret_cast<double2 *>(buf);
#pragma unroll
        for (int i = 0; i < NB; ++i) {
          const int k = MIR ? (i < E / 2 || t == 0 ? mir_bin(i) : FH) : t + i * P;
          if (k < FH) {
            if constexpr (r == 0)
              sm[k] = make_double2(acc[W * i], acc[W * i + 1]);
            else
              sm[k] = make_double2(acc[W * i + W - 1], 0.0);
          }
        }
        __syncthreads();
        for (int k = threadIdx.x; k < FH; k += NT) {
          double2 s = make_double2(0.0, 0.0);
          for (int gg = 0; gg < G; ++gg) {
            const double2 v2 =
                reinterpret_cast<const double2 *>(bufs + gg * NBUF * GS)[k];
            s.x += v2.x;
            s.y += v2.y;
          }
          reinterpret_cast<double2 *>(p.scratch)[ROUNDS * (u * FH + k) + r] = s;
        }
        __syncthreads();
      });
    }
  }
}

} // namespace ib200

// spectral_stft_ws.cuh — warp-specialised STFT fast path.
//
// Same result, input and output conditions as stft_fast_kernel
// (spectral_kernels.cuh: unit sample stride, nperseg == nfft, no or DC-only
// detrend, complex (C, F, S) output with unit segment stride), with the work
// of a CTA split by role instead of by phase:
//   * warps 0 .. NFT/32-1 are GF transform groups of P threads; for each tile
//     (GF segment pairs) every group loads, windows and transforms one pair
//     into its slot of staging buffer b = tile & 1;
//   * the other NST threads are store warps: they unpack the pairs of a full
//     buffer into the tile's 2*GF output columns of every bin row, with the
//     same sector-aligned carry scheme as stft_fast_kernel, and release it.
// The roles meet only at named hardware barriers (bar.arrive / bar.sync on
// FULL(b) and EMPTY(b), counted over the whole CTA), so one buffer is
// transformed while the other is written out: the FP work of the transforms
// and the memory work of the stores overlap on every SM instead of
// alternating behind __syncthreads.
#pragma once
#include "spectral_kernels.cuh"

namespace ib200 {

__device__ __forceinline__ void named_arrive(int id, int count) {
  asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(count) : "memory");
}
__device__ __forceinline__ void named_sync(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

template <typename T, int L> struct StftWsShape {
  static constexpr int E = values_per_thread<T>(L);
  static constexpr int P = L / E;
  static constexpr int NFT = 512;                   // transform threads
  static constexpr int GF = P <= NFT ? NFT / P : 0; // transform groups
#ifndef IB200_STFT_WS_NST
#define IB200_STFT_WS_NST 256
#endif
  static constexpr int NST = IB200_STFT_WS_NST;    // store threads
  static constexpr int NT = NFT + NST;
  static constexpr int Q = GF;                      // pairs per tile
  static constexpr int SPR = 2 * Q;                 // columns per tile row
  static constexpr int SEC = 32 / (2 * (int)sizeof(T));
  // pair stride: slot spad_size(L) holds a copy of Z[0]; for f32 the extra
  // 16/Q slots put the Q pairs x 16/Q rows a store warp reads at once on
  // distinct banks (pair p, row r -> bank 2 (GS p + r) mod 32)
  static constexpr int GS =
      spad_size(L) + (sizeof(T) == 4 && GF >= 1 && GF <= 8 ? 16 / GF : 2);
  static constexpr int FH = L / 2 + 1;
  static constexpr int CN =
      (FH * (SEC - 1) * 2 * (int)sizeof(T) + 15) / 16 * 16 / (2 * (int)sizeof(T));
  static constexpr int WS = E + 16 / (int)sizeof(T);
  // shape usable: whole sectors per tile row, group barriers of whole warps
  static constexpr bool ok = GF >= 2 && P % 32 == 0 && SPR >= SEC &&
                             SPR % SEC == 0 && NST % SPR == 0 &&
                             (NST / SPR) % SEC == 0 && GF + 5 <= 16;
  // twm: 2 full per-thread twiddle rows, 1 first-twiddle rows (powers by
  // multiplication: less shared-memory traffic, more FMA work), 0 table
  __host__ __device__ static constexpr int tw_stride(int twm) {
    return twm == 2 ? ThreadTw<T, L, E>::stride()
                    : (twm == 1 ? ThreadTw1<T, L, E>::stride() : 0);
  }
  __host__ __device__ static constexpr size_t smem(int twm) {
    return (size_t)2 * Q * GS * 2 * sizeof(T) +
           (size_t)P * tw_stride(twm) * 2 * sizeof(T) +
           (size_t)CN * 2 * sizeof(T) + (size_t)P * WS * sizeof(T);
  }
};

template <typename T, int L, int SH, int TWM>
__global__ void __launch_bounds__(StftWsShape<T, L>::NT)
    stft_ws_kernel(const SpecArgs<T> p, int nsub) {
  using V = typename V2T<T>::type;
  using SS = StftWsShape<T, L>;
  constexpr int TWROW = SS::tw_stride(TWM);
  constexpr int E = SS::E, P = SS::P, GF = SS::GF, NFT = SS::NFT, NT = SS::NT;
  constexpr int Q = SS::Q, SPR = SS::SPR, SEC = SS::SEC, GS = SS::GS;
  constexpr int FH = SS::FH, CN = SS::CN, WS = SS::WS;
  constexpr int R0 = Plan<L, E>::radix(0);
  constexpr int RPI = SS::NST / SPR; // bin rows per store iteration
  constexpr int NIT = (FH + RPI - 1) / RPI;
  // barrier ids: 0 CTA, 1..GF transform groups, then FULL(b), EMPTY(b)
  constexpr int FULL0 = GF + 1, EMPTY0 = GF + 3;
  static_assert(SS::ok, "shape");
  static_assert(SH >= 0 && SH < R0, "overlap shift");
  extern __shared__ __align__(16) unsigned char smem_raw[];
  V *stage = reinterpret_cast<V *>(smem_raw);              // [2][Q][GS]
  V *tws = stage + 2 * Q * GS;                              // [P][TWROW]
  V *carry = tws + P * TWROW;                               // [FH][SEC-1]
  T *wsm = reinterpret_cast<T *>(carry + CN);                // [P][WS]

  fill_batched<8>(
      threadIdx.x, P * E, NT,
      [&](int i) { return T(0.5) * p.win[in_index<L, E, P>(i / E, i % E)]; },
      [&](int i, T v) { wsm[(i / E) * WS + i % E] = v; });
  if constexpr (TWM == 2)
    fill_thread_twiddles<T, L, E, P>(tws, p.tw, threadIdx.x, NT);
  else if constexpr (TWM == 1)
    fill_thread_w1<T, L, E, P>(tws, p.tw, threadIdx.x, NT);
  __syncthreads();

  const int64_t tpc = (p.Tc + Q - 1) / Q;      // tiles per channel
  const int64_t upc = (tpc + nsub - 1) / nsub; // units per channel
  const int64_t nunits = p.C * upc;
  V *out = reinterpret_cast<V *>(p.out);

  if (threadIdx.x < NFT) {
    // ------------------------------------------------------------ transforms
    const int g = threadIdx.x / P;
    const int t = threadIdx.x - g * P;
    const V *row = tws + t * TWROW;
    // first-twiddle rows (TWM 1) are a few values a thread, the same for
    // every pair: held in registers instead of reread per transform
    constexpr int NR1 = TWM == 1 ? ThreadTw1<T, L, E>::total() : 1;
    V row1[NR1];
    static_for<0, NR1>([&](auto iIC) {
      constexpr int i = decltype(iIC)::value;
      row1[i] = TWM == 1 ? row[i] : V{T(1), T(0)};
    });
    int64_t tile = 0; // tiles of this CTA so far (buffer = tile & 1)
    for (int64_t unit = blockIdx.x; unit < nunits; unit += gridDim.x) {
      const int64_t c = unit / upc;
      const int64_t tile0 = (unit - c * upc) * nsub;
      const int ntile = (int)min((int64_t)nsub, tpc - tile0);
      for (int it = 0; it < ntile; ++it, ++tile) {
        const int b = (int)(tile & 1);
        if (tile >= 2)
          named_sync(EMPTY0 + b, NT); // the store warps released buffer b
        V *buf = stage + (b * Q + g) * GS;
        const int64_t task = (tile0 + it) * Q + g;
        if (task < p.Tc) {
          const bool hasb = (2 * task + 1) < p.S;
          const T *xa = p.x + c * p.x_cs + (p.seg0 + 2 * task) * p.step + t;
          V v[1][E];
          T ra[E], wv[E];
          static_for<0, E>([&](auto eIC) {
            constexpr int e = decltype(eIC)::value;
            ra[e] = __ldg(xa + in_index<L, E, P>(0, e));
          });
          // window row: 128-bit reads (the row stride WS keeps them
          // conflict-free)
          if constexpr (sizeof(T) == 4 && E % 4 == 0) {
            const float4 *w4 = reinterpret_cast<const float4 *>(wsm + t * WS);
            static_for<0, E / 4>([&](auto qIC) {
              constexpr int q = decltype(qIC)::value;
              const float4 f = w4[q];
              wv[4 * q] = f.x;
              wv[4 * q + 1] = f.y;
              wv[4 * q + 2] = f.z;
              wv[4 * q + 3] = f.w;
            });
          } else {
            static_for<0, E>([&](auto eIC) {
              constexpr int e = decltype(eIC)::value;
              wv[e] = wsm[t * WS + e];
            });
          }
          static_for<0, E>([&](auto eIC) {
            constexpr int e = decltype(eIC)::value;
            constexpr int r = e % R0;
            const T w = wv[e];
            T bv = T(0);
            if (hasb) {
              if constexpr (SH > 0 && r + SH < R0)
                bv = ra[e + SH];
              else
                bv = __ldg(xa + p.step + in_index<L, E, P>(0, e));
            }
            v[0][e] = {ra[e] * w, bv * w};
          });
          if constexpr (TWM == 2)
            fft_group_tw_m<T, L, E, P, GF, 1>(v, buf, GS, t, g, row);
          else if constexpr (TWM == 1)
            fft_group_w1<T, L, E, P, GF>(v[0], buf, t, g, row1);
          else
            fft_group<T, L, E, P, GF>(v[0], buf, t, g, p.tw);
          if (p.dc_mode == 1 && t == 0)
            v[0][0] = {T(0), T(0)};
          store_bins<L, E, P>(v[0], buf, t);
          if (t == 0)
            buf[spad_size(L)] = v[0][0];
        }
        named_arrive(FULL0 + b, NT); // buffer b holds this tile
      }
    }
    // wait for the last releases so every barrier phase completes
    for (int64_t k = tile >= 2 ? tile - 2 : 0; k < tile; ++k)
      named_sync(EMPTY0 + (int)(k & 1), NT);
    return;
  }

  // ------------------------------------------------------------------ stores
  const int st = threadIdx.x - NFT;
  const int lane = st % SPR;
  const int kr0 = st / SPR;
  static_assert(RPI % SEC == 0, "a thread's rows share one sector phase");
  int64_t tile = 0;
  for (int64_t unit = blockIdx.x; unit < nunits; unit += gridDim.x) {
    const int64_t c = unit / upc;
    const int64_t tile0 = (unit - c * upc) * nsub;
    const int ntile = (int)min((int64_t)nsub, tpc - tile0);
    const int64_t ucol0 = 2 * tile0 * Q; // first column of the unit
    V *outc = out + c * p.o_cs;
    // this thread's store role for the unit (as in stft_fast_kernel)
    const int phi = (int)((reinterpret_cast<uint64_t>(outc + (int64_t)kr0 * p.o_rs +
                                                       ucol0) /
                           sizeof(V)) & (SEC - 1));
    const bool carry_lane = lane < phi;
    const int jj = carry_lane ? SPR - phi + lane : lane - phi; // tile column
    const bool odd = jj & 1;
    for (int it = 0; it < ntile; ++it, ++tile) {
      const int b = (int)(tile & 1);
      named_sync(FULL0 + b, NT); // the transform groups filled buffer b
      const V *zkp = stage + (b * Q + (jj >> 1)) * GS + spad(kr0);
      const V *zmp = stage + (b * Q + (jj >> 1)) * GS + spad(L - kr0);
      const int64_t task0 = (tile0 + it) * Q;
      const bool first = it == 0;
      const bool last = it == ntile - 1;
      const int64_t col0 = 2 * task0;
      V *rp0 = outc + (int64_t)kr0 * p.o_rs + col0 - phi;
      const int64_t rstep = (int64_t)RPI * p.o_rs;
      const bool wmain = (col0 - phi + lane) < p.S && (!carry_lane || !first);
      const bool wtrail = carry_lane && last && (col0 + jj) < p.S;
      const bool wcarry = carry_lane && !last;
      static_for<0, NIT>([&](auto iIC) {
        constexpr int ii = decltype(iIC)::value;
        const int k = kr0 + ii * RPI;
        if (ii + 1 < NIT || k < FH) {
          const V zk = zkp[ii * pad_off<RPI>()];
          const V zm = zmp[-ii * pad_off<RPI>()];
          // even: A = zk + conj zm; odd: B = -i (zk - conj zm)
          const T u = odd ? zk.y : zk.x;
          const T w = odd ? zm.y : zm.x;
          const T u2 = odd ? zm.x : zk.y;
          const T w2 = odd ? zk.x : zm.y;
          const V val = V{u + w, u2 - w2};
          V *rp = rp0 + ii * rstep;
          V *cr = carry + k * (SEC - 1) + lane;
          V sv = val;
          if (carry_lane)
            sv = *cr;
          if (wmain)
            rp[lane] = sv;
          if (wtrail)
            rp[phi + jj] = val;
          if (wcarry)
            *cr = val;
        }
      });
      named_arrive(EMPTY0 + b, NT); // buffer b may be refilled
    }
  }
}

} // namespace ib200

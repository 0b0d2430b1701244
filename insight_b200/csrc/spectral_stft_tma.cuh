// spectral_stft_tma.cuh — STFT fast path for f32 segments of 2048 samples
// (nperseg == nfft == 2048, unit sample stride, no or DC-only detrend) into a
// complex64 (C, F, S) output whose bin rows are contiguous (segment stride 1,
// channel stride F * row stride) and whose base is 32-byte aligned.
//
// The transform is the same radix 16 * 16 * 8 Stockham FFT as the other fast
// paths (two consecutive segments a, b of one channel in one complex
// transform Z = FFT(w*a + i*w*b), w pre-scaled by 1/2), with three changes in
// how the work moves through the SM:
//   * the last pass runs mirrored butterflies: thread t of a group takes
//     butterfly j = 4*(t%32) + t/32 and its mirror 256 - j (0 and 128 for
//     j = 0), so it holds Z[k] and Z[L-k] of all its bins and unpacks
//     A[k] = Z[k] + conj Z[L-k], B[k] = -i (Z[k] - conj Z[L-k]) in registers;
//   * the unpacked columns go to a 64-byte-swizzled staging tile in shared
//     memory and leave by tiled TMA stores (cp.async.bulk.tensor, shared ->
//     this GPU's global memory, no multicast), instead of per-thread stores
//     from separate store warps;
//   * the next tile's samples are loaded into registers during the current
//     transform, and each group ping-pongs between two exchange buffers (two
//     group barriers a transform instead of four).
//
// Output tiling.  A tile is Q = 4 segment pairs (8 columns) of one channel.
// The row stride is odd for the usual shapes, so bin rows start at every
// 8-byte phase of a 32-byte sector.  Rows are split by R mod 4, R = c*F + k
// (row index over all channels): rows of one class lie 4 rows apart, a
// stride that is a multiple of 32 bytes, and share the phase d = (R * o_rs)
// mod 4.  One tensor map per class m describes those rows with the column
// origin moved back by d_m elements to the sector boundary, so a box of 8
// columns at tensor column x0 (the tile's first column) covers the whole
// sectors [x0 - d, x0 + 8 - d) of every row: the last d columns of a tile
// are carried in shared memory into the next tile's box (each value is
// carried by the thread that computed it), as in the sector-aligned stores
// of stft_ws_kernel.  Within a channel, bins k = q, q + 4, ..., q + 1020 of
// class q form one box of 256 rows; bin 1024 is stored directly.  Tiles are
// split evenly over the CTAs as one contiguous run each.  Values are stored
// directly (plain st.global) where a box cannot be used: a shifted class at
// the first tile of a run or channel (no carried columns), the columns
// carried out of a run's last tile, and the whole last tile of a channel
// (a box there would reach past the row end, and a TMA store bounds the
// innermost dimension in 16-byte chunks, so a row ending mid-chunk would
// have the next row's first value overwritten).  Every box lies inside its
// rows.
//
// Ordering, per tile: thread 0 waits until the previous tile's boxes have
// read the staging tile (cp.async.bulk.wait_group.read), a CTA barrier
// (EMPTY) releases the writers, each writer fences its shared-memory writes
// for the async proxy (fence.proxy.async.shared::cta), a CTA barrier (FULL)
// closes the tile and thread 0 issues its boxes.  All waits are hardware
// barriers or bulk-group waits; there are no spin loops.  (A dedicated TMA
// warp that decouples the groups from the stores was measured: its 17th warp
// caps every thread at 96 registers, the transform spills, and the kernel ran
// at 2.86 ms against 1.98 for this layout at the time.)
#pragma once
#include <cuda.h>
#include "spectral_stft_ws.cuh"

namespace ib200 {

struct StftTma {
  static constexpr int L = 2048, E = 16, P = L / E, G = 4;
  static constexpr int NT = G * P;       // threads (thread 0 also issues the boxes)
  static constexpr int F = L / 2 + 1;    // 1025 bins
  static constexpr int Q = G;            // segment pairs per tile
  static constexpr int W = 2 * Q;        // columns per tile
  static constexpr int ROWS = 256;       // rows of one class box
  static constexpr int BOX_BYTES = ROWS * W * 8;
  static constexpr int XS = spad_size(L);
  static constexpr size_t STG = 4 * (size_t)BOX_BYTES;
  static constexpr size_t XCH = (size_t)G * 2 * XS * sizeof(float2);
  static constexpr size_t CAR = 4 * (size_t)ROWS * 3 * sizeof(float2);
  static constexpr size_t SMEM = 1024 + STG + XCH + CAR; // 1024: alignment
  static constexpr int FULL = G + 1, EMPTY = G + 2;      // CTA barriers
};

struct StftTmaArgs {
  const float *x;       // channel 0, sample 0
  int64_t x_cs, step, seg0;
  int S;                // segments (columns) per channel
  int tpc;              // tiles per channel
  int ntiles;           // C * tpc
  const float *win;     // [2048]
  const float2 *tw;     // [2048], W_2048^m
  float2 *out;          // element (c, k, s) at out[c*o_cs + k*o_rs + s]
  int64_t o_cs, o_rs;
  int dc_mode;          // 0 none, 1 DC bin := 0
};

// Byte offset of (row i, column sc) in the 64-byte-swizzled box of class q:
// 16-byte chunk index XOR bits 7-8 of the row offset (CU_TENSOR_MAP_SWIZZLE_64B).
__device__ __forceinline__ uint32_t stma_off(int q, int i, int sc) {
  return (uint32_t)(q * StftTma::BOX_BYTES + i * 64 +
                    ((sc * 8) ^ (((i >> 1) & 3) << 4)));
}

__device__ __forceinline__ void tma_store_box(const CUtensorMap *m, uint32_t src,
                                              int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];"
      ::"l"(reinterpret_cast<uint64_t>(m)), "r"(src), "r"(x), "r"(y)
      : "memory");
}

// The tile's boxes: class q (bins k = q + 4i of channel c) from its staging
// box, except classes with carried columns at the first tile of a run, and
// none at a channel's last tile.  Every box lies inside its rows.
__device__ __forceinline__ void issue_boxes(
    const CUtensorMap *tm0, const CUtensorMap *tm1, const CUtensorMap *tm2,
    const CUtensorMap *tm3, uint32_t stg_s, int c, int tl, int tpc, bool first,
    int orp) {
  if (tl + 1 == tpc)
    return; // stored directly (see the writers)
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const int64_t R = (int64_t)c * StftTma::F + q;
    const int m = (int)(R & 3);
    const int d = (m * orp) & 3;
    if (first && d != 0)
      continue; // stored directly by the writers
    const CUtensorMap *tm = m == 0 ? tm0 : m == 1 ? tm1 : m == 2 ? tm2 : tm3;
    tma_store_box(tm, stg_s + q * StftTma::BOX_BYTES, (int)(2 * tl * StftTma::W),
                  (int)(R >> 2));
  }
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

template <int SH>
__global__ void __launch_bounds__(StftTma::NT, 1)
    stft_tma_kernel(const StftTmaArgs p, const __grid_constant__ CUtensorMap tm0,
                    const __grid_constant__ CUtensorMap tm1,
                    const __grid_constant__ CUtensorMap tm2,
                    const __grid_constant__ CUtensorMap tm3) {
  using K = StftTma;
  using V = float2;
  constexpr int L = K::L, E = K::E, P = K::P, F = K::F;
  // samples of segment b not shared with segment a (hop = SH * 128)
  constexpr int NB = SH > 0 ? SH : E;
  static_assert(SH >= 0 && SH < E, "overlap shift");
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const uint32_t sraw = (uint32_t)__cvta_generic_to_shared(smem_raw);
  const uint32_t pad = (1024u - (sraw & 1023u)) & 1023u;
  unsigned char *stg = smem_raw + pad;                       // [4][256][8] V
  V *xch = reinterpret_cast<V *>(stg + K::STG);              // [G][2][XS]
  V *car = reinterpret_cast<V *>(stg + K::STG + K::XCH);     // [4][256][3]
  const uint32_t stg_s = sraw + pad;

  const int fb = (int)((int64_t)blockIdx.x * p.ntiles / gridDim.x);
  const int fe = (int)((int64_t)(blockIdx.x + 1) * p.ntiles / gridDim.x);
  const int orp = (int)(p.o_rs & 3);
  constexpr int NT = K::NT;

  // ---------------------------------------------------------------- transforms
  const int g = threadIdx.x / P;
  const int t = threadIdx.x - g * P;
  const int w = t >> 5, l = t & 31;
  const int jb0 = 4 * l + w;                      // last-pass butterfly
  const int jb1 = jb0 == 0 ? 128 : 256 - jb0;     // and its mirror
  const bool t0 = jb0 == 0;
  const int q1 = w, q2 = (4 - w) & 3;             // classes of their bins
  const int i1 = l, i2 = jb1 >> 2;                // rows of their r = 0 bins
  V *bufA = xch + (2 * g) * K::XS;
  V *bufB = bufA + K::XS;
  V *car1 = car + q1 * K::ROWS * 3;
  V *car2 = car + q2 * K::ROWS * 3;

  float wv[E];
  static_for<0, E>([&](auto eIC) {
    constexpr int e = decltype(eIC)::value;
    wv[e] = 0.5f * __ldg(p.win + t + P * e);
  });
  const V tw1 = p.tw[(t & 15) * (L / 256)]; // pass 1: W_256^(t mod 16)
  const V twa = p.tw[jb0];                  // pass 2: W_2048^j
  const V twb = p.tw[jb1];

  float nx[E + NB]; // this tile's samples: segment a, then b's own
  // both segments of the pair exist (all but a channel's last pair or two)
  auto full_pair = [&](int tl) { return 2 * (tl * K::Q + g) + 1 < p.S; };
  auto load_tile = [&](int c, int tl) {
    const int task = tl * K::Q + g;
    const float *xa = p.x + c * p.x_cs + (p.seg0 + 2 * (int64_t)task) * p.step + t;
    if (full_pair(tl)) {
      static_for<0, E>([&](auto eIC) {
        constexpr int e = decltype(eIC)::value;
        nx[e] = __ldg(xa + P * e);
      });
      static_for<0, NB>([&](auto eIC) {
        constexpr int e = decltype(eIC)::value;
        nx[E + e] = __ldg(xa + p.step + P * (E - NB + e));
      });
    } else { // segment b (and maybe a) past the channel's last segment
      const bool va = 2 * task < p.S;
      static_for<0, E>([&](auto eIC) {
        constexpr int e = decltype(eIC)::value;
        nx[e] = va ? __ldg(xa + P * e) : 0.f;
      });
      static_for<0, NB>([&](auto eIC) {
        constexpr int e = decltype(eIC)::value;
        nx[E + e] = 0.f;
      });
    }
  };

  int c = fb / p.tpc, tl = fb - c * p.tpc;
  if (fb < fe)
    load_tile(c, tl);
  for (int f = fb; f < fe; ++f) {
    const bool first = f == fb || tl == 0;
    const bool last = f + 1 == fe || tl + 1 == p.tpc;
    const int x0 = tl * K::W;
    V v[E];
    if (full_pair(tl)) {
      static_for<0, E>([&](auto eIC) {
        constexpr int e = decltype(eIC)::value;
        float b;
        if constexpr (SH > 0 && e + SH < E)
          b = nx[e + SH];
        else
          b = nx[E + e - (E - NB)];
        v[e] = {nx[e] * wv[e], b * wv[e]};
      });
    } else { // segment b is zero
      static_for<0, E>([&](auto eIC) {
        constexpr int e = decltype(eIC)::value;
        v[e] = {nx[e] * wv[e], 0.f};
      });
    }
    // next tile of this run
    int cn = c, tn = tl + 1;
    if (tn == p.tpc) {
      tn = 0;
      ++cn;
    }
    if (f + 1 < fe)
      load_tile(cn, tn);

    // pass 0 (radix 16), pass 1 (radix 16), ping-pong exchanges
    dft_reg<float, 16>(v);
    pass_store<L, E, P, 0>(v, bufA, t);
    group_sync<K::G, P>(g);
    pass_load<L, E, P, 1>(v, bufA, t);
    apply_twiddles<16>(v, tw1);
    dft_reg<float, 16>(v);
    pass_store<L, E, P, 1>(v, bufB, t);
    group_sync<K::G, P>(g);
    // pass 2 (radix 8) on butterflies jb0 (v[0..7]) and jb1 (v[8..15])
    static_for<0, 8>([&](auto rIC) {
      constexpr int r = decltype(rIC)::value;
      v[r] = bufB[spad(jb0) + pad_off<r * 256>()];
      v[8 + r] = bufB[spad(jb1) + pad_off<r * 256>()];
    });
    apply_twiddles<8>(v, twa);
    dft_reg<float, 8>(v);
    apply_twiddles<8>(v + 8, twb);
    dft_reg<float, 8>(v + 8);
    // bin jb + 256 r of butterfly b is v[8 b + bitrev8(r)]
    if (p.dc_mode == 1 && t0)
      v[0] = {0.f, 0.f};

    // unpack: bins jb0 + 256 r and jb1 + 256 r, r = 0..3
    V A1[4], B1[4], A2[4], B2[4];
    static_for<0, 4>([&](auto rIC) {
      constexpr int r = decltype(rIC)::value;
      const V zk1 = v[bitrev<8>(r)];
      const V m1g = v[8 + bitrev<8>(7 - r)];      // Z[L-k] in the mirror
      const V m1s = v[bitrev<8>((8 - r) & 7)];    // j = 0: in butterfly 0
      const V zm1 = t0 ? m1s : m1g;
      const V zk2 = v[8 + bitrev<8>(r)];
      const V m2g = v[bitrev<8>(7 - r)];
      const V m2s = v[8 + bitrev<8>(7 - r)];      // j = 0: 128 mirrors itself
      const V zm2 = t0 ? m2s : m2g;
      A1[r] = {zk1.x + zm1.x, zk1.y - zm1.y};
      B1[r] = {zk1.y + zm1.y, zm1.x - zk1.x};
      A2[r] = {zk2.x + zm2.x, zk2.y - zm2.y};
      B2[r] = {zk2.y + zm2.y, zm2.x - zk2.x};
    });

    // thread 0 issued the previous tile's boxes: it waits until they have
    // read stg, then the CTA barrier releases everyone's writes
    if (threadIdx.x == 0)
      asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
    named_sync(K::EMPTY, NT);
    // phase of class q's rows in this channel: ((c*F + q) * o_rs) mod 4
    const int cf4 = (int)(((int64_t)c * F) & 3);
    const int d1 = (((cf4 + q1) & 3) * orp) & 3;
    const int d2 = (((cf4 + q2) & 3) * orp) & 3;
    if (!first && !last) {
      // ------------------------------------------- common tile: staging only
      // class q, rows i + 64 r: byte offsets rb + 4096 r; carry slots
      // cr[i*3 + s] + 192 r
      auto stage = [&](int q, int i, V *cr, int d, const V *A, const V *B) {
        const int sA = 2 * g + d;
        const int rb = q * K::BOX_BYTES + i * 64;
        const int sw = ((i >> 1) & 3) << 4;
        V *c0 = cr + i * 3;
        if (sA + 1 < K::W) {
          const int oA = rb + ((8 * sA) ^ sw);
          if ((sA & 1) == 0) {
            static_for<0, 4>([&](auto rIC) {
              constexpr int r = decltype(rIC)::value;
              *reinterpret_cast<float4 *>(stg + oA + 4096 * r) =
                  make_float4(A[r].x, A[r].y, B[r].x, B[r].y);
            });
          } else {
            const int oB = rb + ((8 * sA + 8) ^ sw);
            static_for<0, 4>([&](auto rIC) {
              constexpr int r = decltype(rIC)::value;
              *reinterpret_cast<V *>(stg + oA + 4096 * r) = A[r];
              *reinterpret_cast<V *>(stg + oB + 4096 * r) = B[r];
            });
          }
        } else if (sA < K::W) { // A in column 7, B carried into column 0
          const int oA = rb + ((8 * sA) ^ sw);
          const int o0 = rb + sw;
          static_for<0, 4>([&](auto rIC) {
            constexpr int r = decltype(rIC)::value;
            *reinterpret_cast<V *>(stg + oA + 4096 * r) = A[r];
            *reinterpret_cast<V *>(stg + o0 + 4096 * r) = c0[192 * r];
            c0[192 * r] = B[r];
          });
        } else { // both carried: slots s0, s0 + 1 (columns s0, s0 + 1)
          const int s0 = sA - K::W;
          const int oa = rb + ((8 * s0) ^ sw);
          const int ob = rb + ((8 * s0 + 8) ^ sw);
          static_for<0, 4>([&](auto rIC) {
            constexpr int r = decltype(rIC)::value;
            *reinterpret_cast<V *>(stg + oa + 4096 * r) = c0[192 * r + s0];
            *reinterpret_cast<V *>(stg + ob + 4096 * r) = c0[192 * r + s0 + 1];
            c0[192 * r + s0] = A[r];
            c0[192 * r + s0 + 1] = B[r];
          });
        }
      };
      stage(q1, i1, car1, d1, A1, B1);
      stage(q2, i2, car2, d2, A2, B2);
      if (t0) { // bin 1024 (outside the class boxes): Z[1024] mirrors itself
        const V z = v[bitrev<8>(4)];
        V *gp = p.out + c * p.o_cs + (int64_t)(L / 2) * p.o_rs + x0 + 2 * g;
        gp[0] = V{z.x + z.x, 0.f};
        gp[1] = V{z.y + z.y, 0.f};
      }
    } else {
      // ------------- first or last tile of a run or channel: general stores
      V *outc = p.out + c * p.o_cs + x0 + 2 * g;
      const bool okA = x0 + 2 * g < p.S, okB = x0 + 2 * g + 1 < p.S;
      const bool nobox = tl + 1 == p.tpc; // a channel's last tile: no boxes
      // one bin (class q, row i, bin k) of this thread's two columns
      auto put = [&](int q, int d, V *cr, int i, int k, V A, V B) {
        const int sA = 2 * g + d; // staging column of A (B at sA + 1)
        V *gp = outc + (int64_t)k * p.o_rs;
        const bool dir = nobox || (first && d != 0);
        if (sA + 1 < K::W) {
          if (dir) {
            if (okA)
              gp[0] = A;
            if (okB)
              gp[1] = B;
          } else if ((sA & 1) == 0) {
            *reinterpret_cast<float4 *>(stg + stma_off(q, i, sA)) =
                make_float4(A.x, A.y, B.x, B.y);
          } else {
            *reinterpret_cast<V *>(stg + stma_off(q, i, sA)) = A;
            *reinterpret_cast<V *>(stg + stma_off(q, i, sA + 1)) = B;
          }
        } else if (sA < K::W) { // B is carried (slot 0)
          if (dir) {
            if (okA)
              gp[0] = A;
          } else {
            *reinterpret_cast<V *>(stg + stma_off(q, i, sA)) = A;
          }
          if (!first) { // the previous tile's B of this thread
            if (nobox)
              gp[1 - K::W] = cr[i * 3];
            else
              *reinterpret_cast<V *>(stg + stma_off(q, i, 0)) = cr[i * 3];
          }
          if (last) {
            if (okB)
              gp[1] = B;
          } else {
            cr[i * 3] = B;
          }
        } else { // both carried (slots sA - 8, sA - 7)
          const int s0 = sA - K::W;
          if (!first) {
            if (nobox) {
              gp[-K::W] = cr[i * 3 + s0];
              gp[1 - K::W] = cr[i * 3 + s0 + 1];
            } else {
              *reinterpret_cast<V *>(stg + stma_off(q, i, s0)) = cr[i * 3 + s0];
              *reinterpret_cast<V *>(stg + stma_off(q, i, s0 + 1)) =
                  cr[i * 3 + s0 + 1];
            }
          }
          if (last) {
            if (okA)
              gp[0] = A;
            if (okB)
              gp[1] = B;
          } else {
            cr[i * 3 + s0] = A;
            cr[i * 3 + s0 + 1] = B;
          }
        }
      };
      static_for<0, 4>([&](auto rIC) {
        constexpr int r = decltype(rIC)::value;
        put(q1, d1, car1, i1 + 64 * r, jb0 + 256 * r, A1[r], B1[r]);
        put(q2, d2, car2, i2 + 64 * r, jb1 + 256 * r, A2[r], B2[r]);
      });
      if (t0) { // bin 1024 (outside the class boxes): Z[1024] mirrors itself
        const V z = v[bitrev<8>(4)];
        V *gp = outc + (int64_t)(L / 2) * p.o_rs;
        if (okA)
          gp[0] = V{z.x + z.x, 0.f};
        if (okB)
          gp[1] = V{z.y + z.y, 0.f};
      }
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    named_sync(K::FULL, NT); // every write of the tile is in stg
    if (threadIdx.x == 0)
      issue_boxes(&tm0, &tm1, &tm2, &tm3, stg_s, c, tl, p.tpc, first, orp);
    c = cn;
    tl = tn;
  }
  if (threadIdx.x == 0) // the boxes' writes complete before the kernel ends
    asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

} // namespace ib200

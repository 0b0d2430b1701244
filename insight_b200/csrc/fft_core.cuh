// fft_core.cuh — register/shared-memory Stockham FFT building blocks for the
// fused spectral kernels (sm_100a).
//
// A transform of length L is computed by one "group" of P threads.  Each
// thread keeps E = L / P complex values in registers.  The transform runs as
// a sequence of Stockham autosort passes (radix R_p = min(E, L / Ns_p), Ns the
// product of the previous radices).  Pass p, butterfly j (0 <= j < L/R):
//     k    = j mod Ns
//     a[r] = data[j + r*L/R] * W_{Ns*R}^{r*k}          r = 0..R-1
//     A    = DFT_R(a)                                 (in registers)
//     data'[(j/Ns)*Ns*R + k + r*Ns] = A[r]
// with W_N = exp(-2*pi*i/N) (the forward, unnormalised DFT that FFTW_FORWARD
// and numpy.fft.fft compute).  After the last pass data' is the DFT in
// natural order.  Between passes the values go through a padded shared-memory
// buffer (one pad slot every 16 values keeps the strided writes of the first
// pass bank-conflict free).  Each thread owns B = E/R butterflies per pass,
// j = t + b*P.  The R-point DFTs are radix-2 decimation-in-frequency networks
// unrolled at compile time; their twiddles are compile-time constants
// (cos(2*pi*m/32), m = 0..31, R <= 32).  Stockham twiddles W_{Ns*R}^{r*k}
// are formed per butterfly from one table value W_{Ns*R}^k by binary
// splitting (W^r = W^{r/2} * W^{r-r/2}), so each power is at most log2(R)
// rounded products away from the table value.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>
#include <type_traits>

namespace ib200 {

template <typename T> struct V2T;
template <> struct V2T<float> { using type = float2; };
template <> struct V2T<double> { using type = double2; };

template <typename V> __device__ __forceinline__ V vadd(V a, V b) {
  return {a.x + b.x, a.y + b.y};
}
template <typename V> __device__ __forceinline__ V vsub(V a, V b) {
  return {a.x - b.x, a.y - b.y};
}
// PK: f32 complex adds and subtracts as one packed two-lane instruction each
// (sm_100 FADD2 / FFMA2: half the issue slots of two scalar ones, each lane
// rounded as the scalar operation; a - b is fma(b, -1, a), exact before its
// one rounding).  The butterfly networks of the transforms are mostly these.
// Whether it pays depends on the kernel (measured: csd 5.27 -> 4.85 ms, the
// stft kernel 1.56 -> 1.62 ms), so each kernel chooses.
template <bool PK, typename V> __device__ __forceinline__ V vadd_k(V a, V b) {
  if constexpr (PK && std::is_same<V, float2>::value)
    return __fadd2_rn(a, b);
  else
    return vadd(a, b);
}
template <bool PK, typename V> __device__ __forceinline__ V vsub_k(V a, V b) {
  if constexpr (PK && std::is_same<V, float2>::value)
    return __ffma2_rn(b, make_float2(-1.f, -1.f), a);
  else
    return vsub(a, b);
}
// a * b (complex)
template <typename V> __device__ __forceinline__ V vmul(V a, V b) {
  return {fma(a.x, b.x, -a.y * b.y), fma(a.x, b.y, a.y * b.x)};
}
// conj(a) * b
template <typename V> __device__ __forceinline__ V vcmul(V a, V b) {
  return {fma(a.x, b.x, a.y * b.y), fma(a.x, b.y, -a.y * b.x)};
}

// cos(2*pi*m/32) for m in [0, 32).
__host__ __device__ constexpr double cos32(int m) {
  switch (m & 31) {
  case 0: return 1.0;
  case 1: return 0.98078528040323043;
  case 2: return 0.92387953251128674;
  case 3: return 0.83146961230254524;
  case 4: return 0.70710678118654757;
  case 5: return 0.55557023301960229;
  case 6: return 0.38268343236508984;
  case 7: return 0.19509032201612833;
  case 8: return 0.0;
  case 9: return -0.19509032201612833;
  case 10: return -0.38268343236508984;
  case 11: return -0.55557023301960229;
  case 12: return -0.70710678118654757;
  case 13: return -0.83146961230254524;
  case 14: return -0.92387953251128674;
  case 15: return -0.98078528040323043;
  case 16: return -1.0;
  case 17: return -0.98078528040323043;
  case 18: return -0.92387953251128674;
  case 19: return -0.83146961230254524;
  case 20: return -0.70710678118654757;
  case 21: return -0.55557023301960229;
  case 22: return -0.38268343236508984;
  case 23: return -0.19509032201612833;
  case 24: return 0.0;
  case 25: return 0.19509032201612833;
  case 26: return 0.38268343236508984;
  case 27: return 0.55557023301960229;
  case 28: return 0.70710678118654757;
  case 29: return 0.83146961230254524;
  case 30: return 0.92387953251128674;
  default: return 0.98078528040323043;
  }
}

// v * W_32^Q, W_32 = exp(-2*pi*i/32).  Multiples of a quarter turn are exact.
template <typename T, int Q, typename V>
__device__ __forceinline__ V mul_w32(V v) {
  constexpr int q = Q & 31;
  if constexpr (q == 0) {
    return v;
  } else if constexpr (q == 8) {
    return {v.y, -v.x};
  } else if constexpr (q == 16) {
    return {-v.x, -v.y};
  } else if constexpr (q == 24) {
    return {-v.y, v.x};
  } else {
    constexpr T c = (T)cos32(q);
    constexpr T s = (T)cos32(q + 24); // sin(2*pi*q/32)
    // (x + iy)(c - is) = (xc + ys) + i(yc - xs)
    return {fma(v.x, c, v.y * s), fma(v.y, c, -(v.x * s))};
  }
}

template <int I> using IC = std::integral_constant<int, I>;

template <int B, int E, int S = 1, typename F>
__device__ __forceinline__ void static_for(F &&f) {
  if constexpr (B < E) {
    f(IC<B>{});
    static_for<B + S, E, S>(f);
  }
}

// Fills entries [0, n) (store(i, load(i))) with `nthreads` threads, each
// with BATCH independent loads in flight before their stores.  A plain
// load-then-store loop waits one memory latency per entry, which is what
// dominates a kernel prologue that fills tables before a short run of work.
template <int BATCH, typename Ld, typename St>
__device__ __forceinline__ void fill_batched(int tid, int n, int nthreads,
                                             Ld &&load, St &&store) {
  using X = decltype(load(0));
  for (int i0 = tid; i0 < n; i0 += BATCH * nthreads) {
    X v[BATCH];
#pragma unroll
    for (int q = 0; q < BATCH; ++q) {
      const int i = i0 + q * nthreads;
      if (i < n)
        v[q] = load(i);
    }
#pragma unroll
    for (int q = 0; q < BATCH; ++q) {
      const int i = i0 + q * nthreads;
      if (i < n)
        store(i, v[q]);
    }
  }
}

template <int R> __host__ __device__ constexpr int bitrev(int v) {
  int r = 0;
  for (int m = R >> 1, b = 1; m >= 1; m >>= 1, b <<= 1)
    if (v & m)
      r |= b;
  return r;
}

// In-register R-point forward DFT: natural-order input, output in
// bit-reversed register order (a[i] = X[bitrev(i)]); consumers index with
// bitrev<R>() at compile time instead of moving registers.
template <typename T, int R, bool PK = false, typename V>
__device__ __forceinline__ void dft_reg(V *a) {
  static_assert(R >= 1 && R <= 32 && (R & (R - 1)) == 0, "radix");
  if constexpr (R > 1) {
    // radix-2 DIF network: span H = R/2, R/4, ..., 1
    constexpr int STAGES = R == 2 ? 1 : R == 4 ? 2 : R == 8 ? 3 : R == 16 ? 4 : 5;
    static_for<0, STAGES>([&](auto sIC) {
      constexpr int s = decltype(sIC)::value;
      constexpr int H = R >> (s + 1);
      if constexpr (H >= 1) {
        static_for<0, R, 2 * H>([&](auto bIC) {
          constexpr int blk = decltype(bIC)::value;
          static_for<0, H>([&](auto iIC) {
            constexpr int i = decltype(iIC)::value;
            V u = a[blk + i], w = a[blk + i + H];
            a[blk + i] = vadd_k<PK>(u, w);
            a[blk + i + H] = mul_w32<T, i * (32 / (2 * H))>(vsub_k<PK>(u, w));
          });
        });
      }
    });
  }
}

// Multiply a[1..R-1] by W^r given W = w1, using binary splitting.
template <int R, typename V>
__device__ __forceinline__ void apply_twiddles(V *a, V w1) {
  if constexpr (R > 1) {
    V w[R];
    w[1] = w1;
    static_for<2, R>([&](auto rIC) {
      constexpr int r = decltype(rIC)::value;
      w[r] = vmul(w[r / 2], w[r - r / 2]);
    });
    static_for<1, R>([&](auto rIC) {
      constexpr int r = decltype(rIC)::value;
      a[r] = vmul(a[r], w[r]);
    });
  }
}

// Padded shared-memory index: one spare slot every 16 values.
__device__ __forceinline__ int spad(int i) { return i + (i >> 4); }
__host__ __device__ constexpr int spad_size(int L) { return L + (L >> 4); }

// Compile-time pass plan: radix of pass p and the product of earlier radices.
template <int L, int E> struct Plan {
  __host__ __device__ static constexpr int radix(int p) {
    int ns = 1;
    for (int i = 0; i < p; ++i) {
      int r = (L / ns) < E ? (L / ns) : E;
      ns *= r;
    }
    return (L / ns) < E ? (L / ns) : E;
  }
  __host__ __device__ static constexpr int ns(int p) {
    int ns = 1;
    for (int i = 0; i < p; ++i)
      ns *= radix(i);
    return ns;
  }
  __host__ __device__ static constexpr int passes() {
    int n = 0, ns = 1;
    while (ns < L) {
      ns *= radix(n);
      ++n;
    }
    return n;
  }
};

// Group barrier: the P threads of group g (named barrier g+1), or the whole
// CTA when the CTA holds a single group.
template <int G, int P> __device__ __forceinline__ void group_sync(int g) {
  if constexpr (G == 1) {
    __syncthreads();
  } else {
    asm volatile("bar.sync %0, %1;" ::"r"(g + 1), "r"(P) : "memory");
  }
}

// One Stockham pass reading `v` (registers: butterfly b, element r at
// v[b*R + r]) that were loaded for this pass, applying twiddles and the
// R-point DFTs in place.  Index bookkeeping for the surrounding exchange is
// done by the callers.
template <typename T, int L, int E, int P, int PASS, typename V>
__device__ __forceinline__ void pass_compute(V *v, int t, const V *tw) {
  using PL = Plan<L, E>;
  constexpr int R = PL::radix(PASS);
  constexpr int NS = PL::ns(PASS);
  constexpr int B = E / R;
  static_for<0, B>([&](auto bIC) {
    constexpr int b = decltype(bIC)::value;
    if constexpr (NS > 1) {
      const int j = t + b * P;
      const int k = j & (NS - 1);
      // W_{NS*R}^k = W_L^{k * L/(NS*R)}
      const V w1 = tw[k * (L / (NS * R))];
      apply_twiddles<R>(v + b * R, w1);
    }
    dft_reg<T, R>(v + b * R);
  });
}

// Padded offset of a compile-time distance D from an index whose padding is
// already accounted for: valid when D is a multiple of 16.
template <int D> __host__ __device__ constexpr int pad_off() {
  static_assert(D % 16 == 0, "padded offsets need multiples of 16");
  return D + D / 16;
}

// Write the outputs of pass PASS to shared memory.  Element r of butterfly j
// goes to base + r*NS; with NS == 1 the base is a multiple of R <= 16 so the
// whole run shares one pad slot, with NS % 16 == 0 every step is D = NS.
template <int L, int E, int P, int PASS, typename V>
__device__ __forceinline__ void pass_store(const V *v, V *buf, int t) {
  using PL = Plan<L, E>;
  constexpr int R = PL::radix(PASS);
  constexpr int NS = PL::ns(PASS);
  constexpr int B = E / R;
  static_for<0, B>([&](auto bIC) {
    constexpr int b = decltype(bIC)::value;
    const int j = t + b * P;
    const int k = j & (NS - 1);
    const int base = (j / NS) * NS * R + k;
    if constexpr (NS == 1 && R <= 16) {
      V *q = buf + spad(base);
      static_for<0, R>([&](auto rIC) {
        constexpr int r = decltype(rIC)::value;
        q[r] = v[b * R + bitrev<R>(r)];
      });
    } else if constexpr (NS % 16 == 0) {
      V *q = buf + spad(base);
      static_for<0, R>([&](auto rIC) {
        constexpr int r = decltype(rIC)::value;
        q[pad_off<r * NS>()] = v[b * R + bitrev<R>(r)];
      });
    } else {
      static_for<0, R>([&](auto rIC) {
        constexpr int r = decltype(rIC)::value;
        buf[spad(base + r * NS)] = v[b * R + bitrev<R>(r)];
      });
    }
  });
}

// Read the inputs of pass PASS from shared memory (stride L/R).
template <int L, int E, int P, int PASS, typename V>
__device__ __forceinline__ void pass_load(V *v, const V *buf, int t) {
  using PL = Plan<L, E>;
  constexpr int R = PL::radix(PASS);
  constexpr int B = E / R;
  static_for<0, B>([&](auto bIC) {
    constexpr int b = decltype(bIC)::value;
    const int j = t + b * P;
    if constexpr ((L / R) % 16 == 0) {
      const V *q = buf + spad(j);
      static_for<0, R>([&](auto rIC) {
        constexpr int r = decltype(rIC)::value;
        v[b * R + r] = q[pad_off<r * (L / R)>()];
      });
    } else {
      static_for<0, R>([&](auto rIC) {
        constexpr int r = decltype(rIC)::value;
        v[b * R + r] = buf[spad(j + r * (L / R))];
      });
    }
  });
}

// Write the transform (natural order, as left by fft_group) to shared memory.
template <int L, int E, int P, typename V>
__device__ __forceinline__ void store_bins(const V *v, V *buf, int t) {
  constexpr int R = Plan<L, E>::radix(Plan<L, E>::passes() - 1);
  constexpr int B = E / R;
  static_for<0, B>([&](auto bIC) {
    constexpr int b = decltype(bIC)::value;
    const int j = t + b * P;
    if constexpr ((L / R) % 16 == 0) {
      V *q = buf + spad(j);
      static_for<0, R>([&](auto rIC) {
        constexpr int r = decltype(rIC)::value;
        q[pad_off<r * (L / R)>()] = v[b * R + bitrev<R>(r)];
      });
    } else {
      static_for<0, R>([&](auto rIC) {
        constexpr int r = decltype(rIC)::value;
        buf[spad(j + r * (L / R))] = v[b * R + bitrev<R>(r)];
      });
    }
  });
}

// Per-thread Stockham twiddles.  A thread's butterflies j = t + b*P have the
// same k = j mod NS in every transform, so the R-1 factors W_{NS*R}^{r*k} of
// each pass p >= 1 are loop invariant.  They are read once per CTA from the
// W_L table into a shared-memory row per thread: butterfly (p, b) owns R
// slots (r = 1..R-1 and one pad) at offset(p) + b*R, so every pair of slots
// is 16-byte aligned.  Row strides keep 128-bit reads bank-conflict free.
template <typename T, int L, int E> struct ThreadTw {
  using PL = Plan<L, E>;
  __host__ __device__ static constexpr int block(int p) {
    return (E / PL::radix(p)) * PL::radix(p);
  }
  __host__ __device__ static constexpr int offset(int p) {
    int o = 0;
    for (int q = 1; q < p; ++q)
      o += block(q);
    return o;
  }
  __host__ __device__ static constexpr int total() {
    return offset(PL::passes());
  }
  __host__ __device__ static constexpr int stride() {
    // f32 entries are 8 bytes: stride = 2 (mod 4) keeps eight 16-byte lanes
    // on distinct bank quads; f64 entries are 16 bytes: an odd stride.
    if (sizeof(T) == 4) {
      int s = total() + 2;
      while (s % 4 != 2)
        ++s;
      return s;
    }
    return total() | 1;
  }
};

template <typename T, int L, int E, int P, typename V>
__device__ __forceinline__ void fill_thread_twiddles(V *tws, const V *tw,
                                                     int tid, int nthreads) {
  using PL = Plan<L, E>;
  using TT = ThreadTw<T, L, E>;
  constexpr int NPASS = PL::passes();
  auto load = [&](int i) -> V {
    const int tt = i / TT::total();
    int slot = i - tt * TT::total();
    V val = {T(1), T(0)};
    static_for<1, NPASS>([&](auto pIC) {
      constexpr int p = decltype(pIC)::value;
      constexpr int R = PL::radix(p);
      constexpr int NS = PL::ns(p);
      if (slot >= TT::offset(p) && slot < TT::offset(p) + TT::block(p)) {
        const int rel = slot - TT::offset(p);
        const int b = rel / R;
        const int r = rel - b * R + 1; // slot R-1 of a butterfly is padding
        if (r < R) {
          const int k = (tt + b * P) & (NS - 1);
          val = tw[((int64_t)r * k * (L / (NS * R))) % L];
        }
      }
    });
    return val;
  };
  fill_batched<8>(tid, P * TT::total(), nthreads, load, [&](int i, V v) {
    const int tt = i / TT::total();
    tws[tt * TT::stride() + (i - tt * TT::total())] = v;
  });
}

// Per-thread rows of only the first twiddle W^k of every butterfly of the
// passes after the first (the powers W^{rk} then follow by binary splitting,
// as with the global table): the light table for lengths whose full rows do
// not fit in shared memory.  An odd stride keeps the rows of a warp on
// distinct banks.
template <typename T, int L, int E> struct ThreadTw1 {
  using PL = Plan<L, E>;
  __host__ __device__ static constexpr int offset(int p) {
    int o = 0;
    for (int q = 1; q < p; ++q)
      o += E / PL::radix(q);
    return o;
  }
  __host__ __device__ static constexpr int total() {
    return offset(PL::passes());
  }
  __host__ __device__ static constexpr int stride() { return total() | 1; }
};

// Shape condition of the warp-shuffle last pass (fft_group_w1_lastshfl):
// last radix 2, one radix-E butterfly per thread in the pass before it.
template <int L, int E> struct LastShfl {
  using PL = Plan<L, E>;
  static constexpr int NP = PL::passes();
  static constexpr int RP = PL::radix(NP - 2);  // radix of the pass before
  static constexpr int NSP = PL::ns(NP - 2);
  static constexpr bool ok = NP >= 2 && PL::radix(NP - 1) == 2 && RP == E &&
                             NSP * RP == L / 2 && NSP % 16 == 0 &&
                             (L / E) % 32 == 0;
};

// Lane l of warp w takes butterfly m + h*NSP with h = bit 4 of l and
// m = 16 w + (l & 15): partners are 16 lanes apart (one exchange over lane
// bit 4), and each half-warp reads 16 consecutive butterflies, so the 8-byte
// shared-memory loads of a half-warp fall on 16 distinct bank pairs.
__host__ __device__ constexpr int shfl_half(int t) { return (t >> 4) & 1; }
__host__ __device__ constexpr int shfl_m(int t) { return (t >> 5) * 16 + (t & 15); }

template <int L, int E>
__host__ __device__ constexpr int shfl_j(int t) {
  return shfl_half(t) * LastShfl<L, E>::NSP + shfl_m(t);
}

template <int L, int E>
__host__ __device__ constexpr int shfl_bin(int t, int e) {
  return shfl_half(t) * (L / 2) + shfl_m(t) + LastShfl<L, E>::NSP * bitrev<E>(e);
}

// Mirrored butterfly assignment of the last pass.  Butterfly j of the last
// pass (radix R, NS = L/R) yields bins j + NS*r, whose mirrors L - bin are
// the bins of butterfly NS - j (element R-1-r), or of j itself for j = 0
// and j = NS/2.  With B = E/R >= 2 butterflies per thread, thread t takes
// j = t + b*P for b < B/2 and the mirror of each for b >= B/2 (NS/2 in place
// of the mirror of 0), so it holds both Z[k] and Z[L-k] of all its bins.
template <int L, int E, int P>
__host__ __device__ constexpr int pair_j(int t, int b) {
  using PL = Plan<L, E>;
  constexpr int R = PL::radix(PL::passes() - 1);
  constexpr int NS = L / R, H = E / R / 2;
  if (b < H)
    return t + b * P;
  const int j = t + (b - H) * P;
  return j == 0 ? NS / 2 : NS - j;
}

template <typename T, int L, int E, int P, typename V, bool PAIRS = false,
          bool SHFL = false>
__device__ __forceinline__ void fill_thread_w1(V *rows, const V *tw, int tid,
                                               int nthreads) {
  using PL = Plan<L, E>;
  using TT = ThreadTw1<T, L, E>;
  constexpr int NPASS = PL::passes();
  auto load = [&](int i) -> V {
    const int tt = i / TT::total();
    const int slot = i - tt * TT::total();
    V val = {T(1), T(0)};
    static_for<1, NPASS>([&](auto pIC) {
      constexpr int p = decltype(pIC)::value;
      constexpr int R = PL::radix(p);
      constexpr int NS = PL::ns(p);
      if (slot >= TT::offset(p) && slot < TT::offset(p + 1)) {
        const int b = slot - TT::offset(p);
        int j;
        if constexpr (PAIRS && p == NPASS - 1)
          j = pair_j<L, E, P>(tt, b);
        else if constexpr (SHFL && p == NPASS - 2)
          j = shfl_j<L, E>(tt);
        else if constexpr (SHFL && p == NPASS - 1)
          j = shfl_m(tt); // the shuffle pass uses W_L^m from slot 0
        else
          j = tt + b * P;
        const int k = j & (NS - 1);
        val = tw[k * (L / (NS * R))];
      }
    });
    return val;
  };
  fill_batched<8>(tid, P * TT::total(), nthreads, load, [&](int i, V v) {
    const int tt = i / TT::total();
    rows[tt * TT::stride() + (i - tt * TT::total())] = v;
  });
}

template <typename T, int L, int E, int P, int PASS, bool PK = false, typename V>
__device__ __forceinline__ void pass_compute_w1(V *v, const V *row1) {
  using PL = Plan<L, E>;
  using TT = ThreadTw1<T, L, E>;
  constexpr int R = PL::radix(PASS);
  constexpr int NS = PL::ns(PASS);
  constexpr int B = E / R;
  static_for<0, B>([&](auto bIC) {
    constexpr int b = decltype(bIC)::value;
    if constexpr (NS > 1)
      apply_twiddles<R>(v + b * R, row1[TT::offset(PASS) + b]);
    dft_reg<T, R, PK>(v + b * R);
  });
}

// fft_group with the per-thread first-twiddle rows (row1 = this thread's).
template <typename T, int L, int E, int P, int G, typename V>
__device__ __forceinline__ void fft_group_w1(V *v, V *buf, int t, int g,
                                             const V *row1) {
  constexpr int NP = Plan<L, E>::passes();
  static_for<0, NP>([&](auto pIC) {
    constexpr int p = decltype(pIC)::value;
    if constexpr (p > 0) {
      pass_load<L, E, P, p>(v, buf, t);
      group_sync<G, P>(g);
    }
    pass_compute_w1<T, L, E, P, p>(v, row1);
    if constexpr (p + 1 < NP) {
      pass_store<L, E, P, p>(v, buf, t);
      group_sync<G, P>(g);
    }
  });
}

// fft_group_w1 whose last pass runs the mirrored butterflies of pair_j (the
// rows must come from fill_thread_w1<..., true>).  The transform is left in
// registers: element r of butterfly b, bin pair_j(t, b) + r*L/R, at
// v[b*R + bitrev(r)].
template <typename T, int L, int E, int P, int G, bool PK = false, typename V>
__device__ __forceinline__ void fft_group_w1_pairs(V *v, V *buf, int t, int g,
                                                   const V *row1) {
  using PL = Plan<L, E>;
  constexpr int NP = PL::passes();
  constexpr int RL = PL::radix(NP - 1);
  constexpr int BL = E / RL;
  static_assert(NP >= 2 && BL >= 2, "mirrored pairs need two butterflies");
  static_for<0, NP>([&](auto pIC) {
    constexpr int p = decltype(pIC)::value;
    if constexpr (p > 0 && p + 1 < NP) {
      pass_load<L, E, P, p>(v, buf, t);
      group_sync<G, P>(g);
    } else if constexpr (p > 0) {
      static_for<0, BL>([&](auto bIC) {
        constexpr int b = decltype(bIC)::value;
        const int j = pair_j<L, E, P>(t, b);
        static_for<0, RL>([&](auto rIC) {
          constexpr int r = decltype(rIC)::value;
          if constexpr ((L / RL) % 16 == 0)
            v[b * RL + r] = buf[spad(j) + pad_off<r * (L / RL)>()];
          else
            v[b * RL + r] = buf[spad(j + r * (L / RL))];
        });
      });
      group_sync<G, P>(g);
    }
    pass_compute_w1<T, L, E, P, p, PK>(v, row1);
    if constexpr (p + 1 < NP) {
      pass_store<L, E, P, p>(v, buf, t);
      group_sync<G, P>(g);
    }
  });
}

// Last pass on warp shuffles.  When the last radix is 2 and the pass before
// it gives every thread one butterfly (radix E, L/E = P butterflies, whose
// outputs lie NS*E = L/2 apart for butterflies j and j + NS), thread t takes
// butterfly shfl_j(t) = h*NS + m of that pass (h, m: shfl_half, shfl_m):
// the two lanes with the same m then hold the outputs m + NS*r and
// L/2 + m + NS*r, the two inputs of a radix-2 butterfly of the last pass, in
// the same register r.  The last pass is one exchange between those lanes
// (__shfl_xor_sync over lane bit 4) instead of a shared-memory round trip and
// a group barrier:
//   X[j] = a + w b,  X[j + L/2] = a - w b,   j = m + NS*r,  w = W_L^j,
// where the h = 1 lane forms w b with w = W_L^m W_{2E}^r (W_L^{NS} = W_{2E})
// and both lanes swap their values.  After it, register e of thread t holds
// bin shfl_bin(t, e).  The twiddle rows come from fill_thread_w1 with SHFL =
// true (the pass before the last holds W^k of butterfly shfl_j(t), the last
// pass W_L^m in its first slot).  A group must be whole warps.
template <typename T, int L, int E, int P, int G, typename V>
__device__ __forceinline__ void fft_group_w1_lastshfl(V *v, V *buf, int t, int g,
                                                      const V *row1) {
  using PL = Plan<L, E>;
  using LS = LastShfl<L, E>;
  using TT = ThreadTw1<T, L, E>;
  constexpr int NP = LS::NP;
  constexpr int NSP = LS::NSP;
  static_assert(LS::ok && P == L / E, "shuffle last pass");
  static_for<0, NP - 1>([&](auto pIC) {
    constexpr int p = decltype(pIC)::value;
    if constexpr (p > 0 && p < NP - 2) {
      pass_load<L, E, P, p>(v, buf, t);
      group_sync<G, P>(g);
    } else if constexpr (p > 0) { // p == NP - 2: butterfly shfl_j(t)
      const int j = shfl_j<L, E>(t);
      static_for<0, E>([&](auto rIC) {
        constexpr int r = decltype(rIC)::value;
        if constexpr ((L / E) % 16 == 0)
          v[r] = buf[spad(j) + pad_off<r * (L / E)>()];
        else
          v[r] = buf[spad(j + r * (L / E))];
      });
      group_sync<G, P>(g);
    }
    pass_compute_w1<T, L, E, P, p>(v, row1);
    if constexpr (p + 2 < NP) {
      pass_store<L, E, P, p>(v, buf, t);
      group_sync<G, P>(g);
    }
  });
  // v[bitrev(r)] = output r of butterfly shfl_j(t) = element
  // h * L/2 + m + NSP * r of the last pass's input
  const bool odd = shfl_half(t) != 0;
  const V wm = row1[TT::offset(NP - 1)]; // W_L^m
  const T sgn = odd ? T(-1) : T(1);
  static_for<0, E>([&](auto rIC) {
    constexpr int r = decltype(rIC)::value;
    constexpr int e = bitrev<E>(r);
    // W_L^{NSP r} = W_{2E}^r = W_32^{r * 32 / (2E)}
    static_assert(L / NSP == 2 * E && 2 * E <= 32, "twiddle step");
    const V wr = mul_w32<T, (r * 32 / (2 * E)) % 32>(wm);
    const V f = odd ? wr : V{T(1), T(0)};
    const V own = vmul(v[e], f);
    V recv;
    recv.x = __shfl_xor_sync(0xffffffffu, own.x, 16);
    recv.y = __shfl_xor_sync(0xffffffffu, own.y, 16);
    // h = 0 lane: a + w b = own + recv; h = 1 lane: a - w b = recv - own
    v[e] = {fma(sgn, own.x, recv.x), fma(sgn, own.y, recv.y)};
  });
}

// pass_compute with the per-thread twiddle row instead of the recurrence.
template <typename T, int L, int E, int P, int PASS, typename V>
__device__ __forceinline__ void pass_compute_tw(V *v, const V *row) {
  using PL = Plan<L, E>;
  using TT = ThreadTw<T, L, E>;
  constexpr int R = PL::radix(PASS);
  constexpr int NS = PL::ns(PASS);
  constexpr int B = E / R;
  static_for<0, B>([&](auto bIC) {
    constexpr int b = decltype(bIC)::value;
    if constexpr (NS > 1) {
      const V *w = row + TT::offset(PASS) + b * R;
      if constexpr (sizeof(T) == 4) {
        static_for<0, R / 2>([&](auto qIC) {
          constexpr int q = decltype(qIC)::value;
          const float4 f = reinterpret_cast<const float4 *>(w)[q];
          const V w0 = {f.x, f.y}, w1 = {f.z, f.w};
          // slots 2q, 2q+1 hold r = 2q+1, 2q+2
          v[b * R + 2 * q + 1] = vmul(v[b * R + 2 * q + 1], w0);
          if constexpr (2 * q + 2 < R)
            v[b * R + 2 * q + 2] = vmul(v[b * R + 2 * q + 2], w1);
        });
      } else {
        static_for<1, R>([&](auto rIC) {
          constexpr int r = decltype(rIC)::value;
          v[b * R + r] = vmul(v[b * R + r], w[r - 1]);
        });
      }
    }
    dft_reg<T, R>(v + b * R);
  });
}

// fft_group with per-thread twiddles (row = this thread's twiddle row).
template <typename T, int L, int E, int P, int G, typename V>
__device__ __forceinline__ void fft_group_tw(V *v, V *buf, int t, int g,
                                             const V *row) {
  constexpr int NP = Plan<L, E>::passes();
  static_for<0, NP>([&](auto pIC) {
    constexpr int p = decltype(pIC)::value;
    if constexpr (p > 0) {
      pass_load<L, E, P, p>(v, buf, t);
      group_sync<G, P>(g);
    }
    pass_compute_tw<T, L, E, P, p>(v, row);
    if constexpr (p + 1 < NP) {
      pass_store<L, E, P, p>(v, buf, t);
      group_sync<G, P>(g);
    }
  });
}

// M independent transforms per thread (v[m][E], buffer of transform m at
// buf + m * bstride), sharing the per-thread twiddle loads and the barriers;
// the two instruction streams interleave and hide each other's latency.
template <typename T, int L, int E, int P, int PASS, int M, typename V>
__device__ __forceinline__ void pass_compute_tw_m(V (*v)[E], const V *row) {
  using PL = Plan<L, E>;
  using TT = ThreadTw<T, L, E>;
  constexpr int R = PL::radix(PASS);
  constexpr int NS = PL::ns(PASS);
  constexpr int B = E / R;
  static_for<0, B>([&](auto bIC) {
    constexpr int b = decltype(bIC)::value;
    if constexpr (NS > 1) {
      const V *w = row + TT::offset(PASS) + b * R;
      static_for<0, R / 2>([&](auto qIC) {
        constexpr int q = decltype(qIC)::value;
        V w0, w1;
        if constexpr (sizeof(T) == 4) {
          const float4 f = reinterpret_cast<const float4 *>(w)[q];
          w0 = {f.x, f.y};
          w1 = {f.z, f.w};
        } else {
          w0 = w[2 * q];
          w1 = w[2 * q + 1];
        }
        static_for<0, M>([&](auto mIC) {
          constexpr int m = decltype(mIC)::value;
          v[m][b * R + 2 * q + 1] = vmul(v[m][b * R + 2 * q + 1], w0);
          if constexpr (2 * q + 2 < R)
            v[m][b * R + 2 * q + 2] = vmul(v[m][b * R + 2 * q + 2], w1);
        });
      });
    }
    static_for<0, M>([&](auto mIC) {
      constexpr int m = decltype(mIC)::value;
      dft_reg<T, R>(v[m] + b * R);
    });
  });
}

// SKIP0: pass 0 (which reads only registers) was already computed by the
// caller, e.g. overlapped with other work.
template <typename T, int L, int E, int P, int G, int M, bool SKIP0 = false,
          typename V>
__device__ __forceinline__ void fft_group_tw_m(V (*v)[E], V *buf, int bstride,
                                               int t, int g, const V *row) {
  constexpr int NP = Plan<L, E>::passes();
  static_for<0, NP>([&](auto pIC) {
    constexpr int p = decltype(pIC)::value;
    if constexpr (p > 0) {
      static_for<0, M>([&](auto mIC) {
        constexpr int m = decltype(mIC)::value;
        pass_load<L, E, P, p>(v[m], buf + m * bstride, t);
      });
      group_sync<G, P>(g);
    }
    if constexpr (p > 0 || !SKIP0)
      pass_compute_tw_m<T, L, E, P, p, M>(v, row);
    if constexpr (p + 1 < NP) {
      static_for<0, M>([&](auto mIC) {
        constexpr int m = decltype(mIC)::value;
        pass_store<L, E, P, p>(v[m], buf + m * bstride, t);
      });
      group_sync<G, P>(g);
    }
  });
}

// Full transform after pass 0's inputs are in registers.  On return v holds
// the DFT: v[b*R + r] = X[t + b*P + r*(L/R)] with R the last radix.
// buf is the group's padded buffer (spad_size(L) values).
template <typename T, int L, int E, int P, int G, bool SKIP0 = false,
          typename V>
__device__ __forceinline__ void fft_group(V *v, V *buf, int t, int g,
                                          const V *tw) {
  constexpr int NP = Plan<L, E>::passes();
  static_for<0, NP>([&](auto pIC) {
    constexpr int p = decltype(pIC)::value;
    if constexpr (p > 0) {
      pass_load<L, E, P, p>(v, buf, t);
      group_sync<G, P>(g); // every read of this pass done before rewriting
    }
    if constexpr (p > 0 || !SKIP0)
      pass_compute<T, L, E, P, p>(v, t, tw);
    if constexpr (p + 1 < NP) {
      pass_store<L, E, P, p>(v, buf, t);
      group_sync<G, P>(g);
    }
  });
}

// Every pass but the last, leaving the input of the last pass in buf (stored,
// not yet synchronised: the caller synchronises before reading it).
template <typename T, int L, int E, int P, int G, typename V>
__device__ __forceinline__ void fft_group_prefix(V *v, V *buf, int t, int g,
                                                 const V *tw) {
  constexpr int NP = Plan<L, E>::passes();
  static_for<0, NP - 1>([&](auto pIC) {
    constexpr int p = decltype(pIC)::value;
    if constexpr (p > 0) {
      pass_load<L, E, P, p>(v, buf, t);
      group_sync<G, P>(g);
    }
    pass_compute<T, L, E, P, p>(v, t, tw);
    pass_store<L, E, P, p>(v, buf, t);
    if constexpr (p + 2 < NP)
      group_sync<G, P>(g);
  });
}

// Position (natural-order bin) of register slot e after fft_group (the last
// pass leaves each butterfly's outputs in bit-reversed register order).
template <int L, int E, int P>
__host__ __device__ constexpr int out_bin(int t, int e) {
  constexpr int R = Plan<L, E>::radix(Plan<L, E>::passes() - 1);
  return t + (e / R) * P + bitrev<R>(e % R) * (L / R);
}

// Position (time index) of register slot e for pass-0 inputs.
template <int L, int E, int P>
__host__ __device__ constexpr int in_index(int t, int e) {
  constexpr int R = Plan<L, E>::radix(0);
  return t + (e / R) * P + (e % R) * (L / R);
}

} // namespace ib200

// windows.cpp — F64 window tables for the spectral frontend.
//
// Same formulas and the same order of double operations as the reference's
// window composites (src/ops/signal/windows.cpp), so the tables agree with
// the reference's to the last bit on the same libm:
//   apply_sym          :25-36   (M == 1 -> [1]; periodic = symmetric M+1 cut)
//   cosine_sum_window  :40-55   w = a0 + sum_k (-1)^k a_k cos(n * (2 pi k/(N-1)))
//   boxcar :99, triang :107-123, parzen :129-158, bohman :164-183,
//   bartlett :189-200, cosine :206-214, exponential :220-228,
//   blackman :232-234, nuttall :240-242, blackmanharris :248-250,
//   flattop :256-259, hann :265, hamming :279-287, get_window :557-601.
// The spectral ops ask for get_window(name, nperseg, fftbins = false), i.e.
// the symmetric window (spectral_analysis.cpp:39-41).
#include "windows.h"

#include <cmath>
#include <stdexcept>

#ifndef M_PI
#define M_PI 3.14159265358979323846
#endif

namespace ib200 {
namespace {

template <typename Fn>
std::vector<double> apply_sym(int64_t M, bool sym, Fn &&fn) {
  if (M < 1)
    throw std::invalid_argument("window: M must be >= 1");
  if (M == 1)
    return {1.0};
  const int64_t Mw = sym ? M : M + 1;
  std::vector<double> w = fn(Mw);
  w.resize(M);
  return w;
}

std::vector<double> cosine_sum(int64_t N, const std::vector<double> &a) {
  const double den = N - 1.0;
  std::vector<double> r(N, a[0]);
  for (size_t k = 1; k < a.size(); ++k) {
    const double sign = (k % 2 == 0) ? 1.0 : -1.0;
    const double c = 2.0 * M_PI * k / den;
    const double amp = sign * a[k];
    for (int64_t i = 0; i < N; ++i)
      r[i] = r[i] + std::cos((double)i * c) * amp;
  }
  return r;
}

std::vector<double> general_cosine(int64_t M, std::vector<double> a, bool sym) {
  return apply_sym(M, sym, [&](int64_t N) { return cosine_sum(N, a); });
}

} // namespace

bool window_is_known(const std::string &w) {
  static const char *names[] = {
      "boxcar",  "rect",    "ones",           "dirichlet", "triang",
      "parzen",  "bohman",  "bartlett",       "cosine",    "exponential",
      "blackman", "nuttall", "blackmanharris", "flattop",  "hann",
      "hanning", "hamming"};
  for (const char *n : names)
    if (w == n)
      return true;
  return false;
}

std::vector<double> get_window(const std::string &window, int64_t Nx,
                               bool fftbins) {
  const bool sym = !fftbins;
  if (window == "boxcar" || window == "rect" || window == "ones" ||
      window == "dirichlet")
    return apply_sym(Nx, sym,
                     [](int64_t N) { return std::vector<double>(N, 1.0); });
  if (window == "triang")
    return apply_sym(Nx, sym, [](int64_t N) {
      std::vector<double> v(N);
      const bool odd = (N % 2 == 1);
      for (int64_t i = 0; i < N; ++i) {
        const int64_t n = i + 1;
        if (n <= (N + 1) / 2)
          v[i] = odd ? (2.0 * n / (N + 1.0)) : ((2.0 * n - 1.0) / N);
        else
          v[i] = v[N - 1 - i];
      }
      return v;
    });
  if (window == "parzen")
    return apply_sym(Nx, sym, [](int64_t N) {
      const double half_N = N / 2.0, quarter = (N - 1) / 4.0;
      std::vector<double> v(N);
      for (int64_t i = 0; i < N; ++i) {
        const double an = std::fabs((double)i - (N - 1.0) / 2.0);
        const double u = 1.0 - an / half_N;
        const double tail = 2.0 * ((u * u) * u);
        const double t = an / half_N;
        const double t2 = t * t, t3 = t2 * t;
        const double mid = (1.0 - 6.0 * t2) + 6.0 * t3;
        v[i] = (an > quarter) ? tail : mid;
      }
      return v;
    });
  if (window == "bohman")
    return apply_sym(Nx, sym, [](int64_t N) {
      const double den = N - 1.0;
      std::vector<double> v(N);
      for (int64_t i = 0; i < N; ++i) {
        const double fac = std::fabs((double)i / den - 0.5) * 2.0;
        const double pf = fac * M_PI;
        const double val =
            (1.0 - fac) * std::cos(pf) + (1.0 / M_PI) * std::sin(pf);
        v[i] = (fac < 1.0) ? val : 0.0;
      }
      return v;
    });
  if (window == "bartlett")
    return apply_sym(Nx, sym, [](int64_t N) {
      const double den = N - 1.0;
      std::vector<double> v(N);
      for (int64_t i = 0; i < N; ++i) {
        const double ramp = ((double)i * 2.0) / den;
        v[i] = ((double)i <= (double)(N / 2)) ? ramp : 2.0 - ramp;
      }
      return v;
    });
  if (window == "cosine")
    return apply_sym(Nx, sym, [](int64_t N) {
      std::vector<double> v(N);
      for (int64_t i = 0; i < N; ++i)
        v[i] = std::sin(((double)i + 0.5) * (M_PI / N));
      return v;
    });
  if (window == "exponential")
    return apply_sym(Nx, sym, [](int64_t N) {
      const double c = (N - 1.0) / 2.0, tau = 1.0;
      std::vector<double> v(N);
      for (int64_t i = 0; i < N; ++i)
        v[i] = std::exp(-std::fabs((double)i - c) / tau);
      return v;
    });
  if (window == "blackman")
    return general_cosine(Nx, {0.42, 0.50, 0.08}, sym);
  if (window == "nuttall")
    return general_cosine(Nx, {0.3635819, 0.4891775, 0.1365995, 0.0106411},
                          sym);
  if (window == "blackmanharris")
    return general_cosine(Nx, {0.35875, 0.48829, 0.14128, 0.01168}, sym);
  if (window == "flattop")
    return general_cosine(
        Nx, {0.21557895, 0.41663158, 0.277263158, 0.083578947, 0.006947368},
        sym);
  if (window == "hann" || window == "hanning")
    return general_cosine(Nx, {0.5, 1.0 - 0.5}, sym);
  if (window == "hamming")
    return apply_sym(Nx, sym, [](int64_t N) {
      const double c = 2.0 * M_PI / (N - 1);
      std::vector<double> v(N);
      for (int64_t i = 0; i < N; ++i)
        v[i] = 0.54 + (-0.46) * std::cos((double)i * c);
      return v;
    });
  throw std::invalid_argument("get_window: unknown window name '" + window +
                              "'");
}

} // namespace ib200

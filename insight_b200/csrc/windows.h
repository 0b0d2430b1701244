// windows.h — F64 window tables (reference formulas, src/ops/signal/windows.cpp).
#pragma once
#include <cstdint>
#include <string>
#include <vector>

namespace ib200 {

// get_window(name, Nx, fftbins): fftbins == false gives the symmetric
// window the spectral ops use.  Throws std::invalid_argument with the
// reference's message for an unknown name.
std::vector<double> get_window(const std::string &window, int64_t Nx,
                               bool fftbins);

bool window_is_known(const std::string &window);

} // namespace ib200

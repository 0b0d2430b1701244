// spectral_util.cu — small device helpers of the spectral backend.
#include "spectral_kernels.cuh"

#include <algorithm>

namespace ib200 {
// In-place scaling of reduced raw sums (see scale_sums in launch.h).
__global__ void scale_sums_kernel(double *sums, int64_t C, int64_t F, int cplx,
                                  double factor, int mask) {
  const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i >= C * F)
    return;
  const int64_t k = i % F;
  const double f = (mask && k >= 1 && k <= F - 2) ? 2.0 * factor : factor;
  if (cplx) {
    sums[2 * i] *= f;
    sums[2 * i + 1] *= f;
  } else {
    sums[i] *= f;
  }
}

// f[i] = i * df and t[i] = (i * step + half) / fs, each a single correctly
// rounded double operation as on the host (no contraction), so the device
// axes equal the host's bit for bit.
__global__ void write_axes_kernel(double *f, int64_t F, double df, double *t,
                                  int64_t S, int64_t step, double half, double fs) {
  const int64_t n = F > S ? F : S;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    if (f && i < F)
      f[i] = __dmul_rn((double)i, df);
    if (t && i < S)
      t[i] = __ddiv_rn(__dadd_rn((double)(i * step), half), fs);
  }
}

cudaError_t write_axes_device(double *f, int64_t F, double df, double *t,
                              int64_t S, int64_t step, double half, double fs,
                              cudaStream_t stream) {
  const int64_t n = F > S ? F : S;
  if (n <= 0 || (!f && !t))
    return cudaSuccess;
  const int threads = 256;
  const int64_t blocks = std::min<int64_t>((n + threads - 1) / threads, 1024);
  write_axes_kernel<<<(unsigned)blocks, threads, 0, stream>>>(f, F, df, t, S, step,
                                                              half, fs);
  return cudaGetLastError();
}

cudaError_t scale_sums(double *sums, int64_t C, int64_t F, bool complex_sums,
                       double factor, bool mask, cudaStream_t stream) {
  const int64_t n = C * F;
  if (n <= 0)
    return cudaSuccess;
  const int threads = 256;
  scale_sums_kernel<<<(unsigned)((n + threads - 1) / threads), threads, 0,
                      stream>>>(sums, C, F, complex_sums ? 1 : 0, factor,
                                mask ? 1 : 0);
  return cudaGetLastError();
}
} // namespace ib200

// spectral_util.cu — small device helpers of the spectral backend.
#include "spectral_kernels.cuh"

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

// spectral_istft.cu — f32 / f64 instantiations of the inverse STFT kernels.
#include "spectral_dispatch.cuh"
#include "spectral_istft.cuh"

namespace ib200 {
cudaError_t launch_istft(const IstftDesc &d, int num_sms, cudaStream_t stream,
                         int64_t *launches) {
  if (!nfft_supported(d.nfft))
    return cudaErrorInvalidValue;
  // f64 transforms for both input precisions (see spectral_istft.cuh)
  return d.f64 ? run_istft_t<double, double>(d, num_sms, stream, launches)
               : run_istft_t<double, float>(d, num_sms, stream, launches);
}
} // namespace ib200

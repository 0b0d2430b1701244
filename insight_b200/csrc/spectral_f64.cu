// spectral_f64.cu — f64 instantiations of the fused spectral kernels.
#include "spectral_dispatch.cuh"

namespace ib200 {
cudaError_t launch_f64(const LaunchDesc &d, void *scratch, int num_sms,
                       cudaStream_t stream, int64_t *launches) {
  return launch_t<double>(d, scratch, num_sms, stream, launches);
}
} // namespace ib200

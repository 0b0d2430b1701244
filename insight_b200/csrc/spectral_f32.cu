// spectral_f32.cu — f32 instantiations of the fused spectral kernels.
#include "spectral_dispatch.cuh"

namespace ib200 {
cudaError_t launch_f32(const LaunchDesc &d, void *scratch, int num_sms,
                       cudaStream_t stream, int64_t *launches) {
  return launch_t<float>(d, scratch, num_sms, stream, launches);
}
} // namespace ib200

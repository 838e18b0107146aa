// nl_step_h128.cu -- the decode-step kernel (nl_step_kernel.cuh) for head size 128.
#include "nl_step_kernel.cuh"

namespace nl {
cudaError_t step_launch_h128(const StepArgs &a, cudaStream_t st) {
  return step_launch_hd<128>(a, st);
}
}  // namespace nl

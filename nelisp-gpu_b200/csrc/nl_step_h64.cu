// nl_step_h64.cu -- the decode-step kernel (nl_step_kernel.cuh) for head size 64.
#include "nl_step_kernel.cuh"

namespace nl {
cudaError_t step_launch_h64(const StepArgs &a, cudaStream_t st) {
  return step_launch_hd<64>(a, st);
}
}  // namespace nl

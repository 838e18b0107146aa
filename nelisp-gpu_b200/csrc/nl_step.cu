// nl_step.cu -- the decoder's decode step as one persistent kernel: which
// shapes it serves, the sizes of its buffers, and its launch.  The kernel
// itself is in nl_step_kernel.cuh, instantiated per head size in
// nl_step_h128.cu and nl_step_h64.cu.

#include <cuda_runtime.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include "nl_internal.h"
#include "nl_step.h"

namespace nl {

bool step_supported(uint32_t B, uint32_t H, uint32_t hd, uint32_t hr, uint32_t kvr, uint32_t fr,
                    int tp) {
  // NELISP_DECODER_STEP=kernel selects the one-kernel step, =kernels the
  // separate launches; unset, the separate launches.
  const char *v = getenv("NELISP_DECODER_STEP");
  if (!(v && strcmp(v, "kernel") == 0)) return false;
  const uint32_t grp = kvr ? hr / kvr : 0;
  return tp == 1 && B >= 1 && B <= kStepMaxB && (hd == 64 || hd == 128) && grp >= 1 &&
         grp <= 8 && hr == kvr * grp && H % 128u == 0 && H <= kStepMaxK &&
         hr * hd <= kStepMaxK && (hr * hd) % 128u == 0 && fr % 128u == 0 && fr > 0;
}

uint32_t step_down_chunks(uint32_t fr) {
  const uint32_t nb = fr / 128u, per = kStepMaxK / 128u;
  return (nb + per - 1u) / per;
}

size_t step_dpart_bytes(uint32_t B, uint32_t H, uint32_t fr) {
  return (size_t)step_down_chunks(fr) * B * H * sizeof(long long);
}

cudaError_t step_launch(const StepArgs &a, cudaStream_t st) {
  if (a.hd == 128) return step_launch_h128(a, st);
  if (a.hd == 64) return step_launch_h64(a, st);
  return cudaErrorInvalidValue;
}

}  // namespace nl

// vksoftmax -- the softmax verify CLI of host/vksoftmax.c, on CUDA.
//
//   vksoftmax softmax.spv [M N]
//
// A[i] = (i%7)*0.3f (host/vksoftmax.c:60), one softmax dispatch, a sampled
// check against a double-precision softmax at abs 1e-3 and the row-0 sum
// (:103-114).  Output line and exit status as the reference's.
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>

#include <vector>

#include "nelisp_cuda.h"

int main(int argc, char **argv) {
  if (argc < 2) { fprintf(stderr, "usage: %s softmax.spv [M N]\n", argv[0]); return 1; }
  uint32_t M = (argc >= 4) ? atoi(argv[2]) : 64, N = (argc >= 4) ? atoi(argv[3]) : 256;
  size_t sz = (size_t)M * N;
  if (nl_init(-1) != NL_OK) { fprintf(stderr, "%s\n", nl_last_error()); return 2; }
  printf("device = %s\n", nl_device_name());
  std::vector<float> A(sz ? sz : 1), C(sz ? sz : 1);
  for (size_t i = 0; i < sz; i++) A[i] = (float)((i % 7)) * 0.3f;
  nl_run_buffer bufs[2] = {{(uint32_t)sz, NL_RUN_IN, 0}, {(uint32_t)sz, NL_RUN_OUT, 0}};
  uint32_t push[2] = {M, N};
  if (nl_run("softmax", 2, bufs, 2, push, (M + 63) / 64, A.data(), C.data()) != NL_OK) {
    fprintf(stderr, "%s\n", nl_last_error());
    return 2;
  }
  int bad = 0;
  double maxerr = 0;
  for (uint32_t r = 0; r < M && bad < 5; r += (M / 9 > 0 ? M / 9 : 1)) {
    double mx = -1e30;
    for (uint32_t j = 0; j < N; j++) {
      double v = (double)(((size_t)r * N + j) % 7) * 0.3;
      if (v > mx) mx = v;
    }
    double s = 0;
    for (uint32_t j = 0; j < N; j++) s += exp((double)(((size_t)r * N + j) % 7) * 0.3 - mx);
    for (uint32_t j = 0; j < N; j += (N / 9 > 0 ? N / 9 : 1)) {
      double ref = exp((double)(((size_t)r * N + j) % 7) * 0.3 - mx) / s;
      double got = C[(size_t)r * N + j];
      double err = fabs(got - ref);
      if (err > maxerr) maxerr = err;
      if (err > 1e-3) {
        if (bad < 5) fprintf(stderr, "C[%u,%u]=%g ref=%g\n", r, j, got, ref);
        bad++;
      }
    }
  }
  double rs = 0;
  for (uint32_t j = 0; j < N; j++) rs += C[j];
  printf("softmax %ux%u  row0_sum=%.5f  max_abs_err=%.2e  %s\n", M, N, rs, maxerr,
         bad ? "FAIL" : "PASS");
  nl_shutdown();
  return bad ? 1 : 0;
}

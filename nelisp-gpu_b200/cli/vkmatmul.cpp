// vkmatmul -- the f32 matmul bench/verify CLI of host/vkmatmul.c, on CUDA.
//
//   vkmatmul matmul.spv [M K N] [naive|tiled|reg] [iters]
//
// A[i] = i%4, B[i] = i%3 (host/vkmatmul.c:92-93); ITERS dispatches are
// recorded once (here: captured into a CUDA graph), replayed once as a warm
// up and once timed, and the time is divided by ITERS (:146-169).  A 7x7
// sample of C is checked EXACTLY against a double sum (:172-180).  Output
// line and exit status (0 pass, 1 fail, 2 fatal) as the reference's.
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <vector>

#include "nelisp_cuda.h"

int main(int argc, char **argv) {
  if (argc < 2) { fprintf(stderr, "usage: %s matmul.spv [M K N]\n", argv[0]); return 1; }
  uint32_t M = (argc >= 5) ? atoi(argv[2]) : 128;
  uint32_t K = (argc >= 5) ? atoi(argv[3]) : 128;
  uint32_t N = (argc >= 5) ? atoi(argv[4]) : 128;
  size_t na = (size_t)M * K, nb = (size_t)K * N, nc = (size_t)M * N;
  if (nl_init(-1) != NL_OK) { fprintf(stderr, "%s\n", nl_last_error()); return 2; }
  printf("device = %s\n", nl_device_name());
  std::vector<float> A(na), B(nb);
  for (size_t i = 0; i < na; i++) A[i] = (float)(i % 4);
  for (size_t i = 0; i < nb; i++) B[i] = (float)(i % 3);
  const char *kernel = "matmul";
  uint32_t groups = (uint32_t)((nc + 63) / 64);
  if (argc >= 6 && !strcmp(argv[5], "tiled")) {
    kernel = "matmul-tiled";
    groups = ((M + 15) / 16) * ((N + 15) / 16);
  } else if (argc >= 6 && !strcmp(argv[5], "reg")) {
    kernel = "matmul-reg";
    groups = ((((M + 3) / 4) * ((N + 3) / 4)) + 63) / 64;
  }
  uint32_t iters = (argc >= 7) ? (uint32_t)atoi(argv[6]) : 20;
  if (iters == 0) iters = 1;
  uint32_t ha, hb;
  if (nl_upload(A.data(), (uint32_t)na, &ha) || nl_upload(B.data(), (uint32_t)nb, &hb)) {
    fprintf(stderr, "%s\n", nl_last_error());
    return 2;
  }
  nl_slot slots[3] = {{NL_SLOT_RESIDENT, (uint32_t)na, ha},
                      {NL_SLOT_RESIDENT, (uint32_t)nb, hb},
                      {NL_SLOT_OUT, (uint32_t)nc, 0}};
  std::vector<nl_dispatch> disps(iters);
  for (uint32_t it = 0; it < iters; it++) {
    nl_dispatch &d = disps[it];
    memset(&d, 0, sizeof(d));
    snprintf(d.name, sizeof(d.name), "%s", kernel);
    d.nbuf = 3;
    d.slot[0] = 0; d.slot[1] = 1; d.slot[2] = 2;
    d.npush = 3;
    d.push[0] = M; d.push[1] = K; d.push[2] = N;
    d.groups = groups;
  }
  uint32_t hc;
  if (nl_compile(3, slots, iters, disps.data(), nullptr, &hc) != NL_OK) {
    fprintf(stderr, "%s\n", nl_last_error());
    return 2;
  }
  double ms = 0.0;
  if (nl_time_compiled(hc, 1, &ms) != NL_OK || nl_time_compiled(hc, 1, &ms) != NL_OK) {
    fprintf(stderr, "%s\n", nl_last_error());
    return 2;
  }
  double dt = ms * 1e-3 / (double)iters;
  std::vector<float> C(nc ? nc : 1);
  if (nl_run_compiled(hc, C.data()) != NL_OK) { fprintf(stderr, "%s\n", nl_last_error()); return 2; }
  int bad = 0;
  size_t checks = 0;
  for (uint32_t r = 0; r < M && bad < 5; r += (M / 7 > 0 ? M / 7 : 1))
    for (uint32_t c = 0; c < N && bad < 5; c += (N / 7 > 0 ? N / 7 : 1)) {
      double acc = 0;
      for (uint32_t k = 0; k < K; k++)
        acc += (double)(((size_t)r * K + k) % 4) * (double)(((size_t)k * N + c) % 3);
      float got = C[(size_t)r * N + c];
      if ((double)got != acc) {
        if (bad < 5) fprintf(stderr, "C[%u,%u]=%g want=%g\n", r, c, got, acc);
        bad++;
      }
      checks++;
    }
  double flop = 2.0 * (double)M * N * K;
  printf("matmul %ux%u x %ux%u  gpu=%.4fs  %.1f GFLOP/s  checks=%zu  %s\n", M, K, K, N, dt,
         flop / dt / 1e9, checks, bad ? "FAIL" : "PASS");
  nl_shutdown();
  return bad ? 1 : 0;
}

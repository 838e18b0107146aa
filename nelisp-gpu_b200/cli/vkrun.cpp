// vkrun -- generic one-shot dispatcher with host/vkrun.c's interface, on CUDA.
//
//   vkrun SPV IN_FILE OUT_FILE LOCAL GROUPS PUSH_CSV SIZES_CSV
//
// The kernel is the basename of SPV without its extension
// (kernels/softmax.spv -> softmax); the file itself is not read.  Every
// buffer is loaded from IN_FILE (zero-filled past its end) and every buffer
// is written back to OUT_FILE, as host/vkrun.c:41-45, :125-129 do.  LOCAL is
// accepted for compatibility; the workgroup size is the reference's 64.
// Exit status: 0 ok, 1 usage, 2 failure (unknown kernel, bad arguments,
// device error).
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <string>
#include <vector>

#include "nelisp_cuda.h"

static int parse_csv(const char *s, uint32_t *out, int max) {
  if (!s || !strcmp(s, "-")) return 0;
  int n = 0;
  std::string t(s);
  size_t p = 0;
  while (p <= t.size() && n < max) {
    size_t q = t.find(',', p);
    if (q == std::string::npos) q = t.size();
    if (q > p) out[n++] = (uint32_t)strtoul(t.substr(p, q - p).c_str(), nullptr, 10);
    p = q + 1;
  }
  return n;
}

static std::string kernel_of(const char *spv) {
  std::string s(spv);
  size_t slash = s.find_last_of('/');
  if (slash != std::string::npos) s = s.substr(slash + 1);
  size_t dot = s.rfind(".spv");
  if (dot != std::string::npos && dot + 4 == s.size()) s = s.substr(0, dot);
  return s;
}

int main(int argc, char **argv) {
  if (argc < 8) {
    fprintf(stderr, "usage: %s SPV IN OUT LOCAL GROUPS PUSH SIZES\n", argv[0]);
    return 1;
  }
  std::string name = kernel_of(argv[1]);
  uint32_t groups = (uint32_t)strtoul(argv[5], nullptr, 10);
  uint32_t push[NL_MAX_PUSH], sizes[NL_MAX_BUFS];
  int npush = parse_csv(argv[6], push, NL_MAX_PUSH);
  int nbuf = parse_csv(argv[7], sizes, NL_MAX_BUFS);
  if (nbuf < 1) { fprintf(stderr, "need >=1 buffer\n"); return 1; }
  uint64_t total = 0;
  for (int i = 0; i < nbuf; i++) total += sizes[i];
  std::vector<uint32_t> host(total ? total : 1, 0u);
  FILE *f = fopen(argv[2], "rb");
  if (!f) { fprintf(stderr, "open %s\n", argv[2]); return 2; }
  size_t got = fread(host.data(), 4, total, f);
  (void)got;   // short files are zero-filled, as host/vkrun.c:43-44
  fclose(f);
  if (nl_init(-1) != NL_OK) { fprintf(stderr, "vkrun: %s\n", nl_last_error()); return 2; }
  std::vector<nl_run_buffer> bufs(nbuf);
  for (int i = 0; i < nbuf; i++) bufs[i] = {sizes[i], NL_RUN_INOUT, 0};
  std::vector<uint32_t> out(total ? total : 1, 0u);
  int rc = nl_run(name.c_str(), (uint32_t)nbuf, bufs.data(), (uint32_t)npush, push, groups,
                  host.data(), out.data());
  if (rc != NL_OK) {
    fprintf(stderr, "vkrun: %s\n", nl_last_error());
    nl_shutdown();
    return 2;
  }
  FILE *of = fopen(argv[3], "wb");
  if (!of) { fprintf(stderr, "open %s\n", argv[3]); nl_shutdown(); return 2; }
  fwrite(out.data(), 4, total, of);
  fclose(of);
  nl_shutdown();
  return 0;
}

// nelisp-cuserver -- the persistent compute server of zawatton/nelisp-gpu
// (host/vkserver.c) on CUDA: the same stdin/stdout binary protocol, driven
// by lisp/nelisp-gpu-server.el unchanged (set `nelisp-gpu-server-bin' to this
// binary).
//
//   run: nelisp-cuserver KERNEL_DIR
//
// KERNEL_DIR is accepted and ignored: every kernel is compiled into
// libnelisp_cuda and selected by name, so no .spv file is ever read.
//
// Wire format (little-endian u32 words; host/vkserver.c:11-38, :420-432):
//   0 RUN          name_len name nbuf {size kind [handle]}* npush push* groups inline*
//                  -> status out*            (kinds: 0 in, 1 res, 2 out, 3 inout)
//   1 UPLOAD       n data*                   -> status handle
//   2 FREE         handle                    -> status
//   3 BATCH        nslot {kind size [handle]}* ndisp
//                  {name_len name nbuf slot* npush push* groups}* inline*
//                  -> status out*            (kinds: 0 in, 1 res, 2 tmp, 3 out)
//   4 COMPILE      as BATCH                  -> status handle
//   5 RUN_COMPILED handle                    -> status out*
//   6 FREE_COMPILED handle                   -> status
//   7 WRITE_RESIDENT handle n data*          -> status
//   8 UPLOAD_FILE  pathlen path off_lo off_hi n -> status handle
//
// Error behaviour follows the reference: a truncated request (EOF) exits 0;
// a malformed one that cannot be resynchronised (name too long, too many
// buffers or push constants) exits 2, as does an unknown opcode or a CUDA
// error that leaves the device unusable.  Recoverable errors reply status 1.
// Unlike the reference, a failed RUN or BATCH still sends the byte count the
// client waits for (status 1 followed by zeros), so the client reports the
// error instead of blocking; an unknown kernel name or a bad resident handle
// is such a recoverable error rather than a crash.
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <vector>

#include "nelisp_cuda.h"

namespace {

enum {
  OP_RUN = 0, OP_UPLOAD = 1, OP_FREE = 2, OP_BATCH = 3, OP_COMPILE = 4,
  OP_RUN_COMPILED = 5, OP_FREE_COMPILED = 6, OP_WRITE_RESIDENT = 7,
  OP_UPLOAD_FILE = 8
};

bool rd(uint32_t *v) { return fread(v, 4, 1, stdin) == 1; }
void rd_or_exit(uint32_t *v) { if (!rd(v)) exit(0); }
void rd_words(std::vector<uint32_t> &buf, uint64_t n) {
  buf.resize(n ? n : 1);
  if (n && fread(buf.data(), 4, n, stdin) != n) exit(0);
}
void wr(uint32_t v) { fwrite(&v, 4, 1, stdout); }
void wr_words(const void *p, uint64_t n) { if (n) fwrite(p, 4, n, stdout); }
void wr_zeros(uint64_t n) {
  static const uint32_t z[1024] = {0};
  while (n) {
    uint64_t k = n < 1024 ? n : 1024;
    fwrite(z, 4, k, stdout);
    n -= k;
  }
}
void done() { fflush(stdout); }

// NL_FATAL means the device is gone: exit(2), as VK_CHECK does.
int check(int rc, const char *what) {
  if (rc == NL_FATAL) {
    fprintf(stderr, "nelisp-cuserver: %s: %s\n", what, nl_last_error());
    exit(2);
  }
  if (rc != NL_OK) fprintf(stderr, "nelisp-cuserver: %s: %s\n", what, nl_last_error());
  return rc;
}

void handle_run() {
  uint32_t name_len;
  rd_or_exit(&name_len);
  if (name_len > NL_MAX_NAME) { fprintf(stderr, "name too long\n"); exit(2); }
  char name[NL_MAX_NAME + 1] = {0};
  if (fread(name, 1, name_len, stdin) != name_len) exit(0);
  uint32_t nbuf;
  rd_or_exit(&nbuf);
  if (nbuf > NL_MAX_BUFS) { fprintf(stderr, "nbuf %u > %d\n", nbuf, NL_MAX_BUFS); exit(2); }
  nl_run_buffer bufs[NL_MAX_BUFS];
  uint64_t nin = 0, nout = 0;
  for (uint32_t i = 0; i < nbuf; i++) {
    rd_or_exit(&bufs[i].size);
    rd_or_exit(&bufs[i].kind);
    bufs[i].handle = 0;
    if (bufs[i].kind == NL_RUN_RESIDENT) rd_or_exit(&bufs[i].handle);
    if (bufs[i].kind == NL_RUN_IN || bufs[i].kind == NL_RUN_INOUT) nin += bufs[i].size;
    if (bufs[i].kind == NL_RUN_OUT || bufs[i].kind == NL_RUN_INOUT) nout += bufs[i].size;
  }
  uint32_t npush, push[NL_MAX_PUSH];
  rd_or_exit(&npush);
  if (npush > NL_MAX_PUSH) { fprintf(stderr, "npush %u > %d\n", npush, NL_MAX_PUSH); exit(2); }
  for (uint32_t i = 0; i < npush; i++) rd_or_exit(&push[i]);
  uint32_t groups;
  rd_or_exit(&groups);
  static std::vector<uint32_t> in, out;
  rd_words(in, nin);
  out.resize(nout ? nout : 1);
  int rc = check(nl_run(name, nbuf, bufs, npush, push, groups, in.data(), out.data()), name);
  wr(rc == NL_OK ? 0u : 1u);
  if (rc == NL_OK) wr_words(out.data(), nout);
  else wr_zeros(nout);
  done();
}

void handle_upload() {
  uint32_t n;
  rd_or_exit(&n);
  static std::vector<uint32_t> data;
  rd_words(data, n);
  uint32_t h = 0;
  int rc = check(nl_upload(data.data(), n, &h), "upload");
  wr(rc == NL_OK ? 0u : 1u);
  wr(rc == NL_OK ? h : 0u);
  done();
}

void handle_free() {
  uint32_t h;
  rd_or_exit(&h);
  check(nl_free(h), "free");
  wr(0);
  done();
}

// Shared by BATCH and COMPILE.
struct BatchReq {
  std::vector<nl_slot> slots;
  std::vector<nl_dispatch> disps;
  std::vector<uint32_t> in;
  uint64_t nout = 0;
};

void read_batch(BatchReq &R) {
  uint32_t nslot;
  rd_or_exit(&nslot);
  if (nslot > NL_MAX_SLOTS) { fprintf(stderr, "nslot %u > %d\n", nslot, NL_MAX_SLOTS); exit(2); }
  R.slots.resize(nslot);
  uint64_t nin = 0;
  for (uint32_t i = 0; i < nslot; i++) {
    nl_slot &s = R.slots[i];
    rd_or_exit(&s.kind);
    rd_or_exit(&s.size);
    s.handle = 0;
    if (s.kind == NL_SLOT_RESIDENT) rd_or_exit(&s.handle);
    if (s.kind == NL_SLOT_IN) nin += s.size;
    if (s.kind == NL_SLOT_OUT) R.nout += s.size;
  }
  uint32_t ndisp;
  rd_or_exit(&ndisp);
  if (ndisp > NL_MAX_DISPATCH) { fprintf(stderr, "ndisp %u > %d\n", ndisp, NL_MAX_DISPATCH); exit(2); }
  R.disps.resize(ndisp);
  for (uint32_t d = 0; d < ndisp; d++) {
    nl_dispatch &D = R.disps[d];
    memset(&D, 0, sizeof(D));
    uint32_t nl;
    if (!rd(&nl) || nl > NL_MAX_NAME) exit(2);
    if (fread(D.name, 1, nl, stdin) != nl) exit(0);
    rd_or_exit(&D.nbuf);
    if (D.nbuf > NL_MAX_BUFS) { fprintf(stderr, "nbuf %u > %d\n", D.nbuf, NL_MAX_BUFS); exit(2); }
    for (uint32_t i = 0; i < D.nbuf; i++) rd_or_exit(&D.slot[i]);
    rd_or_exit(&D.npush);
    if (D.npush > NL_MAX_PUSH) { fprintf(stderr, "npush %u > %d\n", D.npush, NL_MAX_PUSH); exit(2); }
    for (uint32_t i = 0; i < D.npush; i++) rd_or_exit(&D.push[i]);
    rd_or_exit(&D.groups);
  }
  rd_words(R.in, nin);
}

void handle_batch() {
  BatchReq R;
  read_batch(R);
  static std::vector<uint32_t> out;
  out.resize(R.nout ? R.nout : 1);
  int rc = check(nl_batch((uint32_t)R.slots.size(), R.slots.data(), (uint32_t)R.disps.size(),
                          R.disps.data(), R.in.data(), out.data()),
                 "batch");
  wr(rc == NL_OK ? 0u : 1u);
  if (rc == NL_OK) wr_words(out.data(), R.nout);
  else wr_zeros(R.nout);
  done();
}

void handle_compile() {
  BatchReq R;
  read_batch(R);
  uint32_t h = 0;
  int rc = check(nl_compile((uint32_t)R.slots.size(), R.slots.data(), (uint32_t)R.disps.size(),
                            R.disps.data(), R.in.data(), &h),
                 "compile");
  wr(rc == NL_OK ? 0u : 1u);
  wr(rc == NL_OK ? h : 0u);
  done();
}

void handle_run_compiled() {
  uint32_t h;
  rd_or_exit(&h);
  uint64_t nout = 0;
  if (nl_compiled_out_words(h, &nout) != NL_OK) {
    // The reference replies a bare status here (host/vkserver.c:593).
    fprintf(stderr, "nelisp-cuserver: bad compiled %u\n", h);
    wr(1);
    done();
    return;
  }
  static std::vector<uint32_t> out;
  out.resize(nout ? nout : 1);
  int rc = check(nl_run_compiled(h, out.data()), "run-compiled");
  wr(rc == NL_OK ? 0u : 1u);
  if (rc == NL_OK) wr_words(out.data(), nout);
  else wr_zeros(nout);
  done();
}

void handle_free_compiled() {
  uint32_t h;
  rd_or_exit(&h);
  check(nl_free_compiled(h), "free-compiled");
  wr(0);
  done();
}

void handle_write_resident() {
  uint32_t h, n;
  rd_or_exit(&h);
  rd_or_exit(&n);
  static std::vector<uint32_t> data;
  rd_words(data, n);
  int rc = check(nl_write_resident(h, data.data(), n), "write-resident");
  wr(rc == NL_OK ? 0u : 1u);
  done();
}

void handle_upload_file() {
  uint32_t plen, olo, ohi, n;
  rd_or_exit(&plen);
  if (plen == 0 || plen > 4095) {
    // host/vkserver.c:374 exits 0 here.
    fprintf(stderr, "nelisp-cuserver: bad path length %u\n", plen);
    exit(0);
  }
  char path[4096];
  if (fread(path, 1, plen, stdin) != plen) exit(0);
  path[plen] = 0;
  rd_or_exit(&olo);
  rd_or_exit(&ohi);
  rd_or_exit(&n);
  uint64_t off = ((uint64_t)ohi << 32) | olo;
  uint32_t h = 0;
  int rc = check(nl_upload_file(path, off, n, &h), "upload-file");
  wr(rc == NL_OK ? 0u : 1u);
  wr(rc == NL_OK ? h : 0u);
  done();
}

}  // namespace

int main(int argc, char **argv) {
  if (argc < 2) {
    fprintf(stderr, "usage: %s KERNEL_DIR\n", argv[0]);
    return 1;
  }
  static char ibuf[1 << 20], obuf[1 << 20];
  setvbuf(stdin, ibuf, _IOFBF, sizeof(ibuf));
  setvbuf(stdout, obuf, _IOFBF, sizeof(obuf));
  if (nl_init(-1) != NL_OK) {
    fprintf(stderr, "nelisp-cuserver: %s\n", nl_last_error());
    return 2;
  }
  fprintf(stderr, "nelisp-cuserver: device = %s\n", nl_device_name());
  fprintf(stderr, "nelisp-cuserver: ready\n");
  fflush(stderr);
  uint32_t op;
  while (rd(&op)) {
    switch (op) {
      case OP_RUN: handle_run(); break;
      case OP_UPLOAD: handle_upload(); break;
      case OP_FREE: handle_free(); break;
      case OP_BATCH: handle_batch(); break;
      case OP_COMPILE: handle_compile(); break;
      case OP_RUN_COMPILED: handle_run_compiled(); break;
      case OP_FREE_COMPILED: handle_free_compiled(); break;
      case OP_WRITE_RESIDENT: handle_write_resident(); break;
      case OP_UPLOAD_FILE: handle_upload_file(); break;
      default:
        fprintf(stderr, "nelisp-cuserver: bad opcode %u\n", op);
        return 2;
    }
  }
  nl_shutdown();
  return 0;
}

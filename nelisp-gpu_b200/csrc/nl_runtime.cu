// nl_runtime.cu -- libnelisp_cuda's host runtime: device context, resident
// buffers, and the run / batch / compile executor behind the C ABI.
//
// Replaces host/vkserver.c's Vulkan instance, buffer and dispatch code:
//   init_vulkan (:213-245)            -> nl_init: device, stream, staging
//   resident table (:83-86, :336-418) -> cudaMalloc'd buffers, same handle
//                                        allocation order (first free slot)
//   staged_write (:169-205)           -> pinned 64 MiB staging for files
//   handle_run / handle_batch         -> one stream; stream order stands in
//     (:274-334, :437-506)               for the reference's barriers
//   handle_compile / run_compiled     -> stream capture into a CUDA graph,
//     (:511-604)                         memset nodes zero tmp/out slots
// Allocation failure of a resident buffer falls back to pinned host memory
// the GPU reads over the bus, as the reference falls back to host-visible
// memory when VRAM is exhausted (:141-147).

#include <cuda_runtime.h>
#include <errno.h>
#include <fcntl.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

#include <thread>

#include <vector>

#include "nl_internal.h"

namespace nl {
namespace {

constexpr size_t kStageBytes = 64u << 20;  // host/vkserver.c:163

struct Resident {
  void *ptr = nullptr;
  uint32_t words = 0;
  bool used = false;
  bool host = false;   // pinned host fallback
};

struct Compiled {
  bool used = false;
  cudaGraphExec_t exec = nullptr;
  void *mem = nullptr;           // one allocation for every owned slot + scratch
  bool mem_host = false;
  std::vector<void *> slot_ptr;
  std::vector<uint32_t> slot_words;
  std::vector<uint32_t> out_slots;
  uint64_t out_words = 0;
  uint64_t kernels = 0;          // kernels per replay
};

// staging slots of the host-buffer GEMV entry: calls that may be in flight at
// once.  A call beyond that reuses the slot of the call kHostSlots before it,
// whose nl_host_wait then also waits for the newer call.
constexpr int kHostSlots = 8;

struct Context {
  bool ready = false;
  int device = -1;
  cudaStream_t stream = nullptr;
  char devname[256] = {0};
  Resident res[NL_MAX_RESIDENT];
  uint32_t nres = 0;
  Compiled comp[NL_MAX_COMPILED];
  void *stage = nullptr;
  void *arena = nullptr;
  size_t arena_bytes = 0;
  void *ws = nullptr;
  size_t ws_bytes = 0;
  uint64_t launches = 0;
  bool capturing = false;
  uint64_t capture_launches = 0;
  // host-buffer GEMV entry: copy streams and device staging slots.  Ticket t
  // (1-based) uses slot (t-1) % kHostSlots; the slot's events order its reuse.
  cudaStream_t h2d = nullptr, d2h = nullptr;
  struct HostSlot {
    void *buf = nullptr;
    size_t bytes = 0;
    bool used = false;
    cudaEvent_t in_done = nullptr, k_done = nullptr, out_done = nullptr;
  } hs[kHostSlots];
  uint64_t host_tickets = 0;
};

Context g;
char g_err[1024] = "";
thread_local char g_msg[512];

size_t align256(size_t b) { return (b + 255u) & ~(size_t)255u; }

bool is_fatal(cudaError_t e) {
  switch (e) {
    case cudaErrorIllegalAddress:
    case cudaErrorLaunchFailure:
    case cudaErrorIllegalInstruction:
    case cudaErrorMisalignedAddress:
    case cudaErrorAssert:
    case cudaErrorHardwareStackError:
    case cudaErrorInvalidPc:
    case cudaErrorLaunchTimeout:
    case cudaErrorECCUncorrectable:
    case cudaErrorUnknown:
    case cudaErrorContextIsDestroyed:
      return true;
    default:
      return false;
  }
}

// Device memory, or pinned host memory the GPU can address when the device
// is full.
void *alloc_words(uint32_t words, bool *host) {
  size_t bytes = (size_t)(words ? words : 1) * 4u;
  void *p = nullptr;
  *host = false;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e == cudaSuccess) return p;
  cudaGetLastError();
  if (e != cudaErrorMemoryAllocation) return nullptr;
  if (cudaHostAlloc(&p, bytes, cudaHostAllocMapped) == cudaSuccess) {
    *host = true;
    return p;
  }
  cudaGetLastError();
  return nullptr;
}

void free_words(void *p, bool host) {
  if (!p) return;
  if (host) cudaFreeHost(p);
  else cudaFree(p);
}

int ensure_ready() { return g.ready ? NL_OK : nl_init(-1); }

int sync_status(const char *what) {
  const int rc = cuda_status(cudaStreamSynchronize(g.stream), what);
  if (rc == NL_OK && take_wait_timeout())
    return set_error(NL_ERROR, "%s: a kernel's bounded wait timed out; its outputs are invalid",
                     what);
  return rc;
}

void *arena_get(size_t bytes) {
  if (bytes == 0) bytes = 256;
  if (g.arena_bytes >= bytes) return g.arena;
  cudaStreamSynchronize(g.stream);
  if (g.arena) cudaFree(g.arena);
  g.arena = nullptr;
  size_t want = bytes > 2 * g.arena_bytes ? bytes : 2 * g.arena_bytes;
  if (cudaMalloc(&g.arena, want) != cudaSuccess) {
    cudaGetLastError();
    if (cudaMalloc(&g.arena, bytes) != cudaSuccess) {
      cudaGetLastError();
      g.arena_bytes = 0;
      g.arena = nullptr;
      return nullptr;
    }
    want = bytes;
  }
  g.arena_bytes = want;
  return g.arena;
}

int alloc_slot(uint32_t *h) {
  for (uint32_t i = 0; i < g.nres; i++)
    if (!g.res[i].used) { *h = i; return NL_OK; }
  if (g.nres >= NL_MAX_RESIDENT)
    return set_error(NL_ERROR, "resident table full (%d)", NL_MAX_RESIDENT);
  *h = g.nres++;
  return NL_OK;
}

const Resident *resident(uint32_t h) {
  if (h >= NL_MAX_RESIDENT || h >= g.nres || !g.res[h].used) return nullptr;
  return &g.res[h];
}

// ---- dispatch plans shared by OP_BATCH and OP_COMPILE ----------------------
struct Plan {
  std::vector<void *> slot_ptr;
  std::vector<uint32_t> slot_words;
  std::vector<size_t> slot_off;      // arena offset, SIZE_MAX for residents
  std::vector<const OpSpec *> spec;
  std::vector<OpArgs> args;
  size_t owned_bytes = 0;
  size_t scratch_bytes = 0;
};

int build_plan(uint32_t nslot, const nl_slot *slots, uint32_t ndisp,
               const nl_dispatch *disps, Plan &P) {
  if (nslot > NL_MAX_SLOTS)
    return set_error(NL_ERROR, "nslot %u > %d", nslot, NL_MAX_SLOTS);
  if (ndisp > NL_MAX_DISPATCH)
    return set_error(NL_ERROR, "ndisp %u > %d", ndisp, NL_MAX_DISPATCH);
  P.slot_ptr.assign(nslot, nullptr);
  P.slot_words.assign(nslot, 0);
  P.slot_off.assign(nslot, SIZE_MAX);
  for (uint32_t i = 0; i < nslot; i++) {
    if (slots[i].kind == NL_SLOT_RESIDENT) {
      const Resident *r = resident(slots[i].handle);
      if (!r) return set_error(NL_ERROR, "slot %u: bad resident handle %u", i, slots[i].handle);
      P.slot_ptr[i] = r->ptr;
      P.slot_words[i] = r->words;
    } else if (slots[i].kind <= NL_SLOT_OUT) {
      P.slot_words[i] = slots[i].size;
      P.slot_off[i] = P.owned_bytes;
      P.owned_bytes += align256((size_t)(slots[i].size ? slots[i].size : 1) * 4u);
    } else {
      return set_error(NL_ERROR, "slot %u: bad kind %u", i, slots[i].kind);
    }
  }
  P.spec.resize(ndisp);
  P.args.resize(ndisp);
  for (uint32_t d = 0; d < ndisp; d++) {
    const nl_dispatch &D = disps[d];
    char name[NL_MAX_NAME + 1];
    memcpy(name, D.name, NL_MAX_NAME);
    name[NL_MAX_NAME] = 0;
    const OpSpec *s = find_op(name);
    if (!s) return set_error(NL_ERROR, "dispatch %u: unknown kernel '%s'", d, name);
    if (D.nbuf != s->nbuf || D.npush < s->npush || D.npush > NL_MAX_PUSH)
      return set_error(NL_ERROR, "dispatch %u: %s takes %u buffers and %u push constants, got %u and %u",
                       d, name, s->nbuf, s->npush, D.nbuf, D.npush);
    OpArgs &a = P.args[d];
    memset(&a, 0, sizeof(a));
    a.nbuf = D.nbuf;
    a.npush = D.npush;
    memcpy(a.push, D.push, sizeof(uint32_t) * D.npush);
    a.groups = D.groups;
    for (uint32_t b = 0; b < D.nbuf; b++) {
      if (D.slot[b] >= nslot)
        return set_error(NL_ERROR, "dispatch %u (%s): slot index %u >= nslot %u", d, name, D.slot[b], nslot);
      a.words[b] = P.slot_words[D.slot[b]];
    }
    const char *m = s->check(a);
    if (m) return set_error(NL_ERROR, "dispatch %u (%s): %s", d, name, m);
    size_t sc = s->scratch(a);
    if (sc > P.scratch_bytes) P.scratch_bytes = sc;
    P.spec[d] = s;
  }
  return NL_OK;
}

void bind_plan(Plan &P, char *base, const nl_dispatch *disps, void *scratch) {
  for (size_t i = 0; i < P.slot_ptr.size(); i++)
    if (P.slot_off[i] != SIZE_MAX) P.slot_ptr[i] = base + P.slot_off[i];
  for (size_t d = 0; d < P.args.size(); d++) {
    OpArgs &a = P.args[d];
    for (uint32_t b = 0; b < a.nbuf; b++) a.buf[b] = P.slot_ptr[disps[d].slot[b]];
    a.stream = g.stream;
    a.scratch = scratch;
    a.scratch_bytes = P.scratch_bytes;
  }
}

int launch_plan(Plan &P) {
  for (size_t d = 0; d < P.args.size(); d++) {
    cudaError_t e = P.spec[d]->launch(P.args[d]);
    if (e != cudaSuccess) return cuda_status(e, P.spec[d]->name);
  }
  return NL_OK;
}

}  // namespace

// ---- error and accounting helpers --------------------------------------------
int set_error(int code, const char *fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

int cuda_status(cudaError_t e, const char *what) {
  if (e == cudaSuccess) return NL_OK;
  bool fatal = is_fatal(e);
  if (!fatal) cudaGetLastError();  // clear a non-sticky error
  return set_error(fatal ? NL_FATAL : NL_ERROR, "%s: %s (%s)", what,
                   cudaGetErrorString(e), cudaGetErrorName(e));
}

void count_launches(uint64_t n) {
  if (g.capturing) g.capture_launches += n;
  else g.launches += n;
}

const char *fmt_msg(const char *fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_msg, sizeof(g_msg), fmt, ap);
  va_end(ap);
  return g_msg;
}

const char *need_words(const OpArgs &a, uint32_t b, uint64_t need,
                       const char *what) {
  if (b >= a.nbuf) return fmt_msg("buffer %u (%s) missing", b, what);
  if ((uint64_t)a.words[b] < need)
    return fmt_msg("buffer %u (%s) holds %u words, the push constants need %llu",
                   b, what, a.words[b], (unsigned long long)need);
  return nullptr;
}

void *library_workspace(size_t bytes, cudaStream_t stream) {
  if (bytes == 0) bytes = 256;
  if (g.ws_bytes >= bytes) return g.ws;
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(stream, &cs) != cudaSuccess || cs != cudaStreamCaptureStatusNone) {
    cudaGetLastError();
    return nullptr;   // growing would allocate inside a capture
  }
  cudaDeviceSynchronize();   // the old workspace may still be in use
  if (g.ws) cudaFree(g.ws);
  g.ws = nullptr;
  size_t want = bytes > 2 * g.ws_bytes ? bytes : 2 * g.ws_bytes;
  if (cudaMalloc(&g.ws, want) != cudaSuccess) {
    cudaGetLastError();
    g.ws_bytes = 0;
    g.ws = nullptr;
    return nullptr;
  }
  g.ws_bytes = want;
  return g.ws;
}

// ---- bounded-wait flag ----------------------------------------------------------
namespace {
int *g_wait_host = nullptr, *g_wait_dev = nullptr;
}  // namespace

int *wait_flag_device() {
  if (!g_wait_host) {
    int *h = nullptr;
    if (cudaHostAlloc((void **)&h, sizeof(int), cudaHostAllocMapped | cudaHostAllocPortable) !=
        cudaSuccess) {
      cudaGetLastError();
      return nullptr;
    }
    *h = 0;
    int *d = nullptr;
    if (cudaHostGetDevicePointer((void **)&d, h, 0) != cudaSuccess) {
      cudaGetLastError();
      cudaFreeHost(h);
      return nullptr;
    }
    g_wait_dev = d;
    g_wait_host = h;
  }
  return g_wait_dev;
}

int *wait_flag_if_allocated() { return g_wait_dev; }

bool take_wait_timeout() {
  if (!g_wait_host || !*(volatile int *)g_wait_host) return false;
  *(volatile int *)g_wait_host = 0;
  return true;
}

}  // namespace nl

using namespace nl;

// ---- context ------------------------------------------------------------------
extern "C" int nl_init(int device) {
  if (g.ready) return NL_OK;
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  if (e != cudaSuccess || n == 0)
    return set_error(NL_FATAL, "no CUDA device (%s)", cudaGetErrorString(e));
  int pick = device;
  if (pick < 0) {
    const char *env = getenv("NELISP_GPU_DEVICE");
    pick = env ? atoi(env) : 0;
  }
  if (pick < 0 || pick >= n) pick = 0;   // host/vkserver.c:223
  if ((e = cudaSetDevice(pick)) != cudaSuccess) return cuda_status(e, "cudaSetDevice");
  if ((e = cudaFree(0)) != cudaSuccess) return cuda_status(e, "context");
  if ((e = cudaStreamCreateWithFlags(&g.stream, cudaStreamNonBlocking)) != cudaSuccess)
    return cuda_status(e, "cudaStreamCreate");
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, pick) == cudaSuccess)
    snprintf(g.devname, sizeof(g.devname), "%s", prop.name);
  g.device = pick;
  wait_flag_device();             // before any stream capture
  g.ready = true;
  return NL_OK;
}

extern "C" void nl_shutdown(void) {
  if (!g.ready) return;
  cudaStreamSynchronize(g.stream);
  for (uint32_t h = 0; h < NL_MAX_COMPILED; h++) nl_free_compiled(h);
  for (uint32_t h = 0; h < g.nres; h++) nl_free(h);
  g.nres = 0;
  if (g.arena) cudaFree(g.arena);
  if (g.ws) cudaFree(g.ws);
  for (Context::HostSlot &hs : g.hs) {
    if (hs.buf) cudaFree(hs.buf);
    for (cudaEvent_t *ev : {&hs.in_done, &hs.k_done, &hs.out_done})
      if (*ev) cudaEventDestroy(*ev);
    hs = Context::HostSlot();
  }
  g.host_tickets = 0;
  if (g.h2d) cudaStreamDestroy(g.h2d);
  if (g.d2h) cudaStreamDestroy(g.d2h);
  g.h2d = g.d2h = nullptr;
  if (g.stage) cudaFreeHost(g.stage);
  g.arena = g.ws = g.stage = nullptr;
  g.arena_bytes = g.ws_bytes = 0;
  cudaStreamDestroy(g.stream);
  g.stream = nullptr;
  g.ready = false;
  g.device = -1;
}

extern "C" const char *nl_last_error(void) { return g_err; }
extern "C" const char *nl_version(void) { return "libnelisp_cuda 0.1 (sm_100a)"; }
extern "C" int nl_device(void) { return g.ready ? g.device : -1; }
extern "C" const char *nl_device_name(void) { return g.devname; }
extern "C" uint64_t nl_launch_count(void) { return g.launches; }

extern "C" int nl_kernel_count(void) { return op_count(); }
extern "C" const char *nl_kernel_name(int index) {
  const OpSpec *s = op_at(index);
  return s ? s->name : nullptr;
}
extern "C" int nl_kernel_arity(const char *name, uint32_t *nbuf, uint32_t *npush) {
  const OpSpec *s = find_op(name);
  if (!s) return set_error(NL_ERROR, "unknown kernel '%s'", name ? name : "(null)");
  if (nbuf) *nbuf = s->nbuf;
  if (npush) *npush = s->npush;
  return NL_OK;
}

// ---- resident buffers ----------------------------------------------------------
extern "C" int nl_upload(const void *words, uint32_t nwords, uint32_t *handle) {
  int rc = ensure_ready();
  if (rc) return rc;
  uint32_t h = 0;
  if ((rc = alloc_slot(&h))) return rc;
  Resident &r = g.res[h];
  r.ptr = alloc_words(nwords, &r.host);
  if (!r.ptr) return set_error(NL_ERROR, "upload: cannot allocate %u words", nwords);
  if (nwords) {
    cudaError_t e = cudaMemcpy(r.ptr, words, (size_t)nwords * 4u, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
      free_words(r.ptr, r.host);
      r.ptr = nullptr;
      return cuda_status(e, "upload");
    }
  }
  r.words = nwords;
  r.used = true;
  *handle = h;
  return NL_OK;
}

namespace nl {
namespace {

// ---- file -> device at NVMe speed ---------------------------------------------
// host/vkserver.c:371-410 freads the region into mapped memory in one call.
// Here the region streams through kReadSlots pinned slots of kReadSlot bytes:
// each slot is filled by kReadThreads parallel preads (several requests in
// flight keep an NVMe queue busy) and copied to the device asynchronously, so
// the copy of one slot overlaps the reads of the next.  The file is opened
// with O_DIRECT where the file system takes it (no page-cache copy); reads
// then start on a 4 KiB boundary and the slot's leading bytes are skipped.
constexpr size_t kReadSlot = 16u << 20;
constexpr int kReadSlots = 4;                  // kReadSlots * kReadSlot = kStageBytes
constexpr int kReadThreads = 4;
constexpr size_t kDirectAlign = 4096;
static_assert(kReadSlots * kReadSlot == kStageBytes, "staging layout");

struct FileReader {
  int fd = -1;
  bool direct = false;
  ~FileReader() {
    if (fd >= 0) close(fd);
  }
  bool open_path(const char *path) {
#ifdef O_DIRECT
    fd = open(path, O_RDONLY | O_DIRECT);
    if (fd >= 0) {
      direct = true;
      return true;
    }
#endif
    fd = open(path, O_RDONLY);
    direct = false;
    return fd >= 0;
  }
  void reopen_buffered(const char *path) {
    if (fd >= 0) close(fd);
    fd = open(path, O_RDONLY);
    direct = false;
  }
};

// Reads [off, off + len) into buf with kReadThreads parallel preads; returns
// the bytes read before the first short read (EOF), or -1 on an I/O error.
long long read_span(int fd, char *buf, uint64_t off, size_t len, int *err_no) {
  const size_t part = ((len + kReadThreads - 1) / kReadThreads + kDirectAlign - 1) &
                      ~(kDirectAlign - 1);
  long long got[kReadThreads] = {0};
  int errs[kReadThreads] = {0};
  std::thread th[kReadThreads];
  int nth = 0;
  for (int t = 0; t < kReadThreads; t++) {
    const size_t b = (size_t)t * part;
    if (b >= len) break;
    const size_t n = b + part <= len ? part : len - b;
    th[nth++] = std::thread([=, &got, &errs] {
      size_t done = 0;
      while (done < n) {
        const ssize_t r = pread(fd, buf + b + done, n - done, (off_t)(off + b + done));
        if (r < 0) {
          if (errno == EINTR) continue;
          errs[t] = errno;
          break;
        }
        if (r == 0) break;
        done += (size_t)r;
      }
      got[t] = (long long)done;
    });
  }
  for (int t = 0; t < nth; t++) th[t].join();
  long long total = 0;
  for (int t = 0; t < nth; t++) {
    if (errs[t]) {
      *err_no = errs[t];
      return -1;
    }
    total += got[t];
    const size_t b = (size_t)t * part, n = b + part <= len ? part : len - b;
    if ((size_t)got[t] < n) break;            // EOF inside this part
  }
  return total;
}

}  // namespace

// Copies NBYTES at OFFSET of PATH to device memory DST.  Returns NL_OK, or
// NL_ERROR with a message (*MISSING_WORDS set on a short file).
namespace {
int file_to_device_impl(const char *path, uint64_t offset, size_t nbytes, void *dst,
                        uint64_t *missing_words, bool allow_direct) {
  *missing_words = 0;
  FileReader fr;
  if (allow_direct ? !fr.open_path(path) : (fr.reopen_buffered(path), fr.fd < 0))
    return set_error(NL_ERROR, "cannot open %s: %s", path, strerror(errno));
  if (nbytes == 0) return NL_OK;
  if (!g.stage && cudaHostAlloc(&g.stage, kStageBytes, cudaHostAllocDefault) != cudaSuccess) {
    cudaGetLastError();
    g.stage = nullptr;
  }
  if (!g.stage) return set_error(NL_ERROR, "upload-file: no pinned staging memory");
  if (!g.h2d && cudaStreamCreateWithFlags(&g.h2d, cudaStreamNonBlocking) != cudaSuccess)
    return cuda_status(cudaGetLastError(), "upload-file: stream");
  static cudaEvent_t slot_ev[kReadSlots] = {};
  for (cudaEvent_t &ev : slot_ev)
    if (!ev && cudaEventCreateWithFlags(&ev, cudaEventDisableTiming) != cudaSuccess)
      return cuda_status(cudaGetLastError(), "upload-file: events");
  const uint64_t start = fr.direct ? offset & ~(uint64_t)(kDirectAlign - 1) : offset;
  const size_t skew = (size_t)(offset - start);
  const uint64_t span = skew + nbytes;           // bytes of file from START that matter
  uint64_t done = 0;                              // file bytes consumed from START
  for (int slot = 0; done < span; slot = (slot + 1) % kReadSlots) {
    char *buf = (char *)g.stage + (size_t)slot * kReadSlot;
    cudaError_t e = cudaEventSynchronize(slot_ev[slot]);   // its previous copy is done
    if (e != cudaSuccess) return cuda_status(e, "upload-file");
    size_t want = span - done < kReadSlot ? (size_t)(span - done) : kReadSlot;
    size_t req = fr.direct ? (want + kDirectAlign - 1) & ~(kDirectAlign - 1) : want;
    int err_no = 0;
    long long got = read_span(fr.fd, buf, start + done, req, &err_no);
    if (got < 0 && fr.direct && err_no == EINVAL && done == 0)   // O_DIRECT refused
      return file_to_device_impl(path, offset, nbytes, dst, missing_words, false);
    if (got < 0) return set_error(NL_ERROR, "read %s: %s", path, strerror(err_no));
    const size_t use = (size_t)got < want ? (size_t)got : want;
    // device bytes: file [start + done + lo, start + done + use) minus the skew
    const size_t lo = done < skew ? (size_t)(skew - done) : 0;
    if (use > lo) {
      const uint64_t dpos = done + lo - skew;
      if ((e = cudaMemcpyAsync((char *)dst + dpos, buf + lo, use - lo, cudaMemcpyHostToDevice,
                               g.h2d)) != cudaSuccess ||
          (e = cudaEventRecord(slot_ev[slot], g.h2d)) != cudaSuccess)
        return cuda_status(e, "upload-file");
    }
    done += use;
    if (use < want) {                            // short file
      const uint64_t have = done > skew ? done - skew : 0;
      *missing_words = (nbytes - have + 3) / 4u;
      cudaStreamSynchronize(g.h2d);
      return set_error(NL_ERROR, "%s short read, %llu words missing", path,
                       (unsigned long long)*missing_words);
    }
  }
  return cuda_status(cudaStreamSynchronize(g.h2d), "upload-file");
}
}  // namespace

int file_to_device(const char *path, uint64_t offset, size_t nbytes, void *dst,
                   uint64_t *missing_words) {
  return file_to_device_impl(path, offset, nbytes, dst, missing_words, true);
}

}  // namespace nl

extern "C" int nl_upload_file(const char *path, uint64_t offset, uint32_t nwords,
                              uint32_t *handle) {
  int rc = ensure_ready();
  if (rc) return rc;
  {
    // the reference opens and seeks before allocating (host/vkserver.c:384-386)
    FileReader probe;
    if (!probe.open_path(path))
      return set_error(NL_ERROR, "cannot open %s: %s", path, strerror(errno));
  }
  uint32_t h = 0;
  if ((rc = alloc_slot(&h))) return rc;
  Resident &r = g.res[h];
  r.ptr = alloc_words(nwords, &r.host);
  if (!r.ptr && nwords) return set_error(NL_ERROR, "upload-file: cannot allocate %u words", nwords);
  r.words = nwords;
  r.used = true;
  uint64_t missing = 0;
  rc = file_to_device(path, offset, (size_t)nwords * 4u, r.ptr, &missing);
  if (rc != NL_OK) {
    char msg[1024];
    snprintf(msg, sizeof(msg), "%s", nl_last_error());
    nl_free(h);
    return set_error(rc, "%s", msg);
  }
  *handle = h;
  return NL_OK;
}

extern "C" int nl_upload_file_ternary(const char *path, uint64_t offset, uint32_t rows,
                                      uint32_t cols, int per_row, uint32_t *h_wp,
                                      uint32_t *h_s) {
  int rc = ensure_ready();
  if (rc) return rc;
  if (!h_wp || !h_s) return set_error(NL_ERROR, "upload-file-ternary: null handle pointer");
  if (!rows || !cols) return set_error(NL_ERROR, "upload-file-ternary: empty matrix");
  const uint64_t wng = (cols + 15u) / 16u, wwords = (uint64_t)rows * wng;
  if (wwords > 0xffffffffull) return set_error(NL_ERROR, "upload-file-ternary: too large");
  const size_t fbytes = (size_t)rows * cols * 4u;
  void *tmp = nullptr;
  const size_t scratch = quant_w_scratch_bytes(rows);
  cudaError_t e = cudaMalloc(&tmp, align256(fbytes) + scratch);
  if (e != cudaSuccess) return cuda_status(e, "upload-file-ternary: f32 staging");
  uint64_t missing = 0;
  if ((rc = file_to_device(path, offset, fbytes, tmp, &missing)) != NL_OK) {
    cudaFree(tmp);
    return rc;
  }
  uint32_t hw = 0, hs = 0;
  if ((rc = alloc_slot(&hw))) { cudaFree(tmp); return rc; }
  Resident &rw = g.res[hw];
  rw.ptr = alloc_words((uint32_t)wwords, &rw.host);
  rw.words = (uint32_t)wwords;
  rw.used = true;
  if ((rc = alloc_slot(&hs))) { nl_free(hw); cudaFree(tmp); return rc; }
  Resident &rs = g.res[hs];
  rs.ptr = alloc_words(rows, &rs.host);
  rs.words = rows;
  rs.used = true;
  if (!rw.ptr || !rs.ptr) {
    nl_free(hw);
    nl_free(hs);
    cudaFree(tmp);
    return set_error(NL_ERROR, "upload-file-ternary: cannot allocate the packed weights");
  }
  e = quant_w_pack_launch((const float *)tmp, rows, cols, per_row != 0, (uint32_t *)rw.ptr,
                          (float *)rs.ptr, (char *)tmp + align256(fbytes), g.stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(g.stream);
  cudaFree(tmp);
  if (e != cudaSuccess) {
    nl_free(hw);
    nl_free(hs);
    return cuda_status(e, "upload-file-ternary");
  }
  *h_wp = hw;
  *h_s = hs;
  return NL_OK;
}

extern "C" int nl_write_resident(uint32_t handle, const void *words, uint32_t nwords) {
  int rc = ensure_ready();
  if (rc) return rc;
  const Resident *r = resident(handle);
  if (!r) return set_error(NL_ERROR, "write bad resident %u", handle);
  if (nwords > r->words)
    return set_error(NL_ERROR, "write %u words into resident %u of %u words", nwords, handle, r->words);
  if (!nwords) return NL_OK;
  return cuda_status(cudaMemcpy(r->ptr, words, (size_t)nwords * 4u, cudaMemcpyHostToDevice),
                     "write-resident");
}

extern "C" int nl_read_resident(uint32_t handle, void *words, uint32_t nwords) {
  int rc = ensure_ready();
  if (rc) return rc;
  const Resident *r = resident(handle);
  if (!r) return set_error(NL_ERROR, "read bad resident %u", handle);
  if (nwords > r->words)
    return set_error(NL_ERROR, "read %u words from resident %u of %u words", nwords, handle, r->words);
  if (!nwords) return NL_OK;
  cudaStreamSynchronize(g.stream);
  return cuda_status(cudaMemcpy(words, r->ptr, (size_t)nwords * 4u, cudaMemcpyDeviceToHost),
                     "read-resident");
}

extern "C" int nl_free(uint32_t handle) {
  if (!g.ready) return NL_OK;
  if (handle < g.nres && g.res[handle].used) {
    cudaStreamSynchronize(g.stream);
    Resident &r = g.res[handle];
    free_words(r.ptr, r.host);
    r.ptr = nullptr;
    r.words = 0;
    r.used = false;
    r.host = false;
  }
  return NL_OK;
}

extern "C" int nl_resident_info(uint32_t handle, void **dev_ptr, uint32_t *nwords) {
  const Resident *r = resident(handle);
  if (!r) return set_error(NL_ERROR, "bad resident %u", handle);
  if (dev_ptr) *dev_ptr = r->ptr;
  if (nwords) *nwords = r->words;
  return NL_OK;
}

// ---- OP_RUN --------------------------------------------------------------------
extern "C" int nl_run(const char *name, uint32_t nbuf, const nl_run_buffer *bufs,
                      uint32_t npush, const uint32_t *push, uint32_t groups,
                      const void *inline_words, void *out_words) {
  int rc = ensure_ready();
  if (rc) return rc;
  const OpSpec *s = find_op(name);
  if (!s) return set_error(NL_ERROR, "unknown kernel '%s'", name ? name : "(null)");
  if (nbuf > NL_MAX_BUFS || npush > NL_MAX_PUSH || nbuf != s->nbuf || npush < s->npush)
    return set_error(NL_ERROR, "%s takes %u buffers and %u push constants, got %u and %u",
                     s->name, s->nbuf, s->npush, nbuf, npush);
  OpArgs a;
  memset(&a, 0, sizeof(a));
  a.nbuf = nbuf;
  a.npush = npush;
  if (npush) memcpy(a.push, push, sizeof(uint32_t) * npush);
  a.groups = groups;
  a.stream = g.stream;
  size_t off[NL_MAX_BUFS], total = 0;
  for (uint32_t i = 0; i < nbuf; i++) {
    uint32_t k = bufs[i].kind;
    if (k == NL_RUN_RESIDENT) {
      const Resident *r = resident(bufs[i].handle);
      if (!r) return set_error(NL_ERROR, "buffer %u: bad resident handle %u", i, bufs[i].handle);
      a.buf[i] = r->ptr;
      a.words[i] = r->words;
      off[i] = SIZE_MAX;
    } else if (k == NL_RUN_IN || k == NL_RUN_OUT || k == NL_RUN_INOUT) {
      a.words[i] = bufs[i].size;
      off[i] = total;
      total += align256((size_t)(bufs[i].size ? bufs[i].size : 1) * 4u);
    } else {
      return set_error(NL_ERROR, "buffer %u: bad kind %u", i, k);
    }
  }
  const char *m = s->check(a);
  if (m) return set_error(NL_ERROR, "%s: %s", s->name, m);
  size_t sc = s->scratch(a);
  char *base = (char *)arena_get(total + align256(sc));
  if (!base) return set_error(NL_ERROR, "run: cannot allocate %zu bytes", total + sc);
  const char *src = (const char *)inline_words;
  for (uint32_t i = 0; i < nbuf; i++) {
    if (off[i] == SIZE_MAX) continue;
    a.buf[i] = base + off[i];
    size_t bytes = (size_t)bufs[i].size * 4u;
    cudaError_t e = cudaSuccess;
    if (bufs[i].kind == NL_RUN_OUT) {
      if (bytes) e = cudaMemsetAsync(a.buf[i], 0, bytes, g.stream);
    } else if (bytes) {
      e = cudaMemcpyAsync(a.buf[i], src, bytes, cudaMemcpyHostToDevice, g.stream);
      src += bytes;
    }
    if (e != cudaSuccess) return cuda_status(e, "run: input copy");
  }
  a.scratch = sc ? base + total : nullptr;
  a.scratch_bytes = sc;
  cudaError_t e = s->launch(a);
  if (e != cudaSuccess) return cuda_status(e, s->name);
  char *dst = (char *)out_words;
  for (uint32_t i = 0; i < nbuf; i++) {
    uint32_t k = bufs[i].kind;
    if (k != NL_RUN_OUT && k != NL_RUN_INOUT) continue;
    size_t bytes = (size_t)bufs[i].size * 4u;
    if (bytes) {
      e = cudaMemcpyAsync(dst, a.buf[i], bytes, cudaMemcpyDeviceToHost, g.stream);
      if (e != cudaSuccess) return cuda_status(e, "run: output copy");
    }
    dst += bytes;
  }
  return sync_status(s->name);
}

// ---- OP_BATCH -------------------------------------------------------------------
extern "C" int nl_batch(uint32_t nslot, const nl_slot *slots, uint32_t ndisp,
                        const nl_dispatch *disps, const void *inline_words,
                        void *out_words) {
  int rc = ensure_ready();
  if (rc) return rc;
  Plan P;
  if ((rc = build_plan(nslot, slots, ndisp, disps, P))) return rc;
  char *base = (char *)arena_get(P.owned_bytes + align256(P.scratch_bytes));
  if (!base) return set_error(NL_ERROR, "batch: cannot allocate %zu bytes", P.owned_bytes);
  bind_plan(P, base, disps, P.scratch_bytes ? base + P.owned_bytes : nullptr);
  const char *src = (const char *)inline_words;
  for (uint32_t i = 0; i < nslot; i++) {
    if (slots[i].kind == NL_SLOT_RESIDENT) continue;
    size_t bytes = (size_t)slots[i].size * 4u;
    if (!bytes) continue;
    cudaError_t e;
    if (slots[i].kind == NL_SLOT_IN) {
      e = cudaMemcpyAsync(P.slot_ptr[i], src, bytes, cudaMemcpyHostToDevice, g.stream);
      src += bytes;
    } else {
      e = cudaMemsetAsync(P.slot_ptr[i], 0, bytes, g.stream);
    }
    if (e != cudaSuccess) return cuda_status(e, "batch: slot setup");
  }
  if ((rc = launch_plan(P))) return rc;
  char *dst = (char *)out_words;
  for (uint32_t i = 0; i < nslot; i++) {
    if (slots[i].kind != NL_SLOT_OUT) continue;
    size_t bytes = (size_t)slots[i].size * 4u;
    if (bytes) {
      cudaError_t e = cudaMemcpyAsync(dst, P.slot_ptr[i], bytes, cudaMemcpyDeviceToHost, g.stream);
      if (e != cudaSuccess) return cuda_status(e, "batch: output copy");
    }
    dst += bytes;
  }
  return sync_status("batch");
}

// ---- OP_COMPILE / OP_RUN_COMPILED / OP_FREE_COMPILED ----------------------------
extern "C" int nl_compile(uint32_t nslot, const nl_slot *slots, uint32_t ndisp,
                          const nl_dispatch *disps, const void *inline_words,
                          uint32_t *handle) {
  int rc = ensure_ready();
  if (rc) return rc;
  int c = -1;
  for (int i = 0; i < NL_MAX_COMPILED; i++)
    if (!g.comp[i].used) { c = i; break; }
  if (c < 0) return set_error(NL_ERROR, "compiled table full (%d)", NL_MAX_COMPILED);
  Plan P;
  if ((rc = build_plan(nslot, slots, ndisp, disps, P))) return rc;
  Compiled &C = g.comp[c];
  size_t total = P.owned_bytes + align256(P.scratch_bytes);
  bool host = false;
  void *mem = alloc_words((uint32_t)ceil_div64(total, 4), &host);
  if (!mem) return set_error(NL_ERROR, "compile: cannot allocate %zu bytes", total);
  bind_plan(P, (char *)mem, disps, P.scratch_bytes ? (char *)mem + P.owned_bytes : nullptr);
  // Inline inputs are written once, as the reference writes them at compile time.
  const char *src = (const char *)inline_words;
  for (uint32_t i = 0; i < nslot; i++) {
    if (slots[i].kind != NL_SLOT_IN) continue;
    size_t bytes = (size_t)slots[i].size * 4u;
    if (bytes) {
      cudaError_t e = cudaMemcpy(P.slot_ptr[i], src, bytes, cudaMemcpyHostToDevice);
      if (e != cudaSuccess) { free_words(mem, host); return cuda_status(e, "compile: input copy"); }
    }
    src += bytes;
  }
  cudaStreamSynchronize(g.stream);
  cudaGraph_t graph = nullptr;
  cudaError_t e = cudaStreamBeginCapture(g.stream, cudaStreamCaptureModeThreadLocal);
  if (e != cudaSuccess) { free_words(mem, host); return cuda_status(e, "compile: capture"); }
  g.capturing = true;
  g.capture_launches = 0;
  rc = NL_OK;
  for (uint32_t i = 0; i < nslot && rc == NL_OK; i++) {
    if (slots[i].kind != NL_SLOT_TMP && slots[i].kind != NL_SLOT_OUT) continue;
    size_t bytes = (size_t)slots[i].size * 4u;
    if (bytes) rc = cuda_status(cudaMemsetAsync(P.slot_ptr[i], 0, bytes, g.stream), "compile: memset");
  }
  if (rc == NL_OK) rc = launch_plan(P);
  g.capturing = false;
  e = cudaStreamEndCapture(g.stream, &graph);
  if (rc == NL_OK && e != cudaSuccess) rc = cuda_status(e, "compile: end capture");
  cudaGraphExec_t exec = nullptr;
  if (rc == NL_OK) {
    e = cudaGraphInstantiate(&exec, graph, 0);
    if (e != cudaSuccess) rc = cuda_status(e, "compile: instantiate");
  }
  if (graph) cudaGraphDestroy(graph);
  if (rc != NL_OK) {
    if (exec) cudaGraphExecDestroy(exec);
    free_words(mem, host);
    return rc;
  }
  C.used = true;
  C.exec = exec;
  C.mem = mem;
  C.mem_host = host;
  C.slot_ptr = P.slot_ptr;
  C.slot_words = P.slot_words;
  C.out_slots.clear();
  C.out_words = 0;
  for (uint32_t i = 0; i < nslot; i++)
    if (slots[i].kind == NL_SLOT_OUT) { C.out_slots.push_back(i); C.out_words += slots[i].size; }
  C.kernels = g.capture_launches;
  *handle = (uint32_t)c;
  return NL_OK;
}

extern "C" int nl_run_compiled(uint32_t handle, void *out_words) {
  int rc = ensure_ready();
  if (rc) return rc;
  if (handle >= NL_MAX_COMPILED || !g.comp[handle].used)
    return set_error(NL_ERROR, "bad compiled %u", handle);
  Compiled &C = g.comp[handle];
  cudaError_t e = cudaGraphLaunch(C.exec, g.stream);
  if (e != cudaSuccess) return cuda_status(e, "run-compiled");
  count_launches(C.kernels);
  char *dst = (char *)out_words;
  for (uint32_t i : C.out_slots) {
    size_t bytes = (size_t)C.slot_words[i] * 4u;
    if (bytes) {
      e = cudaMemcpyAsync(dst, C.slot_ptr[i], bytes, cudaMemcpyDeviceToHost, g.stream);
      if (e != cudaSuccess) return cuda_status(e, "run-compiled: output copy");
    }
    dst += bytes;
  }
  return sync_status("run-compiled");
}

extern "C" int nl_free_compiled(uint32_t handle) {
  if (!g.ready) return NL_OK;
  if (handle < NL_MAX_COMPILED && g.comp[handle].used) {
    Compiled &C = g.comp[handle];
    cudaStreamSynchronize(g.stream);
    cudaGraphExecDestroy(C.exec);
    free_words(C.mem, C.mem_host);
    C = Compiled();
  }
  return NL_OK;
}

extern "C" int nl_compiled_out_words(uint32_t handle, uint64_t *nwords) {
  if (handle >= NL_MAX_COMPILED || !g.comp[handle].used)
    return set_error(NL_ERROR, "bad compiled %u", handle);
  *nwords = g.comp[handle].out_words;
  return NL_OK;
}

extern "C" int nl_time_compiled(uint32_t handle, uint32_t reps, double *ms_per_rep) {
  int rc = ensure_ready();
  if (rc) return rc;
  if (handle >= NL_MAX_COMPILED || !g.comp[handle].used)
    return set_error(NL_ERROR, "bad compiled %u", handle);
  if (reps == 0) reps = 1;
  Compiled &C = g.comp[handle];
  cudaEvent_t e0, e1;
  cudaEventCreate(&e0);
  cudaEventCreate(&e1);
  cudaEventRecord(e0, g.stream);
  for (uint32_t r = 0; r < reps; r++) cudaGraphLaunch(C.exec, g.stream);
  cudaEventRecord(e1, g.stream);
  rc = sync_status("time-compiled");
  float ms = 0.0f;
  cudaEventElapsedTime(&ms, e0, e1);
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  count_launches(C.kernels * reps);
  if (ms_per_rep) *ms_per_rep = (double)ms / reps;
  return rc;
}

// ---- device-pointer dispatch ------------------------------------------------------
extern "C" int nl_dispatch_dev(const char *name, uint32_t nbuf, void *const *bufs,
                               const uint32_t *nwords, uint32_t npush,
                               const uint32_t *push, uint32_t groups, void *stream) {
  int rc = ensure_ready();
  if (rc) return rc;
  const OpSpec *s = find_op(name);
  if (!s) return set_error(NL_ERROR, "unknown kernel '%s'", name ? name : "(null)");
  if (nbuf > NL_MAX_BUFS || npush > NL_MAX_PUSH || nbuf != s->nbuf || npush < s->npush)
    return set_error(NL_ERROR, "%s takes %u buffers and %u push constants, got %u and %u",
                     s->name, s->nbuf, s->npush, nbuf, npush);
  OpArgs a;
  memset(&a, 0, sizeof(a));
  a.nbuf = nbuf;
  a.npush = npush;
  if (npush) memcpy(a.push, push, sizeof(uint32_t) * npush);
  a.groups = groups;
  a.stream = (cudaStream_t)stream;
  for (uint32_t i = 0; i < nbuf; i++) {
    a.buf[i] = bufs[i];
    a.words[i] = nwords[i];
  }
  const char *m = s->check(a);
  if (m) return set_error(NL_ERROR, "%s: %s", s->name, m);
  size_t sc = s->scratch(a);
  if (sc) {
    a.scratch = library_workspace(sc, a.stream);
    if (!a.scratch) return set_error(NL_ERROR, "%s: no workspace of %zu bytes", s->name, sc);
    a.scratch_bytes = sc;
  }
  return cuda_status(s->launch(a), s->name);
}

// ---- typed entry points -------------------------------------------------------------
extern "C" size_t nl_ternary_workspace_bytes(uint32_t seq, uint32_t cols) {
  return ternary_ws_bytes_best(1, seq, cols, false);
}

// The (cos, sin) table of the fused decode attention, kept for the last
// (maxseq, head size, base) asked for.
namespace {
struct RopeTable {
  float2 *tab = nullptr;
  uint32_t maxseq = 0, hd = 0;
  float base = 0.0f;
} g_rope;
}  // namespace

extern "C" int nl_decode_attn_rope_dev(const float *QKV, float *CK, float *CV, const int32_t *POS,
                                       float *C, uint32_t batch, uint32_t heads,
                                       uint32_t kv_heads, uint32_t head_dim, uint32_t max_seq,
                                       float rope_base, void *stream) {
  int rc = ensure_ready();
  if (rc) return rc;
  if (batch == 0) return NL_OK;
  if (heads == 0 || kv_heads == 0 || max_seq == 0 || heads % kv_heads)
    return set_error(NL_ERROR, "decode-attn-rope: heads %u, kv heads %u, max_seq %u", heads,
                     kv_heads, max_seq);
  const AttnGeom geo = attn_geom(batch, heads * head_dim, heads, kv_heads, max_seq,
                                 (uint64_t)batch * max_seq * kv_heads * head_dim);
  const size_t scr = attn_rope_scratch_bytes(geo);
  if (!scr)
    return set_error(NL_ERROR,
                     "decode-attn-rope: head size %u (32, 64, 128 or 256) with at most 8 query "
                     "heads per kv head",
                     head_dim);
  if (((uintptr_t)CK | (uintptr_t)CV) & 15u)
    return set_error(NL_ERROR, "decode-attn-rope: the caches must be 16-byte aligned");
  cudaStream_t st = (cudaStream_t)stream;
  if (!g_rope.tab || g_rope.maxseq < max_seq || g_rope.hd != head_dim ||
      g_rope.base != rope_base) {
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(st, &cs) != cudaSuccess || cs != cudaStreamCaptureStatusNone) {
      cudaGetLastError();
      return set_error(NL_ERROR, "decode-attn-rope: first call for this shape inside a capture");
    }
    cudaDeviceSynchronize();   // the old table may still be read
    if (g_rope.tab) cudaFree(g_rope.tab);
    g_rope = RopeTable{};
    void *p = nullptr;
    cudaError_t e = cudaMalloc(&p, (size_t)max_seq * (head_dim / 2) * sizeof(float2));
    if (e != cudaSuccess) return cuda_status(e, "decode-attn-rope: table");
    if ((e = rope_table_launch((float2 *)p, max_seq, head_dim, rope_base, st)) != cudaSuccess) {
      cudaFree(p);
      return cuda_status(e, "decode-attn-rope: table");
    }
    g_rope.tab = (float2 *)p;
    g_rope.maxseq = max_seq;
    g_rope.hd = head_dim;
    g_rope.base = rope_base;
  }
  void *ws = library_workspace(scr, st);
  if (!ws) return set_error(NL_ERROR, "decode-attn-rope: no workspace of %zu bytes", scr);
  return cuda_status(attn_rope_decode_launch(QKV, CK, CV, POS, C, geo, g_rope.tab, ws, st,
                                             nullptr, nullptr),
                     "decode-attn-rope");
}

static int ternary_common(uint32_t count, const float *X, uint64_t xs, const uint32_t *WP,
                          uint64_t wsd, const float *S, uint64_t ss, const float *BIAS,
                          float *Y, uint64_t ys, uint32_t seq, uint32_t out, uint32_t cols,
                          uint32_t nblk, uint32_t wng, bool per_block, void *ws,
                          size_t ws_bytes, void *stream) {
  int rc = ensure_ready();
  if (rc) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  if (!ws && ternary_fast_shape(cols, nblk, wng, per_block)) {
    ws_bytes = ternary_ws_bytes_best(count, seq, cols, per_block);
    ws = library_workspace(ws_bytes, st);
    if (!ws) ws_bytes = 0;   // the generic kernel needs none
  }
  return cuda_status(ternary_gemv_launch(count, X, xs, WP, wsd, S, ss, BIAS, Y, ys, seq, out,
                                         cols, nblk, wng, per_block, UINT64_MAX, ws,
                                         ws_bytes, st),
                     "ternary");
}

extern "C" int nl_ternary_rows_dev(const float *X, const uint32_t *WP, const float *BIAS,
                                   const float *BETA, float *Y, uint32_t seq, uint32_t out,
                                   uint32_t cols, uint32_t nblk, uint32_t wng,
                                   void *workspace, size_t ws_bytes, void *stream) {
  return ternary_common(1, X, 0, WP, 0, BETA, 0, BIAS, Y, 0, seq, out, cols, nblk, wng, true,
                        workspace, ws_bytes, stream);
}

extern "C" int nl_ternary_gemv_dev(const float *X, const uint32_t *WP, const float *S,
                                   const float *BIAS, float *Y, uint32_t seq, uint32_t out,
                                   uint32_t cols, void *workspace, size_t ws_bytes,
                                   void *stream) {
  return ternary_common(1, X, 0, WP, 0, S, 0, BIAS, Y, 0, seq, out, cols, (cols + 127) / 128,
                        (cols + 15) / 16, false, workspace, ws_bytes, stream);
}

extern "C" int nl_wait_status(void) {
  if (take_wait_timeout())
    return set_error(NL_ERROR, "a kernel's bounded wait timed out; its outputs are invalid");
  return NL_OK;
}

namespace nl {
namespace {
// One thread waits on an mbarrier that expects two arrivals and gets one: the
// phase never completes, the wait gives up after ROUNDS rounds of at most
// 100 us each and reports.
__global__ void selftest_wait_kernel(int *err, uint32_t rounds) {
  __shared__ __align__(8) uint64_t bar;
  const uint32_t a = (uint32_t)__cvta_generic_to_shared(&bar);
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(a), "r"(2u));
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(a) : "memory");
  for (uint32_t i = 0; i < rounds; i++) {
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done) : "r"(a), "r"(0u), "r"(100000u) : "memory");
    if (done) return;
  }
  report_wait_timeout(err);
}
}  // namespace
}  // namespace nl

extern "C" int nl_selftest_wait_timeout(void) {
  int rc = ensure_ready();
  if (rc) return rc;
  int *err = wait_flag_device();
  if (!err) return set_error(NL_ERROR, "no host-mapped wait flag");
  selftest_wait_kernel<<<1, 1, 0, g.stream>>>(err, 64);
  count_launches(1);
  if ((rc = cuda_status(cudaStreamSynchronize(g.stream), "selftest-wait"))) return rc;
  return nl_wait_status();
}

extern "C" int nl_ternary_gemv_host_submit(uint32_t count, const float *X_host,
                                           uint64_t x_stride, const uint32_t *WP,
                                           uint64_t w_stride, const float *S, uint64_t s_stride,
                                           float *Y_host, uint64_t y_stride, uint32_t seq,
                                           uint32_t out, uint32_t cols, uint64_t *ticket) {
  int rc = ensure_ready();
  if (rc) return rc;
  if (!ticket) return set_error(NL_ERROR, "ternary-gemv-host: null ticket");
  *ticket = 0;
  if (count == 0 || seq == 0 || out == 0) return NL_OK;
  if (!X_host || !Y_host || !WP || !S)
    return set_error(NL_ERROR, "ternary-gemv-host: null buffer");
  if (count > 1 && (x_stride < (uint64_t)seq * cols || y_stride < (uint64_t)seq * out))
    return set_error(NL_ERROR, "ternary-gemv-host: strides overlap the problems");
  cudaError_t e = cudaSuccess;
  if (!g.h2d && (e = cudaStreamCreateWithFlags(&g.h2d, cudaStreamNonBlocking)) != cudaSuccess)
    return cuda_status(e, "ternary-gemv-host: streams");
  if (!g.d2h && (e = cudaStreamCreateWithFlags(&g.d2h, cudaStreamNonBlocking)) != cudaSuccess)
    return cuda_status(e, "ternary-gemv-host: streams");
  Context::HostSlot &hs = g.hs[g.host_tickets % kHostSlots];
  for (cudaEvent_t *ev : {&hs.in_done, &hs.k_done, &hs.out_done})
    if (!*ev && (e = cudaEventCreateWithFlags(ev, cudaEventDisableTiming)) != cudaSuccess)
      return cuda_status(e, "ternary-gemv-host: events");
  const uint64_t xs = count > 1 ? x_stride : (uint64_t)seq * cols;
  const uint64_t ys = count > 1 ? y_stride : (uint64_t)seq * out;
  const size_t xin = ((count - 1) * xs + (uint64_t)seq * cols) * 4u;
  const size_t yout = ((count - 1) * ys + (uint64_t)seq * out) * 4u;
  const size_t xbytes = align256(xin);
  if (hs.bytes < xbytes + yout) {
    // the slot's previous call must be done with it before it is replaced
    if (hs.used && (e = cudaEventSynchronize(hs.out_done)) != cudaSuccess)
      return cuda_status(e, "ternary-gemv-host: staging");
    if (hs.buf) cudaFree(hs.buf);
    hs.buf = nullptr;
    hs.bytes = 0;
    hs.used = false;
    if ((e = cudaMalloc(&hs.buf, xbytes + align256(yout))) != cudaSuccess)
      return cuda_status(e, "ternary-gemv-host: staging");
    hs.bytes = xbytes + align256(yout);
  }
  float *dx = (float *)hs.buf, *dy = (float *)((char *)hs.buf + xbytes);
  const uint32_t nblk = (cols + 127) / 128, wng = (cols + 15) / 16;
  size_t wsb = ternary_ws_bytes_best(count, seq, cols, false);
  void *ws = ternary_fast_shape(cols, nblk, wng, false) ? library_workspace(wsb, g.stream) : nullptr;
  if (!ws) wsb = 0;
  // copy in once the slot's previous kernel has read its inputs; run once the
  // inputs are there and the slot's previous outputs have been copied out;
  // copy out once the kernel is done
  if ((hs.used && (e = cudaStreamWaitEvent(g.h2d, hs.k_done, 0)) != cudaSuccess) ||
      (e = cudaMemcpyAsync(dx, X_host, xin, cudaMemcpyHostToDevice, g.h2d)) != cudaSuccess ||
      (e = cudaEventRecord(hs.in_done, g.h2d)) != cudaSuccess ||
      (e = cudaStreamWaitEvent(g.stream, hs.in_done, 0)) != cudaSuccess ||
      (hs.used && (e = cudaStreamWaitEvent(g.stream, hs.out_done, 0)) != cudaSuccess))
    return cuda_status(e, "ternary-gemv-host: copy in");
  if ((e = ternary_gemv_launch(count, dx, xs, WP, w_stride, S, s_stride, nullptr, dy, ys, seq,
                               out, cols, nblk, wng, false, UINT64_MAX, ws, wsb, g.stream)) !=
      cudaSuccess)
    return cuda_status(e, "ternary-gemv-host");
  if ((e = cudaEventRecord(hs.k_done, g.stream)) != cudaSuccess ||
      (e = cudaStreamWaitEvent(g.d2h, hs.k_done, 0)) != cudaSuccess ||
      (e = cudaMemcpyAsync(Y_host, dy, yout, cudaMemcpyDeviceToHost, g.d2h)) != cudaSuccess ||
      (e = cudaEventRecord(hs.out_done, g.d2h)) != cudaSuccess)
    return cuda_status(e, "ternary-gemv-host: copy out");
  hs.used = true;
  *ticket = ++g.host_tickets;
  return NL_OK;
}

extern "C" int nl_host_wait(uint64_t ticket) {
  int rc = ensure_ready();
  if (rc) return rc;
  if (ticket == 0) return NL_OK;          // an empty call's ticket
  if (ticket > g.host_tickets) return set_error(NL_ERROR, "host-wait: unknown ticket %llu",
                                                (unsigned long long)ticket);
  // copies out complete in ticket order on one stream: the slot's latest
  // copy-out is this ticket's or a later one
  Context::HostSlot &hs = g.hs[(ticket - 1) % kHostSlots];
  rc = cuda_status(cudaEventSynchronize(hs.out_done), "host-wait");
  if (rc == NL_OK && take_wait_timeout())
    return set_error(NL_ERROR, "host-wait: a kernel's bounded wait timed out");
  return rc;
}

extern "C" int nl_ternary_gemv_batched_host(uint32_t count, const float *X_host,
                                            uint64_t x_stride, const uint32_t *WP,
                                            uint64_t w_stride, const float *S, uint64_t s_stride,
                                            float *Y_host, uint64_t y_stride, uint32_t seq,
                                            uint32_t out, uint32_t cols) {
  uint64_t t = 0;
  const int rc = nl_ternary_gemv_host_submit(count, X_host, x_stride, WP, w_stride, S, s_stride,
                                             Y_host, y_stride, seq, out, cols, &t);
  return rc ? rc : nl_host_wait(t);
}

extern "C" int nl_ternary_gemv_batched_dev(uint32_t count, const float *X, uint64_t x_stride,
                                           const uint32_t *WP, uint64_t w_stride,
                                           const float *S, uint64_t s_stride, float *Y,
                                           uint64_t y_stride, uint32_t seq, uint32_t out,
                                           uint32_t cols, void *workspace, size_t ws_bytes,
                                           void *stream) {
  return ternary_common(count, X, x_stride, WP, w_stride, S, s_stride, nullptr, Y, y_stride,
                        seq, out, cols, (cols + 127) / 128, (cols + 15) / 16, false,
                        workspace, ws_bytes, stream);
}

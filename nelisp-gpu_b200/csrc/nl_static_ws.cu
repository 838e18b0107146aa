// nl_static_ws.cu -- the ternary GEMV on a workspace that is a file-scope
// device array, for callers that must not let the library allocate.
//
// nl_ternary_gemv_dev with a NULL workspace grows a library buffer with
// cudaMalloc on first use (and on any larger request); this variant instead
// runs the same prep + GEMV launches on g_static_ws, whose device address is
// looked up once per device.  It calls no cudaMalloc / cudaFree and no
// allocating library routine, and refuses to run before nl_init (which
// allocates the host-mapped flag the kernels' bounded waits report through).
//
// Nothing in the workspace must start at zero: the prep launch writes every
// fragment word of the live rows, their scales, flags and offset sums (all
// eight slots of each live row) before the GEMV launch reads them, in stream
// order, on every call; the padding columns of the last n-tile only reach MMA
// output columns the epilogue discards.
//
// Calls that overlap in time (different streams, or host threads) share the
// one array and race; the caller serialises them.

#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>

#include "nelisp_cuda.h"
#include "nl_internal.h"

namespace nl {
namespace {

static_assert(NL_TERNARY_STATIC_WS_BYTES % 256 == 0, "workspace size");

__device__ __align__(256) unsigned char g_static_ws[NL_TERNARY_STATIC_WS_BYTES];

constexpr int kMaxDevices = 64;
void *g_static_addr[kMaxDevices];
std::mutex g_static_mu;

// Device address of g_static_ws on the current device, looked up with that
// device current on the first call for it.
int static_ws(void **out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_status(e, "ternary static: cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices)
    return set_error(NL_ERROR, "ternary static: device %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_static_mu);
  if (!g_static_addr[dev]) {
    void *p = nullptr;
    e = cudaGetSymbolAddress(&p, g_static_ws);
    if (e != cudaSuccess) return cuda_status(e, "ternary static: cudaGetSymbolAddress");
    if (!p) return set_error(NL_ERROR, "ternary static: no address for the workspace");
    g_static_addr[dev] = p;
  }
  *out = g_static_addr[dev];
  return NL_OK;
}

}  // namespace
}  // namespace nl

using namespace nl;

extern "C" int nl_ternary_gemv_static_dev(const float *X, const uint32_t *WP, const float *S,
                                          const float *BIAS, float *Y, uint32_t seq,
                                          uint32_t out, uint32_t cols, void *stream) {
  // The kernels' bounded waits report through the host-mapped flag that
  // nl_init allocates; allocating it here would break this entry point's
  // promise, so a call before nl_init is refused.
  if (!wait_flag_if_allocated())
    return set_error(NL_ERROR,
                     "ternary static: call nl_init first (this entry point allocates "
                     "nothing, not even the library's context)");
  // The workspace the fastest path for this shape takes (the value
  // nl_ternary_workspace_bytes reports), so that no fast path declines for
  // want of room and the call never silently degrades.
  const size_t need = ternary_ws_bytes_best(1, seq, cols, false);
  if (need > (size_t)NL_TERNARY_STATIC_WS_BYTES)
    return set_error(NL_ERROR,
                     "ternary static: seq %u x cols %u needs %zu bytes of workspace, above "
                     "the static maximum of %zu",
                     seq, cols, need, (size_t)NL_TERNARY_STATIC_WS_BYTES);
  void *ws = nullptr;
  int rc = static_ws(&ws);
  if (rc) return rc;
  return cuda_status(ternary_gemv_launch(1, X, 0, WP, 0, S, 0, BIAS, Y, 0, seq, out, cols,
                                         (cols + 127) / 128, (cols + 15) / 16, false,
                                         UINT64_MAX, ws, NL_TERNARY_STATIC_WS_BYTES,
                                         (cudaStream_t)stream),
                     "ternary static");
}

// nl_internal.h -- shared declarations of libnelisp_cuda's translation units.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "nelisp_cuda.h"

namespace nl {

// Arguments of one dispatch of a registry kernel: the reference's binding
// list (buffers in binding order, sizes in 32-bit words), its push constants
// and its workgroup count, plus the stream and the scratch memory the
// launcher may use.
struct OpArgs {
  void *buf[NL_MAX_BUFS];
  uint32_t words[NL_MAX_BUFS];
  uint32_t nbuf;
  uint32_t push[NL_MAX_PUSH];
  uint32_t npush;
  uint32_t groups;
  cudaStream_t stream;
  void *scratch;
  size_t scratch_bytes;
};

// A registry entry.  `check` validates buffer sizes against the extents the
// push constants imply and returns NULL or a message; `scratch` reports the
// scratch bytes `launch` needs; `launch` enqueues the kernels (no host
// synchronisation, no allocation: it must be safe inside stream capture).
struct OpSpec {
  const char *name;
  uint32_t nbuf;
  uint32_t npush;
  const char *(*check)(const OpArgs &);
  size_t (*scratch)(const OpArgs &);
  cudaError_t (*launch)(const OpArgs &);
};

// Registry (nl_registry.cu).
const OpSpec *find_op(const char *name);
int op_count();
const OpSpec *op_at(int index);

// Per-family tables, defined next to their kernels.
extern const OpSpec kTernaryOps[];
extern const int kTernaryOpsCount;
extern const OpSpec kInt8Ops[];
extern const int kInt8OpsCount;
extern const OpSpec kDenseOps[];
extern const int kDenseOpsCount;
extern const OpSpec kRowOps[];
extern const int kRowOpsCount;
extern const OpSpec kAttnOps[];
extern const int kAttnOpsCount;
extern const OpSpec kKvOps[];
extern const int kKvOpsCount;
extern const OpSpec kMiscOps[];
extern const int kMiscOpsCount;
extern const OpSpec kQuantOps[];
extern const int kQuantOpsCount;
extern const OpSpec kTrainOps[];
extern const int kTrainOpsCount;

// Error reporting (nl_runtime.cu).
int set_error(int code, const char *fmt, ...);
int cuda_status(cudaError_t e, const char *what);

// Bounded waits.  A kernel whose bounded wait gives up records it in a
// host-mapped flag (wait_flag_device(), allocated by nl_init before any
// capture); the synchronising entry points report and clear it.
int *wait_flag_device();
// The flag's device address if it is allocated already, else nullptr; never
// allocates (for entry points that promise no allocation).
int *wait_flag_if_allocated();
bool take_wait_timeout();
__device__ __forceinline__ void report_wait_timeout(int *err) {
  if (err) {
    *(volatile int *)err = 1;
    __threadfence_system();
  }
}

// Launch accounting: every kernel the library enqueues is counted.
void count_launches(uint64_t n);

// Bounds-check helper for `check` functions: buffer B must hold at least
// NEED words.  Returns NULL when it does.
const char *need_words(const OpArgs &a, uint32_t b, uint64_t need,
                       const char *what);
// Formats a message into a per-thread buffer.
const char *fmt_msg(const char *fmt, ...);

// The number of reference invocations a dispatch of GROUPS workgroups of
// LOCAL invocations covers; kernels leave outputs of invocations at or past
// this index untouched, emulating a short grid.
static inline uint64_t invocations(uint32_t groups, uint32_t local) {
  return (uint64_t)groups * local;
}

// Ternary GEMV entry used by the typed API and the registry.
cudaError_t ternary_gemv_launch(uint32_t count, const float *X,
                                uint64_t x_stride, const uint32_t *WP,
                                uint64_t w_stride, const float *SCALE,
                                uint64_t s_stride, const float *BIAS,
                                float *Y, uint64_t y_stride, uint32_t seq,
                                uint32_t out, uint32_t cols, uint32_t nblk,
                                uint32_t wng, bool per_block, uint64_t limit,
                                void *ws, size_t ws_bytes,
                                cudaStream_t stream);
size_t ternary_ws_bytes(uint32_t count, uint32_t seq, uint32_t cols);
// The tcgen05 GEMM for seq > 16 sequence rows of one problem
// (k_ternary_umma.cu): its workspace, whether it applies, and the launch
// (prep + GEMM + flagged rows); *LAUNCHED false: it did not apply.
size_t ternary_umma_ws_bytes(uint32_t seq, uint32_t cols);
bool ternary_umma_applies(uint32_t count, uint32_t seq, uint32_t cols, bool per_block);
cudaError_t ternary_umma_launch(const float *X, const uint32_t *WP, const float *S,
                                const float *BIAS, float *Y, uint32_t seq, uint32_t out,
                                uint32_t cols, void *ws, size_t ws_bytes, cudaStream_t st,
                                bool *launched);
// Workspace for the fastest path of (count, seq, cols): the larger of the
// two.
size_t ternary_ws_bytes_best(uint32_t count, uint32_t seq, uint32_t cols, bool per_block);
// The two halves of the fast path, for callers that fuse the prep into the
// kernel producing the activations: the prep alone, and the GEMV alone on a
// workspace the prep has filled (seq <= 16; shapes the fast path does not
// cover, or a NULL workspace, take the generic kernel, which reads X).
cudaError_t ternary_prep_launch(const float *X, uint64_t x_stride, uint32_t count,
                                uint32_t seq, uint32_t cols, void *ws, cudaStream_t stream,
                                bool pdl = false);
// Outputs of a tensor-parallel partial GEMV written straight into every
// rank's receive slot (peer memory over NVLink, own slot included), each
// value as one 64-bit word (tag << 32 | f32 bits) with tag = *ep * tmul +
// tadd, the index of this use of the slots: a reader polls each word until
// its tag shows up, so no fence or counter is needed.  n = 0: the plain
// output Y.
struct PeerOut {
  unsigned long long *dst[8];
  const unsigned long long *ep;
  unsigned int tmul, tadd;
  int n;
};
// CTAs of the decode GEMV for this shape (0 when another kernel would run).
uint32_t ternary_dec_ctas(uint32_t count, uint32_t out, uint32_t cols, uint32_t seq);
cudaError_t ternary_main_launch(uint32_t count, const float *X, uint64_t x_stride,
                                const uint32_t *WP, uint64_t w_stride, const float *SCALE,
                                uint64_t s_stride, const float *BIAS, float *Y,
                                uint64_t y_stride, uint32_t seq, uint32_t out, uint32_t cols,
                                bool per_block, void *ws, cudaStream_t stream,
                                const PeerOut *po = nullptr);
bool ternary_fast_shape(uint32_t cols, uint32_t nblk, uint32_t wng,
                        bool per_block);

// Split-K single-query attention over a [B x maxseq x kvheads*hd] cache,
// positions 0..POS[0] (POS a float, as the reference's buffer).
struct AttnGeom {
  uint32_t B, heads, kvheads, hd, grp, kvdim, maxseq;  // maxseq: rows per sequence
  uint32_t nsplit, chunk;                                // key range per split
  uint64_t cache_words;                                  // CK/CV capacity
  float coef;                                            // 1/sqrt(hd)
};
AttnGeom attn_geom(uint32_t B, uint32_t dim, uint32_t heads, uint32_t kvheads,
                   uint32_t maxseq, uint64_t cache_words);
size_t attn_scratch_bytes(const AttnGeom &g);
// PDL: launched with programmatic stream serialization (both kernels wait
// for the preceding grid before reading anything).
cudaError_t attn_decode_launch(const float *Q, const float *CK, const float *CV,
                               const float *POS, float *C, const AttnGeom &g, void *scratch,
                               cudaStream_t st, bool pdl = false);

// Programmatic dependent launch.  A kernel launched with launch_pdl may
// start while the kernel before it in the stream is still running; it must
// touch nothing that kernel (or anything earlier) writes before pdl_wait(),
// which returns once the preceding grid has completed and its writes are
// visible.  A kernel calls pdl_trigger() to let its dependent start early.
#if defined(__CUDACC__)
__device__ __forceinline__ void pdl_wait() {
  asm volatile("griddepcontrol.wait;\n" ::: "memory");
}
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
}
// A launch with the programmatic-serialization attribute when PDL is set,
// an ordinary launch otherwise.
template <typename... KArgs, typename... Args>
cudaError_t launch_k(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                     cudaStream_t st, bool pdl, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t st, Args... args) {
  return launch_k(kernel, grid, block, smem, st, true, args...);
}
#endif

// The decoder's attention step with the half-split RoPE of q and k and the
// cache append of k and v at position POS[0] fused in (k_attn.cu).  ROPE is
// the [maxseq][hd/2] (cos, sin) table rope_table_launch fills.
cudaError_t rope_table_launch(float2 *rope, uint32_t maxseq, uint32_t hd, float base,
                              cudaStream_t st);
// With PREP_WS and ROW_CTR (g.B zeroed ints), the combine also quantizes each
// finished context row into PREP_WS, the O-projection GEMV's workspace.
cudaError_t attn_rope_decode_launch(const float *QKV, float *CK, float *CV, const int *POS,
                                    float *C, const AttnGeom &g, const float2 *rope,
                                    void *scratch, cudaStream_t st, void *prep_ws = nullptr,
                                    int *row_ctr = nullptr);
size_t attn_rope_scratch_bytes(const AttnGeom &g);   // 0: shape not covered
// Causal attention over rows 0..seq-1 of B sequences (attn-causal-gqa per
// sequence): Q / CTX rows of heads*hd floats, K / V rows of kvheads*hd,
// sequence b at + b * q_batch / + b * kv_batch floats.
cudaError_t attn_causal_prefill_launch(const float *Q, const float *CK, const float *CV,
                                       float *CTX, uint32_t B, uint32_t seq, uint32_t heads,
                                       uint32_t kvheads, uint32_t hd, uint64_t q_batch,
                                       uint64_t kv_batch, cudaStream_t st);

// The tcgen05 GEMV for up to 16 sequence rows (k_ternary_tc.cu).
size_t ternary_tc_ws_bytes(uint32_t count, uint32_t seq, uint32_t cols);
bool ternary_tc_applies(uint32_t count, uint32_t seq, uint32_t out, uint32_t cols,
                        bool per_block, uint64_t w_stride);
cudaError_t ternary_tc_launch(uint32_t count, const float *X, uint64_t x_stride,
                              const uint32_t *WP, uint64_t w_stride, const float *SCALE,
                              uint64_t s_stride, const float *BIAS, float *Y, uint64_t y_stride,
                              uint32_t seq, uint32_t out, uint32_t cols, uint64_t limit, void *ws,
                              size_t ws_bytes, cudaStream_t st, bool *launched);

// Copies NBYTES at OFFSET of PATH into device memory DST through the pipelined
// pinned-slot reader (nl_runtime.cu).  NL_OK, or NL_ERROR with a message
// (*MISSING_WORDS set when the file is short).
int file_to_device(const char *path, uint64_t offset, size_t nbytes, void *dst,
                   uint64_t *missing_words);

// Ternarization of an f32 weight matrix with the reference's quant-w rule,
// packed into the two-bit GEMV format (k_quant.cu).  SCRATCH holds
// quant_w_scratch_bytes(rows) bytes.
size_t quant_w_scratch_bytes(uint32_t rows);
cudaError_t quant_w_pack_launch(const float *W, uint32_t rows, uint32_t cols, bool per_row,
                                uint32_t *WP, float *S, void *scratch, cudaStream_t st);

// Library workspace for typed calls that pass no workspace (nl_runtime.cu).
void *library_workspace(size_t bytes, cudaStream_t stream);

static inline int ceil_div(int a, int b) { return (a + b - 1) / b; }
static inline uint64_t ceil_div64(uint64_t a, uint64_t b) {
  return (a + b - 1) / b;
}
static inline bool aligned16(const void *p) {
  return ((uintptr_t)p & 15u) == 0;
}

// Grid-size helper: at most `cap` blocks of `threads` covering `n` items.
static inline unsigned grid_for(uint64_t n, unsigned threads,
                                unsigned cap = 148u * 32u) {
  uint64_t g = ceil_div64(n, threads);
  if (g == 0) g = 1;
  if (g > cap) g = cap;
  return (unsigned)g;
}

}  // namespace nl

#define NL_LAUNCH_CHECK() cudaPeekAtLastError()

/* nelisp_cuda.h -- C ABI of libnelisp_cuda, the CUDA (sm_100a) replacement
 * for the Vulkan compute host of zawatton/nelisp-gpu.
 *
 * Two layers:
 *
 *  1. The operator surface of the reference's persistent server
 *     (host/vkserver.c), one entry point per opcode, so a protocol server
 *     (nelisp-cuserver) or an FFI binding can drive the library exactly as
 *     lisp/nelisp-gpu-server.el drives vkserver.  Buffers are raw 32-bit
 *     words (f32 bit patterns or packed integers), kernels are addressed by
 *     the reference's DSL names (lisp/nelisp-gpu-kernels.el), push constants
 *     are uint32 and `groups` is the reference's 64-wide workgroup count.
 *     Host memory belongs to the caller; device memory to the library.
 *
 *  2. Typed entry points on device pointers and a CUDA stream, for callers
 *     that keep their tensors on the GPU (the decoder, the benchmarks, a
 *     PyTorch/ctypes caller).
 *
 * Status codes: NL_OK (0); NL_ERROR (1) for a recoverable error -- the
 * server's wire status 1 -- with the reason in nl_last_error(); NL_FATAL (2)
 * for a CUDA error after which the context is unusable (the reference's
 * VK_CHECK exit(2), host/vkserver.c:47-48).
 *
 * Not thread-safe: one context per process, as vkserver has one device,
 * one queue and one fence.  The device is nl_init's argument, or
 * NELISP_GPU_DEVICE when that is negative (host/vkserver.c:220).
 */
#ifndef NELISP_CUDA_H
#define NELISP_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define NL_OK 0
#define NL_ERROR 1
#define NL_FATAL 2

/* OP_RUN buffer kinds (host/vkserver.c:16-19). */
#define NL_RUN_IN 0        /* inline input: sent, not returned */
#define NL_RUN_RESIDENT 1  /* resident buffer, by handle */
#define NL_RUN_OUT 2       /* output: zeroed, returned */
#define NL_RUN_INOUT 3     /* inline input, returned */

/* OP_BATCH / OP_COMPILE slot kinds (host/vkserver.c:424-426).  The numbering
 * and the field order differ from OP_RUN's, as in the reference. */
#define NL_SLOT_IN 0
#define NL_SLOT_RESIDENT 1
#define NL_SLOT_TMP 2      /* transient: zeroed (every run, when compiled) */
#define NL_SLOT_OUT 3      /* zeroed, returned */

/* Table limits of host/vkserver.c (:71-100, :435-436). */
#define NL_MAX_BUFS 16
#define NL_MAX_PUSH 16
#define NL_MAX_NAME 63
#define NL_MAX_RESIDENT 4096
#define NL_MAX_COMPILED 16
#define NL_MAX_SLOTS 8192
#define NL_MAX_DISPATCH 8192

/* One OP_RUN buffer descriptor (host/vkserver.c:15). `handle` is read only
 * for NL_RUN_RESIDENT. */
typedef struct {
  uint32_t size;   /* 32-bit words */
  uint32_t kind;
  uint32_t handle;
} nl_run_buffer;

/* One OP_BATCH / OP_COMPILE slot (host/vkserver.c:425). */
typedef struct {
  uint32_t kind;
  uint32_t size;   /* 32-bit words */
  uint32_t handle;
} nl_slot;

/* One dispatch of a batch (host/vkserver.c:428-429, :433). */
typedef struct {
  char name[NL_MAX_NAME + 1];
  uint32_t nbuf;
  uint32_t slot[NL_MAX_BUFS];
  uint32_t npush;
  uint32_t push[NL_MAX_PUSH];
  uint32_t groups;
} nl_dispatch;

/* ---- context -------------------------------------------------------- */

/* Create the context on DEVICE (<0: NELISP_GPU_DEVICE, else 0).  Replaces
 * init_vulkan (host/vkserver.c:213-245).  Idempotent. */
int nl_init(int device);
/* Release every resident buffer, compiled batch and the device context. */
void nl_shutdown(void);
const char *nl_last_error(void);
const char *nl_version(void);
/* The CUDA device ordinal in use, or -1 before nl_init. */
int nl_device(void);
/* Name of the device in use (the reference logs it, host/vkserver.c:225). */
const char *nl_device_name(void);

/* The kernel registry: names the server accepts, and their arity (number of
 * buffers and push constants in lisp/nelisp-gpu-kernels.el). */
int nl_kernel_count(void);
const char *nl_kernel_name(int index);
int nl_kernel_arity(const char *name, uint32_t *nbuf, uint32_t *npush);

/* ---- resident buffers ---------------------------------------------- */

/* OP_UPLOAD (host/vkserver.c:336-351): copy NWORDS words to a new resident
 * device buffer.  Handles are the first free slot of a 4096-entry table, as
 * in the reference.  Status 1 when the table is full. */
int nl_upload(const void *words, uint32_t nwords, uint32_t *handle);
/* OP_UPLOAD_FILE (host/vkserver.c:371-410): read NWORDS words at byte
 * OFFSET of PATH straight into a new resident buffer.  Status 1 (and no
 * handle allocated) on open, seek or short-read failure.  The region streams
 * through four 16 MiB pinned slots, each filled by four parallel preads
 * (O_DIRECT where the file system allows) while the previous slot is copied
 * to the device. */
int nl_upload_file(const char *path, uint64_t offset, uint32_t nwords,
                   uint32_t *handle);

/* OP_UPLOAD_FILE with on-device repacking: reads an f32 weight matrix
 * [rows x cols] (row-major, the importer's dense layout) at OFFSET of PATH
 * through the same pipelined reader, ternarizes it on the device with the
 * reference's quant-w rule (lisp/nelisp-gpu-kernels.el:516-561: beta = mean
 * |W|, per tensor or, with PER_ROW, per row; t = +1 where W/beta >= 0.5, -1
 * where <= -0.5, else 0) and packs it into the two-bit GEMV format (field i
 * of word i/16 at bits 2(i%16); 00 -> 0, 01 -> +1, 11 -> -1).  Returns two
 * resident handles: *H_WP, rows x ceil(cols/16) words, and *H_S, the rows
 * scales (beta of each row).  diag(S) (T x) equals quant-w's fake-quantized
 * weights times x.  Short files and open errors: NL_ERROR, no handles. */
int nl_upload_file_ternary(const char *path, uint64_t offset, uint32_t rows,
                           uint32_t cols, int per_row, uint32_t *h_wp,
                           uint32_t *h_s);
/* OP_WRITE_RESIDENT (host/vkserver.c:356-367): overwrite in place.  Status 1
 * for a bad handle or more words than the buffer holds. */
int nl_write_resident(uint32_t handle, const void *words, uint32_t nwords);
/* Read back the first NWORDS words (the reference reads through the `scale`
 * kernel, lisp/nelisp-gpu-server.el:211-217). */
int nl_read_resident(uint32_t handle, void *words, uint32_t nwords);
/* OP_FREE (host/vkserver.c:412-418): an unknown handle is not an error. */
int nl_free(uint32_t handle);
/* Device address and size of a resident buffer. */
int nl_resident_info(uint32_t handle, void **dev_ptr, uint32_t *nwords);

/* ---- dispatch by kernel name ---------------------------------------- */

/* OP_RUN (host/vkserver.c:274-334).  INLINE_WORDS holds the data of the
 * NL_RUN_IN and NL_RUN_INOUT buffers, concatenated in binding order; OUT_WORDS
 * receives the NL_RUN_OUT and NL_RUN_INOUT buffers, in binding order. */
int nl_run(const char *name, uint32_t nbuf, const nl_run_buffer *bufs,
           uint32_t npush, const uint32_t *push, uint32_t groups,
           const void *inline_words, void *out_words);

/* OP_BATCH (host/vkserver.c:437-506): the dispatches run in order on one
 * stream (stream order is the reference's barrier between dispatches).
 * INLINE_WORDS holds the NL_SLOT_IN slots in slot order; OUT_WORDS receives
 * the NL_SLOT_OUT slots in slot order. */
int nl_batch(uint32_t nslot, const nl_slot *slots, uint32_t ndisp,
             const nl_dispatch *disps, const void *inline_words,
             void *out_words);

/* OP_COMPILE (host/vkserver.c:511-587): allocate the non-resident slots once,
 * copy the inline inputs once and capture the dispatches -- with memset
 * nodes zeroing the tmp and out slots -- into a CUDA graph.  Resident
 * buffers are bound by address at compile time, as the reference binds
 * them into its recorded command buffer.  Status 1 when all 16 entries are
 * in use. */
int nl_compile(uint32_t nslot, const nl_slot *slots, uint32_t ndisp,
               const nl_dispatch *disps, const void *inline_words,
               uint32_t *handle);
/* OP_RUN_COMPILED (host/vkserver.c:591-604): replay the graph; OUT_WORDS
 * receives the out slots in slot order.  Status 1 for a bad handle. */
int nl_run_compiled(uint32_t handle, void *out_words);
/* OP_FREE_COMPILED (host/vkserver.c:606-615). */
int nl_free_compiled(uint32_t handle);
/* Total words OP_RUN_COMPILED returns for HANDLE. */
int nl_compiled_out_words(uint32_t handle, uint64_t *nwords);
/* Replay HANDLE's graph REPS times back to back without copying outputs and
 * report the device time per replay (CUDA events).  This is what
 * host/vkmatmul.c times: one submit of a recorded command buffer
 * (:163-169). */
int nl_time_compiled(uint32_t handle, uint32_t reps, double *ms_per_rep);

/* Any registry kernel on caller-owned device buffers, enqueued on STREAM
 * (a cudaStream_t, used as given: 0 is the legacy default stream).  NWORDS gives each
 * buffer's size for the bounds checks.  Does not synchronise. */
int nl_dispatch_dev(const char *name, uint32_t nbuf, void *const *bufs,
                    const uint32_t *nwords, uint32_t npush,
                    const uint32_t *push, uint32_t groups, void *stream);

/* ---- typed entry points (device pointers) --------------------------- */

/* Workspace the ternary kernels need for SEQ activation rows of COLS
 * columns: the activations re-expressed as three exact int8 limbs per value
 * for the tensor-core path.  Pass at least this many bytes, or NULL to use
 * the library's own workspace. */
size_t nl_ternary_workspace_bytes(uint32_t seq, uint32_t cols);

/* ternary-rows (lisp/nelisp-gpu-kernels.el:713-746) on device pointers:
 * Y[s,o] = BIAS[o] + sum_b BETA[o*nblk+b] * sum_{i in block b} t(o,i) X[s,i]
 * with WP holding sixteen two-bit fields per word (field i at bits 2(i%16)
 * of word i/16; 00 -> 0, 01 -> +1, 11 -> -1, 10 -> -2). */
int nl_ternary_rows_dev(const float *X, const uint32_t *WP, const float *BIAS,
                        const float *BETA, float *Y, uint32_t seq,
                        uint32_t out, uint32_t cols, uint32_t nblk,
                        uint32_t wng, void *workspace, size_t ws_bytes,
                        void *stream);

/* The ternary GEMV with one scale per output row -- y = diag(S)(W x) + BIAS
 * -- i.e. ternary-rows with S[o] in every 128-column block.  WP rows are
 * cols/16 words (cols a multiple of 16).  BIAS may be NULL. */
int nl_ternary_gemv_dev(const float *X, const uint32_t *WP, const float *S,
                        const float *BIAS, float *Y, uint32_t seq,
                        uint32_t out, uint32_t cols, void *workspace,
                        size_t ws_bytes, void *stream);

/* COUNT independent GEMVs of the shape above in one launch: problem z uses
 * X + z*x_stride, WP + z*w_stride, S + z*s_stride and writes Y + z*y_stride
 * (strides in elements).  The workspace must hold COUNT times
 * nl_ternary_workspace_bytes(seq, cols). */
int nl_ternary_gemv_batched_dev(uint32_t count, const float *X,
                                uint64_t x_stride, const uint32_t *WP,
                                uint64_t w_stride, const float *S,
                                uint64_t s_stride, float *Y,
                                uint64_t y_stride, uint32_t seq, uint32_t out,
                                uint32_t cols, void *workspace,
                                size_t ws_bytes, void *stream);

/* One decode position of attention for BATCH sequences, with the three
 * dispatches the decode loop makes in the reference fused into one pass:
 * rope-half on q and on the new key at absolute position POS[0]
 * (lisp/nelisp-gpu-kernels.el:857-882, half-split pairs (m, m + hd/2),
 * theta = pos / base^(2m/hd)), cache-append-b of the rotated key and the
 * value at POS[0] (:358-365), and decode-attn-b over positions 0..POS[0]
 * with scale 1/sqrt(hd) (:368-390).  QKV holds per sequence row
 * [heads*hd q | kv_heads*hd k | kv_heads*hd v] (the fused Q|K|V linear's
 * output); CK / CV are [batch][max_seq][kv_heads*hd] (16-byte aligned) and
 * hold already-rotated keys; C receives [batch][heads*hd].  POS is one
 * int32 on the device.  hd is 32, 64, 128 or 256, heads/kv_heads <= 8.
 * The first call for a (max_seq, hd, base) builds a table in library
 * memory; make it outside any stream capture.  Does not synchronise. */
int nl_decode_attn_rope_dev(const float *QKV, float *CK, float *CV,
                            const int32_t *POS, float *C, uint32_t batch,
                            uint32_t heads, uint32_t kv_heads,
                            uint32_t head_dim, uint32_t max_seq,
                            float rope_base, void *stream);

/* nl_ternary_gemv_batched_dev end to end on host buffers: copies the COUNT
 * activation blocks in from X_HOST, runs the GEMVs on the device-resident
 * weights WP and scales S (device pointers, e.g. from nl_resident_info) and
 * copies the outputs back to Y_HOST, returning once they are there.  The
 * per-call shape of the reference's RUN (inline inputs copied in, outputs
 * copied back; host/vkserver.c:274-334) for a resident-weight GEMV batch.
 * X_HOST and Y_HOST should be pinned (cudaHostAlloc / torch pin_memory) for
 * the copies to run at full speed.  Problem z reads X_HOST + z*x_stride
 * (seq*cols values) and writes Y_HOST + z*y_stride (seq*out values).  Device
 * staging is owned by the library.  Equivalent to nl_ternary_gemv_host_submit
 * followed by nl_host_wait. */
int nl_ternary_gemv_batched_host(uint32_t count, const float *X_host,
                                 uint64_t x_stride, const uint32_t *WP,
                                 uint64_t w_stride, const float *S,
                                 uint64_t s_stride, float *Y_host,
                                 uint64_t y_stride, uint32_t seq, uint32_t out,
                                 uint32_t cols);

/* The same call without waiting: queues the copy in, the GEMVs and the copy
 * out, and returns a TICKET (1, 2, 3, ... per call; 0 for an empty call).
 * The caller keeps X_HOST and Y_HOST untouched until nl_host_wait(TICKET)
 * returns.  Calls' copies and kernels overlap on the device, so a serving
 * loop that keeps two or three requests in flight hides the copies behind
 * the kernels.  The library keeps eight staging slots; the ninth call in
 * flight reuses the first call's slot, and nl_host_wait on the first ticket
 * then also waits for the ninth call. */
int nl_ternary_gemv_host_submit(uint32_t count, const float *X_host,
                                uint64_t x_stride, const uint32_t *WP,
                                uint64_t w_stride, const float *S,
                                uint64_t s_stride, float *Y_host,
                                uint64_t y_stride, uint32_t seq, uint32_t out,
                                uint32_t cols, uint64_t *ticket);

/* Waits until call TICKET's outputs are in its Y_HOST (and every earlier
 * call's too).  Returns NL_ERROR for a ticket never issued, or when a
 * kernel's bounded wait timed out (see nl_wait_status). */
int nl_host_wait(uint64_t ticket);

/* Bounded waits.  The library's kernels that wait on mbarriers (the TMA and
 * tcgen05 ternary kernels) give up after a bounded time and record it in a
 * host-mapped flag; their outputs are then invalid.  The synchronising entry
 * points (nl_run, nl_batch, nl_run_compiled, nl_ternary_gemv_batched_host,
 * nl_host_wait) report it as NL_ERROR.  Callers of the asynchronous *_dev entry points
 * synchronise their stream and then call nl_wait_status: NL_ERROR (with a
 * message) if a wait gave up since the last report, else NL_OK; the flag is
 * cleared.  No reference counterpart (vkserver has no device-side waits). */
int nl_wait_status(void);

/* Self-test of the bounded-wait report: one thread waits on an mbarrier that
 * nothing completes, gives up after a few milliseconds and sets the flag;
 * synchronises and returns what nl_wait_status returns (NL_ERROR when the
 * report works).  The context stays usable. */
int nl_selftest_wait_timeout(void);

/* Size of the file-scope device workspace of nl_ternary_gemv_static_dev. */
#define NL_TERNARY_STATIC_WS_BYTES (2u << 20)

/* nl_ternary_gemv_dev with no workspace argument and no allocation: the
 * scratch is a file-scope device array of NL_TERNARY_STATIC_WS_BYTES
 * (2 MiB).  No reference counterpart: an addition of this library for
 * callers that must not let it allocate (the reference's ternary-rows always
 * takes its buffers from the caller).  Returns NL_ERROR with a message when
 * nl_ternary_workspace_bytes(seq, cols) -- the workspace of the fastest path
 * for the shape -- exceeds the maximum (e.g. seq 16 with cols above 43664,
 * seq 1 above 261984, seq 512 with cols 2560), and when nl_init has not run
 * on this process (the call would otherwise have to allocate the library's
 * wait flag).  The first call on a device looks the array's address up with
 * that device current; make it before any stream capture.  Calls that
 * overlap in time share the array and race: the caller serialises them.
 * Does not synchronise. */
int nl_ternary_gemv_static_dev(const float *X, const uint32_t *WP,
                               const float *S, const float *BIAS, float *Y,
                               uint32_t seq, uint32_t out, uint32_t cols,
                               void *stream);

/* ---- the ternary decoder (tensor-parallel) --------------------------- */

/* A LLaMA-style decoder with ternary linears (BitNet-b1.58-2B shaped): RMSNorm,
 * fused Q|K|V and gate|up ternary linears with per-row f32 scales, half-split
 * RoPE, a per-sequence f32 KV cache, SwiGLU, a tied f32 embedding / LM head
 * and greedy argmax.  Weights are synthetic: generated on the device from
 * SEED by a counter-based hash of (seed, tensor, element), trits -1/0/+1
 * with p = 1/3, row scales (0.5 + u) / sqrt(2K/3), norm gains 0.75 + u/2,
 * embeddings 2u - 1 (u uniform in [0, 1)).  The reference has no decoder of
 * its own in its repository; this composition of its kernels is this
 * library's (no reference interface is replaced). */
typedef struct {
  uint32_t hidden, layers, heads, kv_heads, head_dim, ffn, vocab;
  uint32_t max_batch;   /* <= 16 */
  uint32_t max_seq;     /* KV-cache rows per sequence */
  float rms_eps, rope_base;
  uint64_t seed;
} nl_decoder_config;

typedef struct nl_decoder nl_decoder;

/* NCCL unique id (128 bytes) for a tensor-parallel group; rank 0 makes it
 * and the caller broadcasts it. */
int nl_nccl_unique_id(void *id_out);
/* One rank of a TP_SIZE-way tensor-parallel decoder on the current device
 * (NCCL_ID ignored when TP_SIZE is 1).  KEEP_LOGITS stores every step's
 * logits for nl_decoder_logits. */
int nl_decoder_create(const nl_decoder_config *cfg, int tp_rank, int tp_size,
                      const void *nccl_id, int keep_logits, nl_decoder **out);
/* The weights of a decoder as resident buffers: handles from nl_upload,
 * nl_upload_file or nl_upload_file_ternary (the reference's OP_UPLOAD /
 * OP_UPLOAD_FILE, host/vkserver.c:336-410, through which
 * lisp/nelisp-gpu-server.el:141-197 loads a model's tensors).  Ternary
 * matrices are packed two-bit rows of cols/16 words (the ternary-rows
 * format), scales f32 per row, norms f32 [hidden].  Each array holds LAYERS
 * handles.  Shapes: wq [heads*head_dim x hidden], wk / wv [kv_heads*head_dim
 * x hidden], wo [hidden x heads*head_dim], wgate / wup [ffn x hidden], wdown
 * [hidden x ffn]; embed f32 [vocab x hidden] is also the (tied) LM head. */
typedef struct {
  uint32_t embed, final_norm;
  const uint32_t *wq, *wk, *wv, *wo, *wgate, *wup, *wdown;
  const uint32_t *sq, *sk, *sv, *so, *sgate, *sup, *sdown;
  const uint32_t *attn_norm, *ffn_norm;
} nl_decoder_weights;

/* nl_decoder_create with the weights of W instead of synthetic ones (the
 * config's seed is not used).  Each rank copies its shard out of the full
 * tensors on the device (rows of Q|K|V and gate|up, columns of O and down);
 * the handles may be freed afterwards.  NL_ERROR when a handle's size does
 * not match its tensor's shape. */
int nl_decoder_create_from_weights(const nl_decoder_config *cfg, const nl_decoder_weights *w,
                                   int tp_rank, int tp_size, const void *nccl_id,
                                   int keep_logits, nl_decoder **out);
/* Greedy generation for BATCH sequences: PROMPT is [batch x prompt_len]
 * int32 (host); OUT_TOKENS receives [batch x steps].  Each step is one CUDA
 * graph replay; PREFILL_MS times the prompt_len - 1 replays that fill the
 * cache with the prompt, DECODE_MS the STEPS replays that generate (device
 * time, CUDA events).  All ranks must call it together. */
int nl_decoder_generate(nl_decoder *dec, uint32_t batch, uint32_t prompt_len,
                        const int32_t *prompt, uint32_t steps,
                        int32_t *out_tokens, double *prefill_ms,
                        double *decode_ms);
/* The stored logits: [max_seq][max_batch][vocab rows of this rank]. */
int nl_decoder_logits(nl_decoder *dec, float *out, uint64_t nfloats);
/* SHARD[6] = kv-head begin, kv-head count, ffn begin, ffn count, vocab
 * begin, vocab count of this rank; bytes of weights this rank streams per
 * step; kernels per decode step. */
int nl_decoder_info(nl_decoder *dec, uint32_t *shard, uint64_t *weight_bytes,
                    uint64_t *kernels_per_step);
/* The SHARD[6] that nl_decoder_info would report for rank TP_RANK of a
 * TP_SIZE-way decoder of CFG, from the partition the constructors use,
 * without a device or a decoder (host arithmetic only: no nl_init needed).
 * Ranges of two ranks differ by at most one KV head, one 128-wide FFN block
 * or one vocabulary row, the longer ranges first.  NL_ERROR for a config the
 * constructors refuse, a rank outside [0, TP_SIZE), or a TP_SIZE that leaves
 * some rank without KV heads, FFN blocks or vocabulary rows.  No counterpart
 * in the reference, whose repository has no decoder. */
int nl_decoder_shard(const nl_decoder_config *cfg, int tp_rank, int tp_size,
                     uint32_t *shard);
void nl_decoder_destroy(nl_decoder *dec);

/* Launch counter: how many kernels this library has enqueued since the
 * context was created (each graph replay counts the kernels it holds). */
uint64_t nl_launch_count(void);

#ifdef __cplusplus
}
#endif
#endif /* NELISP_CUDA_H */

// nl_decoder.cu -- the ternary LLaMA-style decoder (BitNet-b1.58-2B shaped)
// assembled from the hot-path kernels, tensor-parallel over NCCL.
//
// The reference holds the kernels of this model but not the model
// (lisp/nelisp-gpu-kernels.el; its decoder lives outside the repository), so
// the composition follows the conventions its kernels document: RMSNorm
// before attention and FFN (rmsnorm-istd/-fwd, :1250-1265, with the eps a
// parameter), a fused Q|K|V and a fused gate|up ternary linear with per-row
// scales (bitlinear-packed-v, :1022-1040, on the two-bit format of
// ternary-rows, :713-746), half-split RoPE at the absolute position
// (rope-half, :857-882), a per-sequence KV cache (cache-append-b, :358-365),
// single-query attention with scale 1/sqrt(hd) (decode-attn-b, :368-390),
// SwiGLU (silu-mul, :187-193), residual adds (add2, :816-821), a tied f32
// LM head and greedy argmax (lowest index on ties).
//
// One decode step is one CUDA graph replay.  The position, the tokens and
// the argmax keys live on the device, so consecutive replays advance the
// sequence without the host: while the prompt is consumed the next token
// comes from it (teacher forcing), afterwards from the argmax.
//
// Tensor parallelism (one process per GPU): KV heads (with their query
// heads) and 128-column FFN blocks are split across ranks, unevenly where
// they do not divide; Q|K|V and gate|up are column-parallel, O and down
// row-parallel, followed by an NCCL all-reduce (sum); the LM head is split
// by vocabulary rows and the (logit, index) argmax keys are all-reduced with
// max.  Every rank generates its own shard of the synthetic weights from
// global element indices (nl_rng.h), so no weights cross the links.

#include <cooperative_groups.h>
#include <cuda.h>
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <map>
#include <vector>

#include "nl_internal.h"
#include "nl_rng.h"
#include "nl_step.h"
#include "ternary_prep.cuh"

namespace nl {
namespace {

// ---- NCCL, loaded on demand (single-GPU use needs no NCCL) -----------------
typedef struct ncclComm *ncclComm_t;
typedef struct { char internal[128]; } ncclUniqueId;
typedef int ncclResult_t;
constexpr int kNcclSum = 0, kNcclMax = 2, kNcclMin = 3, kNcclInt8 = 0, kNcclInt32 = 2,
              kNcclUint64 = 5, kNcclFloat32 = 7;

struct Nccl {
  void *h = nullptr;
  ncclResult_t (*GetUniqueId)(ncclUniqueId *) = nullptr;
  ncclResult_t (*CommInitRank)(ncclComm_t *, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*AllReduce)(const void *, void *, size_t, int, int, ncclComm_t, cudaStream_t) =
      nullptr;
  ncclResult_t (*AllGather)(const void *, void *, size_t, int, ncclComm_t, cudaStream_t) =
      nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  const char *(*GetErrorString)(ncclResult_t) = nullptr;
};

Nccl *nccl() {
  static Nccl n;
  static bool tried = false;
  if (!tried) {
    tried = true;
    // An NCCL already in the process (PyTorch's) is reused; otherwise the
    // library is opened RTLD_LOCAL so that its symbols never shadow those a
    // later-loaded library (libtorch_cuda) expects from a newer NCCL.
    const char *env = getenv("NELISP_NCCL_LIB");
    if (env && *env) n.h = dlopen(env, RTLD_NOW | RTLD_LOCAL);
    if (!n.h) n.h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (!n.h) n.h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
    if (!n.h) n.h = dlopen("libnccl.so", RTLD_NOW | RTLD_LOCAL);
    if (n.h) {
      n.GetUniqueId = (decltype(n.GetUniqueId))dlsym(n.h, "ncclGetUniqueId");
      n.CommInitRank = (decltype(n.CommInitRank))dlsym(n.h, "ncclCommInitRank");
      n.AllReduce = (decltype(n.AllReduce))dlsym(n.h, "ncclAllReduce");
      n.AllGather = (decltype(n.AllGather))dlsym(n.h, "ncclAllGather");
      n.CommDestroy = (decltype(n.CommDestroy))dlsym(n.h, "ncclCommDestroy");
      n.GetErrorString = (decltype(n.GetErrorString))dlsym(n.h, "ncclGetErrorString");
    }
  }
  if (!n.h || !n.GetUniqueId || !n.CommInitRank || !n.AllReduce || !n.CommDestroy) return nullptr;
  return &n;
}

struct Split {
  uint32_t begin, count;
};
Split split(uint32_t n, uint32_t parts, uint32_t r) {
  uint32_t base = n / parts, rem = n % parts;
  return {r * base + (r < rem ? r : rem), base + (r < rem ? 1u : 0u)};
}

// The configurations the decoder's kernels take.
int check_config(const nl_decoder_config &c) {
  const bool hd_ok = c.head_dim == 32 || c.head_dim == 64 || c.head_dim == 128 ||
                     c.head_dim == 256;
  if (c.hidden == 0 || c.hidden % 128 || c.ffn == 0 || c.ffn % 128 || !hd_ok || c.heads == 0 ||
      c.kv_heads == 0 || c.heads % c.kv_heads || c.heads / c.kv_heads > 8 ||
      c.max_batch == 0 || c.max_batch > 16 || c.max_seq == 0 || c.vocab == 0 || c.layers == 0)
    return set_error(NL_ERROR,
                     "decoder config: hidden and ffn multiples of 128, head_dim 32, 64, 128 or "
                     "256, heads a multiple of kv_heads (at most 8 per kv head), "
                     "1 <= max_batch <= 16");
  return NL_OK;
}

// One rank's part of a SIZE-way tensor-parallel decoder: contiguous ranges
// of KV heads (with their query heads: rows of Q|K|V, columns of O, the KV
// cache), of 128-wide FFN blocks (rows of gate|up, columns of down) and of
// vocabulary rows (the LM head).  The ranges of two ranks differ by at most
// one unit, the longer ones first; a rank left without some kind is an error.
struct Shard {
  Split kvh, ffb, voc;
};
int plan_shard(const nl_decoder_config &c, int rank, int size, Shard *s) {
  if (size < 1 || rank < 0 || rank >= size)
    return set_error(NL_ERROR, "decoder: rank %d of %d", rank, size);
  s->kvh = split(c.kv_heads, (uint32_t)size, (uint32_t)rank);
  s->ffb = split(c.ffn / 128, (uint32_t)size, (uint32_t)rank);
  s->voc = split(c.vocab, (uint32_t)size, (uint32_t)rank);
  if (s->kvh.count == 0 || s->ffb.count == 0 || s->voc.count == 0)
    return set_error(NL_ERROR, "decoder: %d ranks leave rank %d without heads, FFN blocks or vocab",
                     size, rank);
  return NL_OK;
}

// ---- weight generation -------------------------------------------------------------
__global__ void gen_ternary_kernel(uint32_t *W, uint32_t rows, uint32_t k_local, uint64_t key,
                                   uint64_t grow0, uint64_t k_full, uint64_t c0) {
  const uint32_t wng = (k_local + 15) / 16;
  const uint64_t n = (uint64_t)rows * wng;
  for (uint64_t idx = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < n;
       idx += (uint64_t)gridDim.x * blockDim.x) {
    const uint32_t r = (uint32_t)(idx / wng), w = (uint32_t)(idx % wng);
    uint32_t word = 0;
    for (uint32_t f = 0; f < 16; f++) {
      const uint32_t c = 16 * w + f;
      if (c >= k_local) break;
      const int t = nl_trit(key, (grow0 + r) * k_full + c0 + c);
      const uint32_t code = t == 1 ? 1u : (t == -1 ? 3u : 0u);
      word |= code << (2 * f);
    }
    W[idx] = word;
  }
}

__global__ void gen_scale_kernel(float *S, uint32_t n, uint64_t key, uint64_t g0, float rs) {
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
    S[i] = __fmul_rn(__fadd_rn(0.5f, nl_unit(key, g0 + i)), rs);
}

__global__ void gen_norm_kernel(float *G, uint32_t n, uint64_t key) {
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
    G[i] = __fadd_rn(0.75f, __fmul_rn(0.5f, nl_unit(key, i)));
}

__global__ void gen_embed_kernel(float *E, uint64_t n, uint64_t key) {
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (uint64_t)gridDim.x * blockDim.x)
    E[i] = __fsub_rn(__fmul_rn(2.0f, nl_unit(key, i)), 1.0f);
}

// ---- step kernels ---------------------------------------------------------------------
namespace cg = cooperative_groups;

// ---- peer all-reduce (tensor parallelism over NVLink) ---------------------------------
// Each rank's O / down GEMV writes its partial rows into its slot of every
// rank's receive buffer (peer stores), every value a 64-bit word tagged with
// the index of this use of the slots (PeerOut); the next kernel on each rank
// polls each word until the tag shows up and sums the slots in rank order
// (so all ranks get the same bits).  The argmax keys go the same way with an
// arrival counter: the LM head's last CTA adds 1 to every rank's counter.  A
// rank cannot overwrite a slot for use u + 1 before every peer has read use
// u: writing use u + 1 needs results each peer computes only after its read
// of use u.  Every wait is bounded; one that gives up sets ERR, which the
// host reports after the generation.
constexpr uint32_t kPeerSpin = 1u << 22;   // polls (~100 ns apart) before giving up

struct PeerSig {
  unsigned long long *ctr[8];
  unsigned int *done;
  int n;
};

__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long *p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];\n" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ bool wait_count(const unsigned long long *ctr, unsigned long long target, int *err) {
  if (*reinterpret_cast<volatile int *>(err)) return false;   // an earlier wait gave up
  for (uint32_t i = 0; i < kPeerSpin; i++) {
    if (ld_acquire_sys(ctr) >= target) return true;
    __nanosleep(100);
  }
  atomicExch(err, 1);
  return false;
}
// The last CTA of the grid to get here arrives at every rank of SIG.
__device__ __forceinline__ void peer_signal(const PeerSig &sig) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    if (atomicInc(sig.done, gridDim.x - 1u) == gridDim.x - 1u) {
      __threadfence_system();
#pragma unroll
      for (int r = 0; r < 8; r++)        // constant indices: SIG stays in parameter space
        if (r < sig.n) atomicAdd_system(sig.ctr[r], 1ull);
    }
  }
}

// A reduction input: either DELTA (already summed) or the TP slots of this
// rank's receive buffer, whose words carry the tag *EP * TMUL + TADD once
// written for this use.
struct PeerIn {
  const unsigned long long *slots;   // nullptr: use delta
  uint32_t tp, slot_stride;          // slot r at slots + r * slot_stride
  const unsigned long long *ep;
  unsigned int tmul, tadd;
  int *err;
};

__device__ __forceinline__ unsigned long long ld_relaxed_sys(const unsigned long long *p) {
  unsigned long long v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];\n" : "=l"(v) : "l"(p) : "memory");
  return v;
}
// The f32 in word P once its tag is TAG (bounded poll; ERR on giving up).
__device__ __forceinline__ float tagged_value(const unsigned long long *p, uint32_t tag,
                                              int *err) {
  unsigned long long w = ld_relaxed_sys(p);
  if ((uint32_t)(w >> 32) != tag) {
    for (uint32_t i = 0; i < kPeerSpin; i++) {
      if (*reinterpret_cast<volatile int *>(err)) break;
      __nanosleep(32);
      w = ld_relaxed_sys(p);
      if ((uint32_t)(w >> 32) == tag) break;
      if (i + 1 == kPeerSpin) atomicExch(err, 1);
    }
  }
  return __uint_as_float((uint32_t)w);
}

enum { kNormGather = 0, kNormAdd = 1 };
constexpr int kNormThreads = 128;   // per CTA of a row cluster

// Row statistics exchanged between the CTAs of a row cluster.
struct RowStats {
  float v;     // partial sum of squares, then partial max |x|
  int bad;     // a non-finite value in this CTA's slice
};

// Sum (MAX = false) or maximum of the cluster's RowStats, read from every
// CTA's shared memory in rank order so that all CTAs get the same bits.
template <bool MAX>
__device__ __forceinline__ RowStats cluster_combine(cg::cluster_group &cl, RowStats *mine) {
  cl.sync();
  RowStats r{0.0f, 0};
#pragma unroll
  for (int k = 0; k < kRowCluster; k++) {
    const RowStats *o = cl.map_shared_rank(mine, k);
    r.v = MAX ? fmaxf(r.v, o->v) : r.v + o->v;
    r.bad |= o->bad;
  }
  return r;
}

// CTA-wide reduction of one value per thread into *OUT (thread 0 writes).
template <bool MAX>
__device__ __forceinline__ void cta_reduce(float v, int bad, float *red, RowStats *out) {
  for (int o = 16; o > 0; o >>= 1) {
    const float w = __shfl_xor_sync(0xffffffffu, v, o);
    v = MAX ? fmaxf(v, w) : v + w;
  }
  bad = __syncthreads_or(bad);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  if (threadIdx.x == 0) {
    float r = 0.0f;
    for (int i = 0; i < (int)(blockDim.x >> 5); i++) r = MAX ? fmaxf(r, red[i]) : r + red[i];
    out->v = r;
    out->bad = bad;
  }
}

// One cluster of kRowCluster CTAs per sequence row b: h = E[tok] (gather) or
// h = h + delta (add); x = (h * rsqrt(mean h^2 + eps)) * g; then x is
// converted into the next GEMV's activation fragments (when WS is set).
// Each CTA owns a column slice; the sum of squares and the maximum of x are
// combined across the cluster.
template <int MODE>
__global__ void __cluster_dims__(kRowCluster, 1, 1) __launch_bounds__(kNormThreads)
k_norm(const int *__restrict__ tok, const float *__restrict__ E, float *__restrict__ h,
       const float *__restrict__ delta, const float *__restrict__ g, float *__restrict__ x,
       void *ws, uint32_t B, uint32_t H, float eps, PeerIn pin) {
  pdl_trigger();                 // the next GEMV may start streaming its weights
  pdl_wait();
  const uint32_t tag = pin.slots ? (uint32_t)(*pin.ep * pin.tmul + pin.tadd) : 0u;
  extern __shared__ __align__(16) float xs[];
  __shared__ float red[32];
  __shared__ RowStats st[2];
  cg::cluster_group cl = cg::this_cluster();
  const uint32_t rank = cl.block_rank();
  const uint32_t b = blockIdx.x / kRowCluster;
  const RowSlice sl = row_slice(H, rank);
  const bool live = b < B;
  float mm = 0.0f;
  int bad = 0;
  if (live) {
    float *hb = h + (size_t)b * H;
    const float *src = MODE == kNormGather ? E + (size_t)__ldg(tok + b) * H : nullptr;
    float ss = 0.0f;
    for (uint32_t i = sl.c0 + threadIdx.x; i < sl.c1; i += blockDim.x) {
      float v;
      if (MODE == kNormGather) {
        v = __ldg(src + i);
      } else if (pin.slots) {
        const unsigned long long *sl = pin.slots + (size_t)b * H + i;
        float sum = tagged_value(sl, tag, pin.err);
        for (uint32_t r = 1; r < pin.tp; r++)
          sum = __fadd_rn(sum, tagged_value(sl + (size_t)r * pin.slot_stride, tag, pin.err));
        v = __fadd_rn(hb[i], sum);
      } else {
        v = __fadd_rn(hb[i], delta[(size_t)b * H + i]);
      }
      hb[i] = v;
      xs[i - sl.c0] = v;
      ss = fmaf(v, v, ss);
    }
    cta_reduce<false>(ss, 0, red, &st[0]);
    const RowStats tot = cluster_combine<false>(cl, &st[0]);
    const float rinv = 1.0f / sqrtf(tot.v / (float)H + eps);
    for (uint32_t i = sl.c0 + threadIdx.x; i < sl.c1; i += blockDim.x) {
      const float xv = __fmul_rn(__fmul_rn(xs[i - sl.c0], rinv), __ldg(g + i));
      xs[i - sl.c0] = xv;
      x[(size_t)b * H + i] = xv;
      mm = fmaxf(mm, fabsf(xv));
      bad |= !isfinite(xv);      // NaN is dropped by fmaxf; catch it here
    }
  } else {
    cl.sync();                   // keep the cluster's barrier count uniform
  }
  cta_reduce<true>(mm, bad, red, &st[1]);
  const RowStats mx = cluster_combine<true>(cl, &st[1]);
  if (ws) {
    __syncthreads();
    quantize_slice(xs, sl, mx.v, mx.bad != 0, live, rank, b, B,
                   prep_at(ws, (int)B, H, 0));
  }
  cl.sync();                     // no CTA leaves while its statistics are read
}

// The same per row in one CTA, one float4 of the row per thread (ROW4
// float4s a thread for longer rows): the row's statistics are two block
// reductions (warp shuffles, one barrier each) instead of the cluster's
// barriers and distributed-shared-memory reads, so a decode step's norm is
// one load round trip and a few barriers.  XS (dynamic shared memory) holds
// the row for the quantisation, which writes the CTA's offset sum to slot 0
// and zeroes the others.
template <int ROW4>
__device__ __forceinline__ void row_stats_quantize(float (&v)[ROW4][4], uint32_t cols, uint32_t b,
                                                   uint32_t B, float *xs, float *red, void *ws) {
  __shared__ long long xred[32];
  const int nw = (int)(blockDim.x >> 5), w = (int)(threadIdx.x >> 5), lane = (int)(threadIdx.x & 31);
  float mm = 0.0f;
  int bad = 0;
#pragma unroll
  for (int k = 0; k < ROW4; k++)
#pragma unroll
    for (int e = 0; e < 4; e++) {
      mm = fmaxf(mm, fabsf(v[k][e]));
      bad |= !isfinite(v[k][e]);
    }
  for (int o = 16; o > 0; o >>= 1) mm = fmaxf(mm, __shfl_xor_sync(0xffffffffu, mm, o));
  if (lane == 0) red[w] = mm;
  bad = __syncthreads_or(bad);
  float rm = 0.0f;
  for (int i = 0; i < nw; i++) rm = fmaxf(rm, red[i]);
  if (!ws) return;
  const int NT = n_tiles((int)B), L = n_limbs((int)B);
  PrepOut P = prep_at(ws, (int)B, cols, 0);
  float mul = 0.0f, inv = 0.0f;
  const bool ok = row_scale(rm, bad != 0, &mul, &inv, L);
  if (threadIdx.x == 0) {
    P.rowinv[b] = inv;
    P.rowflag[b] = !ok;
  }
  long long part = 0;
  for (uint32_t W = threadIdx.x; W < cols / 16u; W += blockDim.x) {
    float q[16];
    const float4 *x4 = reinterpret_cast<const float4 *>(xs + 16u * W);
#pragma unroll
    for (int e = 0; e < 4; e++) {
      const float4 f = x4[e];
      q[4 * e] = f.x; q[4 * e + 1] = f.y; q[4 * e + 2] = f.z; q[4 * e + 3] = f.w;
    }
    part += quantize_word(q, mul, ok, W, b, NT, L, P);
  }
  for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
  if (lane == 0) xred[w] = part;
  __syncthreads();
  if (threadIdx.x < (unsigned)kRowCluster) {
    long long t = 0;
    if (threadIdx.x == 0)
      for (int i = 0; i < nw; i++) t += xred[i];
    P.xsum[b * kRowCluster + threadIdx.x] = t;
  }
}

// h = E[tok] (gather) or h = h + delta; x = (h * rsqrt(mean h^2 + eps)) * g
// and the next GEMV's prep: one CTA of cols/4 threads per sequence row.
template <int MODE>
__global__ void __launch_bounds__(1024)
k_norm_cta(const int *__restrict__ tok, const float *__restrict__ E, float *__restrict__ h,
           const float *__restrict__ delta, const float *__restrict__ g, float *__restrict__ x,
           void *ws, uint32_t B, uint32_t H, float eps, PeerIn pin) {
  pdl_trigger();
  extern __shared__ __align__(16) float xs[];
  __shared__ float red[32];
  const uint32_t b = blockIdx.x, t = threadIdx.x;
  const bool in = 4u * t < H;
  // gamma is a weight, and the residual row was written by the norm kernel
  // several launches back: both are requested before the wait.  That read
  // is ordered because the kernel before this one (a GEMV, which does not
  // trigger its dependents early) starts only after that norm kernel has
  // completed, and this one only after it.
  const float4 gv = in ? __ldg(reinterpret_cast<const float4 *>(g) + t) : make_float4(0.f, 0.f, 0.f, 0.f);
  float4 *h4 = reinterpret_cast<float4 *>(h + (size_t)b * H);
  const float4 hpre = (in && MODE != kNormGather) ? h4[t] : make_float4(0.f, 0.f, 0.f, 0.f);
  pdl_wait();
  const uint32_t tag = pin.slots ? (uint32_t)(*pin.ep * pin.tmul + pin.tadd) : 0u;
  float v[1][4] = {{0.0f, 0.0f, 0.0f, 0.0f}};
  if (in) {
    if (MODE == kNormGather) {
      const float4 f = __ldg(reinterpret_cast<const float4 *>(E + (size_t)__ldg(tok + b) * H) + t);
      v[0][0] = f.x; v[0][1] = f.y; v[0][2] = f.z; v[0][3] = f.w;
    } else {
      const float4 f = hpre;
      const float hv[4] = {f.x, f.y, f.z, f.w};
      float dv[4];
      if (pin.slots) {
#pragma unroll
        for (int e = 0; e < 4; e++) {
          const unsigned long long *sl = pin.slots + (size_t)b * H + 4u * t + e;
          float sum = tagged_value(sl, tag, pin.err);
          for (uint32_t r = 1; r < pin.tp; r++)
            sum = __fadd_rn(sum, tagged_value(sl + (size_t)r * pin.slot_stride, tag, pin.err));
          dv[e] = sum;
        }
      } else {
        const float4 d = reinterpret_cast<const float4 *>(delta + (size_t)b * H)[t];
        dv[0] = d.x; dv[1] = d.y; dv[2] = d.z; dv[3] = d.w;
      }
#pragma unroll
      for (int e = 0; e < 4; e++) v[0][e] = __fadd_rn(hv[e], dv[e]);
    }
    h4[t] = make_float4(v[0][0], v[0][1], v[0][2], v[0][3]);
  }
  float ss = 0.0f;
#pragma unroll
  for (int e = 0; e < 4; e++) ss = fmaf(v[0][e], v[0][e], ss);
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((t & 31) == 0) red[t >> 5] = ss;
  __syncthreads();
  float tot = 0.0f;
  for (int i = 0; i < (int)(blockDim.x >> 5); i++) tot += red[i];
  const float rinv = 1.0f / sqrtf(tot / (float)H + eps);
  __syncthreads();   // red is reused
  if (in) {
    v[0][0] = __fmul_rn(__fmul_rn(v[0][0], rinv), gv.x);
    v[0][1] = __fmul_rn(__fmul_rn(v[0][1], rinv), gv.y);
    v[0][2] = __fmul_rn(__fmul_rn(v[0][2], rinv), gv.z);
    v[0][3] = __fmul_rn(__fmul_rn(v[0][3], rinv), gv.w);
    const float4 xv = make_float4(v[0][0], v[0][1], v[0][2], v[0][3]);
    reinterpret_cast<float4 *>(x + (size_t)b * H)[t] = xv;
    reinterpret_cast<float4 *>(xs)[t] = xv;
  }
  row_stats_quantize<1>(v, H, b, B, xs, red, ws);
}

// a = silu(gate) * up and the down GEMV's prep: one CTA per sequence row,
// ROW4 float4 of the row per thread.
template <int ROW4>
__global__ void __launch_bounds__(1024)
k_silu_cta(const float *__restrict__ gu, float *__restrict__ a, void *ws, uint32_t B,
           uint32_t fr) {
  pdl_trigger();
  pdl_wait();
  extern __shared__ __align__(16) float xs[];
  __shared__ float red[32];
  const uint32_t b = blockIdx.x;
  const float4 *g4 = reinterpret_cast<const float4 *>(gu + (size_t)b * 2 * fr);
  const float4 *u4 = reinterpret_cast<const float4 *>(gu + (size_t)b * 2 * fr + fr);
  float v[ROW4][4];
#pragma unroll
  for (int k = 0; k < ROW4; k++) {
    const uint32_t i = threadIdx.x + (uint32_t)k * blockDim.x;
    if (4u * i < fr) {
      const float4 gv = g4[i], uv = u4[i];
      const float gg[4] = {gv.x, gv.y, gv.z, gv.w}, uu[4] = {uv.x, uv.y, uv.z, uv.w};
#pragma unroll
      for (int e = 0; e < 4; e++) {
        const float sg = 1.0f / (1.0f + expf(-gg[e]));
        v[k][e] = __fmul_rn(__fmul_rn(gg[e], sg), uu[e]);
      }
      const float4 av = make_float4(v[k][0], v[k][1], v[k][2], v[k][3]);
      reinterpret_cast<float4 *>(a + (size_t)b * fr)[i] = av;
      reinterpret_cast<float4 *>(xs)[i] = av;
    } else {
#pragma unroll
      for (int e = 0; e < 4; e++) v[k][e] = 0.0f;
    }
  }
  row_stats_quantize<ROW4>(v, fr, b, B, xs, red, ws);
}

// a = silu(gate) * up, then the down GEMV's prep: one cluster per sequence
// row, each CTA on its column slice, the row maximum combined across the
// cluster.
__global__ void __cluster_dims__(kRowCluster, 1, 1) __launch_bounds__(kNormThreads)
k_silu_prep(const float *__restrict__ gu, float *__restrict__ a, void *ws, uint32_t B,
            uint32_t fr) {
  pdl_trigger();
  pdl_wait();
  extern __shared__ __align__(16) float xs[];
  __shared__ float red[32];
  __shared__ RowStats st;
  cg::cluster_group cl = cg::this_cluster();
  const uint32_t rank = cl.block_rank();
  const uint32_t b = blockIdx.x / kRowCluster;
  const RowSlice sl = row_slice(fr, rank);
  const bool live = b < B;
  float mm = 0.0f;
  int bad = 0;
  if (live) {
    const float *gr = gu + (size_t)b * 2 * fr;
    for (uint32_t j = sl.c0 + threadIdx.x; j < sl.c1; j += blockDim.x) {
      const float gv = gr[j], uv = gr[fr + j];
      const float sg = 1.0f / (1.0f + expf(-gv));
      const float v = __fmul_rn(__fmul_rn(gv, sg), uv);
      xs[j - sl.c0] = v;
      a[(size_t)b * fr + j] = v;
      mm = fmaxf(mm, fabsf(v));
      bad |= !isfinite(v);
    }
  }
  cta_reduce<true>(mm, bad, red, &st);
  const RowStats mx = cluster_combine<true>(cl, &st);
  if (ws) {
    __syncthreads();
    quantize_slice(xs, sl, mx.v, mx.bad != 0, live, rank, b, B,
                   prep_at(ws, (int)B, fr, 0));
  }
  cl.sync();
}

// Prefill rows (hundreds of them fill the GPU without splitting a row): one
// CTA per row, float4 streams.  The same per-element arithmetic as k_norm /
// k_silu_prep; the sum of squares is reduced in a different order.
constexpr int kRowThreads = 256;
__global__ void __launch_bounds__(kRowThreads)
k_rows_add_norm(float *__restrict__ h, const float *__restrict__ delta,
                const float *__restrict__ g, float *__restrict__ x, uint32_t H, float eps) {
  __shared__ float red[kRowThreads / 32];
  const size_t base = (size_t)blockIdx.x * H;
  float4 *h4 = reinterpret_cast<float4 *>(h + base);
  const float4 *d4 = reinterpret_cast<const float4 *>(delta + base);
  float ss = 0.0f;
  for (uint32_t i = threadIdx.x; i < H / 4u; i += blockDim.x) {
    const float4 a = h4[i], b = __ldg(d4 + i);
    const float4 v = make_float4(__fadd_rn(a.x, b.x), __fadd_rn(a.y, b.y), __fadd_rn(a.z, b.z),
                                 __fadd_rn(a.w, b.w));
    h4[i] = v;
    ss = fmaf(v.x, v.x, ss);
    ss = fmaf(v.y, v.y, ss);
    ss = fmaf(v.z, v.z, ss);
    ss = fmaf(v.w, v.w, ss);
  }
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.0f;
#pragma unroll
  for (int w = 0; w < kRowThreads / 32; w++) tot += red[w];
  const float rinv = 1.0f / sqrtf(tot / (float)H + eps);
  float4 *x4 = reinterpret_cast<float4 *>(x + base);
  const float4 *g4 = reinterpret_cast<const float4 *>(g);
  for (uint32_t i = threadIdx.x; i < H / 4u; i += blockDim.x) {
    const float4 v = h4[i], gv = __ldg(g4 + i);   // this thread's own writes above
    x4[i] = make_float4(__fmul_rn(__fmul_rn(v.x, rinv), gv.x), __fmul_rn(__fmul_rn(v.y, rinv), gv.y),
                        __fmul_rn(__fmul_rn(v.z, rinv), gv.z), __fmul_rn(__fmul_rn(v.w, rinv), gv.w));
  }
}
__global__ void __launch_bounds__(kRowThreads)
k_rows_silu(const float *__restrict__ gu, float *__restrict__ a, uint32_t fr) {
  const float *gr = gu + (size_t)blockIdx.x * 2 * fr;
  const float4 *g4 = reinterpret_cast<const float4 *>(gr);
  const float4 *u4 = reinterpret_cast<const float4 *>(gr + fr);
  float4 *a4 = reinterpret_cast<float4 *>(a + (size_t)blockIdx.x * fr);
  for (uint32_t i = threadIdx.x; i < fr / 4u; i += blockDim.x) {
    const float4 gv = __ldg(g4 + i), uv = __ldg(u4 + i);
    const float gg[4] = {gv.x, gv.y, gv.z, gv.w}, uu[4] = {uv.x, uv.y, uv.z, uv.w};
    float r[4];
#pragma unroll
    for (int e = 0; e < 4; e++) {
      const float sg = 1.0f / (1.0f + expf(-gg[e]));
      r[e] = __fmul_rn(__fmul_rn(gg[e], sg), uu[e]);
    }
    a4[i] = make_float4(r[0], r[1], r[2], r[3]);
  }
}

// Order-preserving 64-bit argmax key: larger logit first, then lower index.
__device__ __forceinline__ unsigned long long argmax_key(float v, uint32_t idx) {
  uint32_t u = __float_as_uint(v);
  u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  if (v != v) u = 0;   // NaN never wins
  return ((unsigned long long)u << 32) | (0xFFFFFFFFu - idx);
}

// LM head over this rank's vocabulary rows with the argmax fused: each warp
// takes RPW consecutive rows at a time, lanes stride the hidden dimension in
// float4 steps against x held in shared memory.
template <int NB>
__global__ void __launch_bounds__(256, 2)
k_lmhead(const float *__restrict__ E, const float *__restrict__ x,
         unsigned long long *__restrict__ keys, float *__restrict__ logits,
         const int *__restrict__ pos, uint32_t B, uint32_t vr, uint32_t v0, uint32_t H,
         uint32_t logit_stride, const unsigned long long *ep, uint32_t key_stride,
         PeerSig sig) {
  pdl_trigger();
  pdl_wait();
  constexpr int RPW = 4;
  // Keys of this step: slot ep % 2 when the ranks exchange them peer to peer.
  if (sig.n) keys += (*ep & 1ull) * key_stride;
  extern __shared__ __align__(16) float xs[];   // [NB][H]
  for (uint32_t i = threadIdx.x; i < NB * H; i += blockDim.x)
    xs[i] = (i / H) < B ? x[i] : 0.0f;
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const uint32_t gw = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const uint32_t nw = gridDim.x * (blockDim.x >> 5);
  const uint32_t h4 = H / 4;
  unsigned long long best[NB];
#pragma unroll
  for (int b = 0; b < NB; b++) best[b] = 0ull;
  float *lg = logits ? logits + (size_t)(*pos) * logit_stride : nullptr;
  for (uint32_t r0 = gw * RPW; r0 < vr; r0 += nw * RPW) {
    float acc[RPW][NB];
#pragma unroll
    for (int r = 0; r < RPW; r++)
#pragma unroll
      for (int b = 0; b < NB; b++) acc[r][b] = 0.0f;
    const float4 *er[RPW];
#pragma unroll
    for (int r = 0; r < RPW; r++)
      er[r] = reinterpret_cast<const float4 *>(E + (size_t)min(r0 + r, vr - 1) * H);
    // the next column step's float4s are requested before this step's FMAs
    float4 ev[RPW];
#pragma unroll
    for (int r = 0; r < RPW; r++)
      ev[r] = (uint32_t)lane < h4 ? __ldcs(er[r] + lane) : make_float4(0.f, 0.f, 0.f, 0.f);
    for (uint32_t c = lane; c < h4; c += 32) {
      float4 en[RPW];
#pragma unroll
      for (int r = 0; r < RPW; r++)
        en[r] = c + 32 < h4 ? __ldcs(er[r] + c + 32) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int b = 0; b < NB; b++) {
        const float4 xv = reinterpret_cast<const float4 *>(xs + (size_t)b * H)[c];
#pragma unroll
        for (int r = 0; r < RPW; r++) {
          acc[r][b] = fmaf(ev[r].x, xv.x, acc[r][b]);
          acc[r][b] = fmaf(ev[r].y, xv.y, acc[r][b]);
          acc[r][b] = fmaf(ev[r].z, xv.z, acc[r][b]);
          acc[r][b] = fmaf(ev[r].w, xv.w, acc[r][b]);
        }
      }
#pragma unroll
      for (int r = 0; r < RPW; r++) ev[r] = en[r];
    }
#pragma unroll
    for (int r = 0; r < RPW; r++) {
#pragma unroll
      for (int b = 0; b < NB; b++) {
        float v = acc[r][b];
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        const uint32_t row = r0 + r;
        if (row < vr && (uint32_t)b < B) {
          const unsigned long long k = argmax_key(v, v0 + row);
          if (k > best[b]) best[b] = k;
          if (lg && lane == 0) lg[(size_t)b * vr + row] = v;
        }
      }
    }
  }
  if (lane == 0)
    for (int b = 0; b < NB; b++)
      if ((uint32_t)b < B && best[b]) atomicMax(keys + b, best[b]);
  if (sig.n) peer_signal(sig);
}

// The LM head for 2 to 8 sequence rows: k_lmhead's arithmetic (the same
// per-lane column order, warp reduction and argmax keys, so the same bits),
// with the embedding rows streamed into shared memory by cp.async instead of
// registers.  Every warp keeps kLmStages column steps of its 4 rows in
// flight in its own ring slots (2 KB a step), and each lane reads back only
// the 16-byte pieces it copied itself, so a thread's own cp.async wait orders
// them.  One CTA of 16 warps an SM: with 8 rows of x (80 KB) and the 128 KB
// of rings, twice the bytes in flight of k_lmhead<8>, whose registers hold
// them.  The first steps are requested before the programmatic-launch wait
// (the embeddings are not written by the preceding kernel).  Needs H % 128
// == 0.
constexpr int kLmWarps = 16, kLmStages = 4, kLmRows = 4;
__host__ __device__ inline size_t lmhead_ring_smem(int NB, uint32_t H) {
  return (size_t)NB * H * 4u + (size_t)kLmWarps * kLmStages * kLmRows * 32u * 16u;
}
__device__ __forceinline__ void lm_cp16(void *smem, const void *gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n"
               ::"r"((unsigned)__cvta_generic_to_shared(smem)), "l"(gmem) : "memory");
}
__device__ __forceinline__ void lm_cp_commit() {
  asm volatile("cp.async.commit_group;\n" ::: "memory");
}
__device__ __forceinline__ void lm_cp_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(kLmStages - 1) : "memory");
}
template <int NB>
__global__ void __launch_bounds__(kLmWarps * 32, 1)
k_lmhead_ring(const float *__restrict__ E, const float *__restrict__ x,
              unsigned long long *__restrict__ keys, float *__restrict__ logits,
              const int *__restrict__ pos, uint32_t B, uint32_t vr, uint32_t v0, uint32_t H,
              uint32_t logit_stride, const unsigned long long *ep, uint32_t key_stride,
              PeerSig sig) {
  pdl_trigger();
  extern __shared__ __align__(16) float lsm[];
  float *xs = lsm;                                              // [NB][H]
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float4 *wr = reinterpret_cast<float4 *>(lsm + (size_t)NB * H) +
               (size_t)warp * kLmStages * kLmRows * 32 + lane;   // this lane's ring slots
  const uint32_t gw = blockIdx.x * kLmWarps + (uint32_t)warp;
  const uint32_t nw = gridDim.x * kLmWarps;
  const uint32_t h4 = H / 4, ks = h4 / 32;                      // column steps of a row group
  const uint32_t groups = (vr + kLmRows - 1) / kLmRows;
  const uint32_t mine = groups > gw ? (groups - gw + nw - 1) / nw : 0u;
  const uint32_t total = mine * ks;                             // this warp's steps
  // step i: row group gw + (i / ks) nw, columns 4 (lane + 32 (i % ks)) .. +3
  auto issue = [&](uint32_t i) {
    if (i < total) {
      const uint32_t r0 = (gw + (i / ks) * nw) * kLmRows, c = (uint32_t)lane + 32u * (i % ks);
      float4 *dst = wr + (size_t)(i % kLmStages) * kLmRows * 32;
#pragma unroll
      for (int u = 0; u < kLmRows; u++)
        lm_cp16(dst + u * 32, E + (size_t)min(r0 + (uint32_t)u, vr - 1) * H + 4u * c);
    }
    lm_cp_commit();                  // empty groups keep the count uniform
  };
#pragma unroll
  for (int i = 0; i < kLmStages; i++) issue((uint32_t)i);
  pdl_wait();
  if (sig.n) keys += (*ep & 1ull) * key_stride;
  for (uint32_t i = threadIdx.x; i < NB * h4; i += blockDim.x)
    reinterpret_cast<float4 *>(xs)[i] = (i / h4) < B ? reinterpret_cast<const float4 *>(x)[i]
                                                     : make_float4(0.f, 0.f, 0.f, 0.f);
  __syncthreads();
  unsigned long long best[NB];
#pragma unroll
  for (int b = 0; b < NB; b++) best[b] = 0ull;
  float *lg = logits ? logits + (size_t)(*pos) * logit_stride : nullptr;
  for (uint32_t g0 = 0; g0 < total; g0 += ks) {
    float acc[kLmRows][NB];
#pragma unroll
    for (int r = 0; r < kLmRows; r++)
#pragma unroll
      for (int b = 0; b < NB; b++) acc[r][b] = 0.0f;
    for (uint32_t k = 0; k < ks; k++) {
      const uint32_t i = g0 + k;
      lm_cp_wait();                  // step i has landed (this thread's copies)
      const float4 *src = wr + (size_t)(i % kLmStages) * kLmRows * 32;
      float4 ev[kLmRows];
#pragma unroll
      for (int r = 0; r < kLmRows; r++) ev[r] = src[r * 32];
      const uint32_t c = (uint32_t)lane + 32u * k;
#pragma unroll
      for (int b = 0; b < NB; b++) {
        const float4 xv = reinterpret_cast<const float4 *>(xs + (size_t)b * H)[c];
#pragma unroll
        for (int r = 0; r < kLmRows; r++) {
          acc[r][b] = fmaf(ev[r].x, xv.x, acc[r][b]);
          acc[r][b] = fmaf(ev[r].y, xv.y, acc[r][b]);
          acc[r][b] = fmaf(ev[r].z, xv.z, acc[r][b]);
          acc[r][b] = fmaf(ev[r].w, xv.w, acc[r][b]);
        }
      }
      issue(i + kLmStages);          // into the slots just read (their values are used)
    }
    const uint32_t r0 = (gw + (g0 / ks) * nw) * kLmRows;
#pragma unroll
    for (int r = 0; r < kLmRows; r++) {
#pragma unroll
      for (int b = 0; b < NB; b++) {
        float v = acc[r][b];
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        const uint32_t row = r0 + r;
        if (row < vr && (uint32_t)b < B) {
          const unsigned long long kk = argmax_key(v, v0 + row);
          if (kk > best[b]) best[b] = kk;
          if (lg && lane == 0) lg[(size_t)b * vr + row] = v;
        }
      }
    }
  }
  asm volatile("cp.async.wait_all;\n" ::: "memory");
  if (lane == 0)
    for (int b = 0; b < NB; b++)
      if ((uint32_t)b < B && best[b]) atomicMax(keys + b, best[b]);
  if (sig.n) peer_signal(sig);
}

// Next token: from the prompt while it lasts, else the argmax; reset the
// keys and advance the position.  One CTA.
// With peer keys (PK.n > 0): wait for every rank's LM head of this step, take
// the maximum of the ranks' keys, clear this rank's keys of the next step.
struct PeerKeys {
  const unsigned long long *keys[8];   // every rank's two key slots
  int n;
  uint32_t stride;                     // keys per slot
  const unsigned long long *ctr;
  int *err;
};
__global__ void k_next(unsigned long long *keys, const int *prompt, uint32_t P, int *tok,
                       int *out_tok, int *pos, float *posf, uint32_t B, unsigned long long *ep,
                       PeerKeys pk) {
  pdl_trigger();
  pdl_wait();
  const int p = *pos;
  const unsigned long long e = *ep;
  const uint32_t b = threadIdx.x;
  if (pk.n) {
    if (threadIdx.x == 0) wait_count(pk.ctr, (e + 1ull) * (unsigned long long)pk.n, pk.err);
    __syncthreads();
  }
  if (b < B) {
    unsigned long long key;
    if (pk.n) {
      key = 0ull;
#pragma unroll
      for (int r = 0; r < 8; r++) {      // constant indices: PK stays in parameter space
        if (r >= pk.n) break;
        const unsigned long long k = ld_acquire_sys(pk.keys[r] + (e & 1ull) * pk.stride + b);
        key = k > key ? k : key;
      }
    } else {
      key = keys[b];
    }
    const uint32_t idx = 0xFFFFFFFFu - (uint32_t)(key & 0xFFFFFFFFull);
    int nt;
    if ((uint32_t)p + 1 < P) {
      nt = prompt[(size_t)b * P + p + 1];
    } else {
      nt = (int)idx;
      out_tok[(size_t)(p + 1 - P) * B + b] = nt;
    }
    tok[b] = nt;
    if (!pk.n) keys[b] = 0ull;
  }
  // the next step's slot, for every batch row a later generation may use
  if (pk.n && b < pk.stride) keys[((e + 1ull) & 1ull) * pk.stride + b] = 0ull;
  __syncthreads();
  if (threadIdx.x == 0) {
    *pos = p + 1;
    *posf = (float)(p + 1);
    *ep = e + 1ull;
  }
}

__global__ void k_init(const int *prompt, uint32_t P, int *tok, unsigned long long *keys, int *pos,
                       float *posf, uint32_t B) {
  const uint32_t b = threadIdx.x;
  if (b < B) {
    tok[b] = prompt[(size_t)b * P];
    if (keys) keys[b] = 0ull;   // peer-exchanged keys are cleared by k_next only
  }
  if (threadIdx.x == 0) {
    *pos = 0;
    *posf = 0.0f;
  }
}

// ---- batched prefill ----------------------------------------------------------------
// Positions 0 .. P-2 of every sequence in one pass per layer (rows r = b * n + t,
// n = P - 1): the same layer math as the decode step, with the GEMMs on the
// tcgen05 kernel and causal attention over the prompt; it fills the KV cache,
// and decoding continues with the last prompt token at position P - 1.

// Row r's token: prompt[b * P + t].
__global__ void k_pf_tokens(const int *prompt, uint32_t P, uint32_t n, uint32_t B, int *tok) {
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < B * n; i += gridDim.x * blockDim.x)
    tok[i] = prompt[(size_t)(i / n) * P + i % n];
}

// RoPE of q and k at position t (the decode step's cos/sin table) and the
// cache append of k and v, for every prefill row.
__global__ void k_pf_rope(const float *__restrict__ qkv, float *__restrict__ q,
                          float *__restrict__ ck, float *__restrict__ cv,
                          const float2 *__restrict__ rope, uint32_t B, uint32_t n, uint32_t hr,
                          uint32_t kvr, uint32_t hd, uint32_t maxseq) {
  const uint32_t half = hd / 2, nh = hr + 2 * kvr, rowlen = nh * hd, kvdim = kvr * hd;
  const uint64_t total = (uint64_t)B * n * nh * half;
  for (uint64_t idx = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (uint64_t)gridDim.x * blockDim.x) {
    const uint32_t m = (uint32_t)(idx % half);
    const uint32_t head = (uint32_t)((idx / half) % nh);
    const uint32_t r = (uint32_t)(idx / ((uint64_t)half * nh));
    const uint32_t b = r / n, t = r % n;
    const float *src = qkv + (size_t)r * rowlen + (size_t)head * hd;
    const float a0 = src[m], a1 = src[m + half];
    if (head < hr + kvr) {
      const float2 cs = rope[(size_t)t * half + m];
      const float y0 = __fsub_rn(__fmul_rn(a0, cs.x), __fmul_rn(a1, cs.y));
      const float y1 = __fadd_rn(__fmul_rn(a1, cs.x), __fmul_rn(a0, cs.y));
      float *dst = head < hr ? q + (size_t)r * hr * hd + (size_t)head * hd
                             : ck + ((size_t)b * maxseq + t) * kvdim + (size_t)(head - hr) * hd;
      dst[m] = y0;
      dst[m + half] = y1;
    } else {
      float *dst = cv + ((size_t)b * maxseq + t) * kvdim + (size_t)(head - hr - kvr) * hd;
      dst[m] = a0;
      dst[m + half] = a1;
    }
  }
}

// After the batched prefill: position P - 1 and its token.
__global__ void k_pf_init(const int *prompt, uint32_t P, int *tok, unsigned long long *keys,
                          int *pos, float *posf, uint32_t B) {
  const uint32_t b = threadIdx.x;
  if (b < B) {
    tok[b] = prompt[(size_t)b * P + P - 1];
    if (keys) keys[b] = 0ull;
  }
  if (threadIdx.x == 0) {
    *pos = (int)P - 1;
    *posf = (float)(P - 1);
  }
}

}  // namespace

// ---- the decoder object -------------------------------------------------------------------
struct Layer {
  uint32_t *wqkv = nullptr, *wo = nullptr, *wgu = nullptr, *wd = nullptr;
  float *sqkv = nullptr, *so = nullptr, *sgu = nullptr, *sd = nullptr;
  float *gattn = nullptr, *gffn = nullptr;
  float *ck = nullptr, *cv = nullptr;
};

}  // namespace nl

struct nl_decoder {
  nl_decoder_config cfg;
  int rank = 0, size = 1;
  nl::ncclComm_t comm = nullptr;
  cudaStream_t stream = nullptr;
  nl::Split kvh, ffb, voc;
  uint32_t hr = 0, kvr = 0, fr = 0, vr = 0, v0 = 0, qkv_rows = 0;
  std::vector<nl::Layer> layers;
  float *embed = nullptr, *gfinal = nullptr;
  // activations
  float *h = nullptr, *x = nullptr, *qkv = nullptr, *ctx = nullptr, *o = nullptr,
        *gu = nullptr, *a = nullptr, *d = nullptr, *posf = nullptr, *logits = nullptr;
  int *tok = nullptr, *prompt = nullptr, *out_tok = nullptr, *pos = nullptr;
  unsigned long long *keys = nullptr;
  void *ws_qkv = nullptr, *ws_o = nullptr, *ws_gu = nullptr, *ws_d = nullptr, *attn_scr = nullptr;
  int *attn_ctr = nullptr;       // per sequence row: heads combined (the O prep's trigger)
  float2 *rope = nullptr;   // [max_seq][head_dim / 2] (cos, sin)
  // Peer all-reduce (tensor parallelism): this rank's block of counters,
  // key slots and receive slots, exported to the peers; every rank's block
  // mapped here (own included).
  // batched prefill buffers (rows = batch * (prompt - 1)), grown on demand
  uint32_t pf_cap = 0;
  std::vector<void *> pf_allocs;
  int *pf_tok = nullptr;
  float *pf_h = nullptr, *pf_x = nullptr, *pf_qkv = nullptr, *pf_q = nullptr, *pf_ctx = nullptr,
        *pf_o = nullptr, *pf_gu = nullptr, *pf_a = nullptr, *pf_d = nullptr;
  void *pf_ws = nullptr;
  size_t pf_ws_bytes = 0;
  bool par = false;
  char *par_local = nullptr;
  char *par_peer[8] = {};
  unsigned long long *ep = nullptr;   // decode steps completed
  int *err = nullptr;                 // a peer wait gave up
  bool keep_logits = false;
  std::map<uint32_t, cudaGraphExec_t> graphs;   // by batch
  uint64_t kernels_per_step = 0;
  uint64_t weight_bytes = 0;
  std::vector<void *> allocs;
  uint32_t last_batch = 0, last_positions = 0;
  const nl_decoder_weights *src = nullptr;   // caller's weights while building, or synthetic
  // the one-kernel decode step (nl_step.cu), when the shapes allow it
  bool step_ok = false;
  nl::StepLayer *step_layers = nullptr;   // [layers], device
  float *step_h = nullptr;                // [2][max_batch][hidden]
  unsigned *step_acnt = nullptr, *step_amax = nullptr;
  long long *step_dpart = nullptr;
  unsigned long long *step_bar = nullptr;  // [0] barrier arrivals, [1] launches completed
};

namespace nl {
namespace {

int dalloc(nl_decoder *D, void **p, size_t bytes) {
  cudaError_t e = cudaMalloc(p, bytes ? bytes : 16);
  if (e != cudaSuccess) return cuda_status(e, "decoder: cudaMalloc");
  D->allocs.push_back(*p);
  return NL_OK;
}
#define DALLOC(ptr, bytes)                                            \
  do {                                                                \
    int rc_ = dalloc(D, reinterpret_cast<void **>(&(ptr)), (bytes));  \
    if (rc_) return rc_;                                              \
  } while (0)

float inv_sqrt_fan(uint64_t k) { return (float)(1.0 / sqrt(2.0 * (double)k / 3.0)); }

int gen_ternary(nl_decoder *D, uint32_t *W, uint32_t rows, uint32_t k_local, uint64_t tensor,
                uint64_t grow0, uint64_t k_full, uint64_t c0) {
  uint64_t key = nl_tensor_key(D->cfg.seed, tensor);
  uint64_t n = (uint64_t)rows * ((k_local + 15) / 16);
  gen_ternary_kernel<<<grid_for(n, 256), 256, 0, D->stream>>>(W, rows, k_local, key, grow0,
                                                             k_full, c0);
  return cuda_status(cudaPeekAtLastError(), "decoder: weights");
}
int gen_scale(nl_decoder *D, float *S, uint32_t n, uint64_t tensor, uint64_t g0, uint64_t k_full) {
  gen_scale_kernel<<<grid_for(n, 256), 256, 0, D->stream>>>(
      S, n, nl_tensor_key(D->cfg.seed, tensor), g0, inv_sqrt_fan(k_full));
  return cuda_status(cudaPeekAtLastError(), "decoder: scales");
}
int gen_norm(nl_decoder *D, float *G, uint32_t n, uint64_t tensor) {
  gen_norm_kernel<<<grid_for(n, 256), 256, 0, D->stream>>>(G, n,
                                                            nl_tensor_key(D->cfg.seed, tensor));
  return cuda_status(cudaPeekAtLastError(), "decoder: norms");
}

int allreduce(nl_decoder *D, void *buf, size_t count, int dtype, int op) {
  if (D->size <= 1) return NL_OK;
  Nccl *n = nccl();
  ncclResult_t r = n->AllReduce(buf, buf, count, dtype, op, D->comm, D->stream);
  if (r != 0)
    return set_error(NL_ERROR, "ncclAllReduce: %s", n->GetErrorString ? n->GetErrorString(r) : "?");
  return NL_OK;
}

// Layout of a rank's peer block: arrival counters (set 2: argmax keys), CTA
// completion counters, two slots of argmax keys, then the receive slots of
// sets 0 (O-proj) and 1 (down): [rank][max_batch][hidden] tagged words.
constexpr size_t kParCtr = 0, kParDone = 64, kParKeys = 256, kParSlots = 1024;
size_t par_set_bytes(const nl_decoder *D) {
  return align256((size_t)D->size * D->cfg.max_batch * D->cfg.hidden * 8u);
}
size_t par_bytes(const nl_decoder *D) { return kParSlots + 2 * par_set_bytes(D); }
unsigned long long *par_slot(const nl_decoder *D, char *base, int set, int rank) {
  return reinterpret_cast<unsigned long long *>(base + kParSlots +
                                                (size_t)set * par_set_bytes(D)) +
         (size_t)rank * D->cfg.max_batch * D->cfg.hidden;
}
unsigned long long *par_ctr(char *base, int set) {
  return reinterpret_cast<unsigned long long *>(base + kParCtr) + set;
}
unsigned int *par_done(char *base, int set) {
  return reinterpret_cast<unsigned int *>(base + kParDone) + set;
}
unsigned long long *par_keys(char *base) {
  return reinterpret_cast<unsigned long long *>(base + kParKeys);
}

// Enqueue one decode step for batch B on D->stream.
int enqueue_step(nl_decoder *D, uint32_t B) {
  const nl_decoder_config &c = D->cfg;
  const uint32_t H = c.hidden, hd = c.head_dim;
  const float eps = c.rms_eps;
  cudaStream_t st = D->stream;
  const uint32_t gnorm = B * kRowCluster;
  const size_t smem_h = (size_t)row_slice_cols(H) * sizeof(float);
  // One CTA per row (a float4 a thread) where the row fits 1024 threads;
  // else the 8-CTA clusters.  NELISP_DECODER_NORM=cluster keeps the clusters.
  static const bool cluster_norm = [] {
    const char *v = getenv("NELISP_DECODER_NORM");
    return v && strcmp(v, "cluster") == 0;
  }();
  const bool cta_rows = !cluster_norm && H % 128u == 0 && H / 4u <= 1024u;
  const uint32_t norm_threads = (H / 4u + 31u) / 32u * 32u;
  const uint32_t silu_row4 = cluster_norm || D->fr % 128u ? 0u
                             : D->fr / 4u <= 1024u        ? 1u
                             : D->fr / 4u <= 2048u        ? 2u
                                                          : 0u;
  const uint32_t silu_threads =
      silu_row4 ? ((D->fr / 4u + silu_row4 - 1u) / silu_row4 + 31u) / 32u * 32u : 0u;
  const bool fast_o = ternary_fast_shape(D->hr * hd, D->hr * hd / 128, D->hr * hd / 16, false);
  const bool fast_d = ternary_fast_shape(D->fr, D->fr / 128, D->fr / 16, false);
  const bool fast_h = ternary_fast_shape(H, H / 128, H / 16, false);
  int rc;
  cudaError_t e;
  // Every kernel of the step is launched with programmatic stream
  // serialization and waits for its predecessor before reading anything, so
  // each one's launch overlaps the tail of the one before.
  const AttnGeom geom = attn_geom(B, D->hr * hd, D->hr, D->kvr, c.max_seq,
                                  (uint64_t)c.max_batch * c.max_seq * D->kvr * hd);
  if (D->step_ok && B <= kStepMaxB) {
    // All layers in one persistent kernel; the LM head and the next token follow.
    StepArgs a = {};
    a.layers = D->step_layers;
    a.L = c.layers;
    a.B = B;
    a.H = H;
    a.hd = hd;
    a.hr = D->hr;
    a.kvr = D->kvr;
    a.fr = D->fr;
    a.maxseq = c.max_seq;
    a.max_batch = c.max_batch;
    a.qkv_rows = D->qkv_rows;
    a.eps = eps;
    a.coef = geom.coef;
    a.nsplit = geom.nsplit;
    a.chunk = geom.chunk;
    a.dch = step_down_chunks(D->fr);
    a.embed = D->embed;
    a.gfinal = D->gfinal;
    a.rope = D->rope;
    a.hbuf = D->step_h;
    a.qkv = D->qkv;
    a.ctx = D->ctx;
    a.o = D->o;
    a.a = D->a;
    a.x_final = D->x;
    a.apart = (float *)D->attn_scr;
    a.acnt = D->step_acnt;
    a.amax = D->step_amax;
    a.dpart = D->step_dpart;
    a.tok = D->tok;
    a.pos = D->pos;
    a.bar = D->step_bar;
    a.sep = D->step_bar + 1;
    a.err = D->err;
    e = step_launch(a, st);
    count_launches(1);
    if (e != cudaSuccess) return cuda_status(e, "step: layers");
  } else {
    e = cta_rows ? launch_pdl(k_norm_cta<kNormGather>, dim3(B), dim3(norm_threads), (size_t)H * 4,
                              st, (const int *)D->tok, (const float *)D->embed, D->h,
                              (const float *)nullptr, (const float *)D->layers[0].gattn, D->x,
                              fast_h ? D->ws_qkv : nullptr, B, H, eps, PeerIn{})
                 : launch_pdl(k_norm<kNormGather>, dim3(gnorm), dim3(kNormThreads), smem_h, st,
                              (const int *)D->tok, (const float *)D->embed, D->h,
                              (const float *)nullptr, (const float *)D->layers[0].gattn, D->x,
                              fast_h ? D->ws_qkv : nullptr, B, H, eps, PeerIn{});
    count_launches(1);
    if (e != cudaSuccess) return cuda_status(e, "step: embed");
    // Tensor parallelism: O / down partials go peer to peer (D->par), or
    // through NCCL all-reduces.
    PeerOut po[2] = {};
    PeerIn pin[2] = {};
    if (D->par) {
      for (int set = 0; set < 2; set++) {
        for (int r = 0; r < D->size; r++) po[set].dst[r] = par_slot(D, D->par_peer[r], set, D->rank);
        po[set].n = D->size;
        po[set].ep = D->ep;
        po[set].tmul = c.layers;
        pin[set].slots = par_slot(D, D->par_local, set, 0);
        pin[set].tp = (uint32_t)D->size;
        pin[set].slot_stride = c.max_batch * H;
        pin[set].ep = D->ep;
        pin[set].tmul = c.layers;
        pin[set].err = D->err;
      }
    }
    for (uint32_t l = 0; l < c.layers; l++) {
      Layer &L = D->layers[l];
      e = ternary_main_launch(1, D->x, 0, L.wqkv, 0, L.sqkv, 0, nullptr, D->qkv, 0, B, D->qkv_rows,
                              H, false, fast_h ? D->ws_qkv : nullptr, st);
      if (e != cudaSuccess) return cuda_status(e, "step: qkv");
      // RoPE of q and k, the cache append of k and v, and the split-K
      // attention over positions 0..pos in one kernel; then the split merge,
      // whose last CTA per sequence row quantizes the row for the O GEMV.
      e = attn_rope_decode_launch(D->qkv, L.ck, L.cv, D->pos, D->ctx, geom, D->rope,
                                  D->attn_scr, st, fast_o ? D->ws_o : nullptr,
                                  fast_o ? D->attn_ctr : nullptr);
      if (e != cudaSuccess) return cuda_status(e, "step: attention");
      po[0].tadd = po[1].tadd = pin[0].tadd = pin[1].tadd = l + 1;
      e = ternary_main_launch(1, D->ctx, 0, L.wo, 0, L.so, 0, nullptr, D->o, 0, B, H, D->hr * hd,
                              false, fast_o ? D->ws_o : nullptr, st, D->par ? &po[0] : nullptr);
      if (e != cudaSuccess) return cuda_status(e, "step: o");
      if (!D->par && (rc = allreduce(D, D->o, (size_t)B * H, kNcclFloat32, kNcclSum))) return rc;
      // tag of this layer's use: ep * layers + l + 1 (never 0: the slots start zeroed)
      e = cta_rows
              ? launch_pdl(k_norm_cta<kNormAdd>, dim3(B), dim3(norm_threads), (size_t)H * 4, st,
                           (const int *)nullptr, (const float *)nullptr, D->h, (const float *)D->o,
                           (const float *)L.gffn, D->x, fast_h ? D->ws_gu : nullptr, B, H, eps,
                           pin[0])
              : launch_pdl(k_norm<kNormAdd>, dim3(gnorm), dim3(kNormThreads), smem_h, st,
                           (const int *)nullptr, (const float *)nullptr, D->h, (const float *)D->o,
                           (const float *)L.gffn, D->x, fast_h ? D->ws_gu : nullptr, B, H, eps,
                           pin[0]);
      count_launches(1);
      if (e != cudaSuccess) return cuda_status(e, "step: ffn norm");
      e = ternary_main_launch(1, D->x, 0, L.wgu, 0, L.sgu, 0, nullptr, D->gu, 0, B, 2 * D->fr, H,
                              false, fast_h ? D->ws_gu : nullptr, st);
      if (e != cudaSuccess) return cuda_status(e, "step: gate/up");
      if (silu_row4 == 1)
        e = launch_pdl(k_silu_cta<1>, dim3(B), dim3(silu_threads), (size_t)D->fr * 4, st,
                       (const float *)D->gu, D->a, fast_d ? D->ws_d : nullptr, B, D->fr);
      else if (silu_row4 == 2)
        e = launch_pdl(k_silu_cta<2>, dim3(B), dim3(silu_threads), (size_t)D->fr * 4, st,
                       (const float *)D->gu, D->a, fast_d ? D->ws_d : nullptr, B, D->fr);
      else
        e = launch_pdl(k_silu_prep, dim3(gnorm), dim3(kNormThreads),
                       (size_t)row_slice_cols(D->fr) * sizeof(float), st, (const float *)D->gu,
                       D->a, fast_d ? D->ws_d : nullptr, B, D->fr);
      count_launches(1);
      if (e != cudaSuccess) return cuda_status(e, "step: swiglu");
      e = ternary_main_launch(1, D->a, 0, L.wd, 0, L.sd, 0, nullptr, D->d, 0, B, H, D->fr, false,
                              fast_d ? D->ws_d : nullptr, st, D->par ? &po[1] : nullptr);
      if (e != cudaSuccess) return cuda_status(e, "step: down");
      if (!D->par && (rc = allreduce(D, D->d, (size_t)B * H, kNcclFloat32, kNcclSum))) return rc;
      const bool last = l + 1 == c.layers;
      const float *gn = last ? D->gfinal : D->layers[l + 1].gattn;
      void *wsn = (!last && fast_h) ? D->ws_qkv : nullptr;
      e = cta_rows
              ? launch_pdl(k_norm_cta<kNormAdd>, dim3(B), dim3(norm_threads), (size_t)H * 4, st,
                           (const int *)nullptr, (const float *)nullptr, D->h, (const float *)D->d,
                           gn, D->x, wsn, B, H, eps, pin[1])
              : launch_pdl(k_norm<kNormAdd>, dim3(gnorm), dim3(kNormThreads), smem_h, st,
                           (const int *)nullptr, (const float *)nullptr, D->h, (const float *)D->d,
                           gn, D->x, wsn, B, H, eps, pin[1]);
      count_launches(1);
      if (e != cudaSuccess) return cuda_status(e, "step: attn norm");
    }
  }
  const size_t smem_lm = (size_t)(B <= 1 ? 1 : (B <= 2 ? 2 : (B <= 4 ? 4 : (B <= 8 ? 8 : 16)))) *
                         H * sizeof(float);
  const unsigned lmgrid = 148 * 4;
  const float *E = D->embed + (size_t)D->v0 * H;
  float *lg = D->keep_logits ? D->logits : nullptr;
  const uint32_t lstride = c.max_batch * D->vr;
  unsigned long long *keys = D->par ? par_keys(D->par_local) : D->keys;
  PeerSig sig = {};
  PeerKeys pk = {};
  if (D->par) {
    for (int r = 0; r < D->size; r++) {
      sig.ctr[r] = par_ctr(D->par_peer[r], 2);
      pk.keys[r] = par_keys(D->par_peer[r]);
    }
    sig.done = par_done(D->par_local, 2);
    sig.n = pk.n = D->size;
    pk.stride = c.max_batch;
    pk.ctr = par_ctr(D->par_local, 2);
    pk.err = D->err;
  }
#define NL_LM(NB)                                                                         \
  e = launch_pdl(k_lmhead<NB>, dim3(lmgrid), dim3(256), smem_lm, st, E, (const float *)D->x, \
                 keys, lg, (const int *)D->pos, B, D->vr, D->v0, H, lstride,              \
                 (const unsigned long long *)D->ep, c.max_batch, sig)
#define NL_LMR(NB)                                                                        \
  e = launch_pdl(k_lmhead_ring<NB>, dim3(148), dim3(kLmWarps * 32), lmhead_ring_smem(NB, H), \
                 st, E, (const float *)D->x, keys, lg, (const int *)D->pos, B, D->vr, D->v0, \
                 H, lstride, (const unsigned long long *)D->ep, c.max_batch, sig)
  const bool ring = H % 128u == 0 && lmhead_ring_smem(8, H) <= (size_t)(227u << 10);
  if (B <= 1) NL_LM(1);
  else if (B <= 2 && ring) NL_LMR(2);
  else if (B <= 2) NL_LM(2);
  else if (B <= 4 && ring) NL_LMR(4);
  else if (B <= 4) NL_LM(4);
  else if (B <= 8 && ring) NL_LMR(8);
  else if (B <= 8) NL_LM(8);
  else NL_LM(16);
#undef NL_LMR
#undef NL_LM
  count_launches(1);
  if (e != cudaSuccess) return cuda_status(e, "step: lm head");
  if (!D->par && (rc = allreduce(D, D->keys, B, kNcclUint64, kNcclMax))) return rc;
  e = launch_pdl(k_next, dim3(1), dim3(32), 0, st, keys, (const int *)D->prompt,
                 D->last_positions, D->tok, D->out_tok, D->pos, D->posf, B, D->ep, pk);
  count_launches(1);
  return cuda_status(e, "step: next");
}

int set_smem_limits(nl_decoder *D) {
  const size_t lm = (size_t)16 * D->cfg.hidden * sizeof(float);
  cudaError_t e;
  if ((e = cudaFuncSetAttribute(k_lmhead<16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)lm)) != cudaSuccess ||
      (e = cudaFuncSetAttribute(k_lmhead<8>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)(lm / 2))) != cudaSuccess ||
      (e = cudaFuncSetAttribute(k_lmhead<4>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)(lm / 4))) != cudaSuccess)
    return cuda_status(e, "decoder: lm head smem");
  if (D->cfg.hidden % 128u == 0 && lmhead_ring_smem(8, D->cfg.hidden) <= (size_t)(227u << 10) &&
      ((e = cudaFuncSetAttribute(k_lmhead_ring<8>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)lmhead_ring_smem(8, D->cfg.hidden))) != cudaSuccess ||
       (e = cudaFuncSetAttribute(k_lmhead_ring<4>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)lmhead_ring_smem(4, D->cfg.hidden))) != cudaSuccess ||
       (e = cudaFuncSetAttribute(k_lmhead_ring<2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)lmhead_ring_smem(2, D->cfg.hidden))) != cudaSuccess))
    return cuda_status(e, "decoder: lm head ring smem");
  const size_t hs = (size_t)row_slice_cols(D->cfg.hidden) * sizeof(float),
               fs = (size_t)row_slice_cols(D->fr) * sizeof(float);
  if ((e = cudaFuncSetAttribute(k_norm<kNormGather>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)hs)) != cudaSuccess ||
      (e = cudaFuncSetAttribute(k_norm<kNormAdd>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)hs)) != cudaSuccess ||
      (e = cudaFuncSetAttribute(k_silu_prep, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)fs)) != cudaSuccess)
    return cuda_status(e, "decoder: smem");
  const int hrow = (int)(D->cfg.hidden * 4u), frow = (int)(D->fr * 4u);
  if ((e = cudaFuncSetAttribute(k_norm_cta<kNormGather>,
                                cudaFuncAttributeMaxDynamicSharedMemorySize, hrow)) != cudaSuccess ||
      (e = cudaFuncSetAttribute(k_norm_cta<kNormAdd>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                hrow)) != cudaSuccess ||
      (e = cudaFuncSetAttribute(k_silu_cta<1>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                frow)) != cudaSuccess ||
      (e = cudaFuncSetAttribute(k_silu_cta<2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                frow)) != cudaSuccess)
    return cuda_status(e, "decoder: smem");
  return NL_OK;
}

}  // namespace
}  // namespace nl

using namespace nl;

extern "C" int nl_nccl_unique_id(void *id_out) {
  Nccl *n = nccl();
  if (!n) return set_error(NL_ERROR, "libnccl.so.2 not available");
  ncclUniqueId id;
  ncclResult_t r = n->GetUniqueId(&id);
  if (r != 0) return set_error(NL_ERROR, "ncclGetUniqueId failed (%d)", r);
  memcpy(id_out, &id, sizeof(id));
  return NL_OK;
}

extern "C" void nl_decoder_destroy(nl_decoder *D) {
  if (!D) return;
  if (D->stream) cudaStreamSynchronize(D->stream);
  for (auto &kv : D->graphs) cudaGraphExecDestroy(kv.second);
  D->graphs.clear();
  if (D->par) {
    // Peers may still read this rank's keys: free only after every rank has
    // finished its generation (an NCCL all-reduce as the barrier).
    Nccl *n = nccl();
    if (n && D->comm && D->ep &&
        n->AllReduce(D->ep, D->ep, 1, kNcclUint64, kNcclMax, D->comm, D->stream) == 0)
      cudaStreamSynchronize(D->stream);
    for (int q = 0; q < D->size; q++)
      if (q != D->rank && D->par_peer[q]) cudaIpcCloseMemHandle(D->par_peer[q]);
    if (D->par_local) cudaFree(D->par_local);
  }
  if (D->comm && nccl()) nccl()->CommDestroy(D->comm);
  for (void *p : D->allocs) cudaFree(p);
  for (void *p : D->pf_allocs) cudaFree(p);
  if (D->stream) cudaStreamDestroy(D->stream);
  delete D;
}

// The device address of resident buffer HANDLE, which must hold WORDS words.
static int weight_ptr(uint32_t handle, uint64_t words, const char *what, const uint32_t **p) {
  void *ptr = nullptr;
  uint32_t n = 0;
  if (nl_resident_info(handle, &ptr, &n) != NL_OK || !ptr)
    return set_error(NL_ERROR, "decoder weights: %s: handle %u is not resident", what, handle);
  if ((uint64_t)n != words)
    return set_error(NL_ERROR, "decoder weights: %s: handle %u holds %u words, the shape needs %llu",
                     what, handle, n, (unsigned long long)words);
  *p = static_cast<const uint32_t *>(ptr);
  return NL_OK;
}
// ROWS rows of WNG words each (row pitch PITCH words, starting at word W0 of
// row R0) of resident HANDLE, whose full shape is FULL_ROWS x PITCH, into DST.
static int copy_block(nl_decoder *D, void *dst, uint32_t handle, uint64_t full_rows,
                      uint64_t pitch, uint64_t r0, uint64_t rows, uint64_t w0, uint64_t wng,
                      const char *what) {
  const uint32_t *p = nullptr;
  int rc = weight_ptr(handle, full_rows * pitch, what, &p);
  if (rc) return rc;
  return cuda_status(cudaMemcpy2DAsync(dst, wng * 4, p + r0 * pitch + w0, pitch * 4, wng * 4,
                                       rows, cudaMemcpyDeviceToDevice, D->stream),
                     "decoder weights: copy");
}

static int decoder_build(nl_decoder *D) {
  const nl_decoder_config &c = D->cfg;
  const uint32_t H = c.hidden, hd = c.head_dim;
  const uint32_t grp = c.heads / c.kv_heads;
  Shard sh;
  if (int rc = plan_shard(c, D->rank, D->size, &sh)) return rc;
  D->kvh = sh.kvh;
  D->ffb = sh.ffb;
  D->voc = sh.voc;
  D->kvr = D->kvh.count;
  D->hr = D->kvr * grp;
  D->fr = D->ffb.count * 128;
  D->vr = D->voc.count;
  D->v0 = D->voc.begin;
  D->qkv_rows = (D->hr + 2 * D->kvr) * hd;
  cudaError_t e = cudaStreamCreateWithFlags(&D->stream, cudaStreamNonBlocking);
  if (e != cudaSuccess) return cuda_status(e, "decoder: stream");
  const uint32_t h0 = D->kvh.begin * grp, kv0 = D->kvh.begin, f0 = D->ffb.begin * 128;
  const uint32_t qd = c.heads * hd, kvd = c.kv_heads * hd;
  uint64_t wb = 0;
  D->layers.resize(c.layers);
  for (uint32_t l = 0; l < c.layers; l++) {
    Layer &L = D->layers[l];
    const uint64_t T = (uint64_t)l * 16;
    const size_t wq = (size_t)D->qkv_rows * (H / 16), wo = (size_t)H * (D->hr * hd / 16);
    const size_t wgu = (size_t)2 * D->fr * (H / 16), wdn = (size_t)H * (D->fr / 16);
    DALLOC(L.wqkv, wq * 4);
    DALLOC(L.wo, wo * 4);
    DALLOC(L.wgu, wgu * 4);
    DALLOC(L.wd, wdn * 4);
    DALLOC(L.sqkv, (size_t)D->qkv_rows * 4);
    DALLOC(L.so, (size_t)H * 4);
    DALLOC(L.sgu, (size_t)2 * D->fr * 4);
    DALLOC(L.sd, (size_t)H * 4);
    DALLOC(L.gattn, (size_t)H * 4);
    DALLOC(L.gffn, (size_t)H * 4);
    const size_t cache = (size_t)c.max_batch * c.max_seq * D->kvr * hd * 4;
    DALLOC(L.ck, cache);
    DALLOC(L.cv, cache);
    wb += (wq + wo + wgu + wdn) * 4 + ((size_t)D->qkv_rows + 2 * H + 2 * D->fr) * 4 + 2 * H * 4;
    const uint32_t rq = D->hr * hd, rk = D->kvr * hd;
    int rc;
    if (const nl_decoder_weights *w = D->src) {
      // this rank's shard out of the caller's full tensors
      const uint64_t hw = H / 16, qw = (uint64_t)qd / 16, fw = c.ffn / 16;
      if ((rc = copy_block(D, L.wqkv, w->wq[l], qd, hw, (uint64_t)h0 * hd, rq, 0, hw, "wq")) ||
          (rc = copy_block(D, L.wqkv + (size_t)rq * hw, w->wk[l], kvd, hw, (uint64_t)kv0 * hd,
                           rk, 0, hw, "wk")) ||
          (rc = copy_block(D, L.wqkv + (size_t)(rq + rk) * hw, w->wv[l], kvd, hw,
                           (uint64_t)kv0 * hd, rk, 0, hw, "wv")) ||
          (rc = copy_block(D, L.sqkv, w->sq[l], qd, 1, (uint64_t)h0 * hd, rq, 0, 1, "sq")) ||
          (rc = copy_block(D, L.sqkv + rq, w->sk[l], kvd, 1, (uint64_t)kv0 * hd, rk, 0, 1,
                           "sk")) ||
          (rc = copy_block(D, L.sqkv + rq + rk, w->sv[l], kvd, 1, (uint64_t)kv0 * hd, rk, 0, 1,
                           "sv")) ||
          (rc = copy_block(D, L.wo, w->wo[l], H, qw, 0, H, (uint64_t)h0 * hd / 16, rq / 16,
                           "wo")) ||
          (rc = copy_block(D, L.so, w->so[l], H, 1, 0, H, 0, 1, "so")) ||
          (rc = copy_block(D, L.wgu, w->wgate[l], c.ffn, hw, f0, D->fr, 0, hw, "wgate")) ||
          (rc = copy_block(D, L.wgu + (size_t)D->fr * hw, w->wup[l], c.ffn, hw, f0, D->fr, 0, hw,
                           "wup")) ||
          (rc = copy_block(D, L.sgu, w->sgate[l], c.ffn, 1, f0, D->fr, 0, 1, "sgate")) ||
          (rc = copy_block(D, L.sgu + D->fr, w->sup[l], c.ffn, 1, f0, D->fr, 0, 1, "sup")) ||
          (rc = copy_block(D, L.wd, w->wdown[l], H, fw, 0, H, f0 / 16, D->fr / 16, "wdown")) ||
          (rc = copy_block(D, L.sd, w->sdown[l], H, 1, 0, H, 0, 1, "sdown")) ||
          (rc = copy_block(D, L.gattn, w->attn_norm[l], H, 1, 0, H, 0, 1, "attn_norm")) ||
          (rc = copy_block(D, L.gffn, w->ffn_norm[l], H, 1, 0, H, 0, 1, "ffn_norm")))
        return rc;
      wb += (wq + wo + wgu + wdn) * 4 + ((size_t)D->qkv_rows + 2 * H + 2 * D->fr) * 4 + 2 * H * 4;
      continue;
    }
    if ((rc = gen_ternary(D, L.wqkv, rq, H, T + NL_T_WQ, (uint64_t)h0 * hd, H, 0)) ||
        (rc = gen_ternary(D, L.wqkv + (size_t)rq * (H / 16), rk, H, T + NL_T_WK,
                          (uint64_t)kv0 * hd, H, 0)) ||
        (rc = gen_ternary(D, L.wqkv + (size_t)(rq + rk) * (H / 16), rk, H, T + NL_T_WV,
                          (uint64_t)kv0 * hd, H, 0)) ||
        (rc = gen_scale(D, L.sqkv, rq, T + NL_T_SQ, (uint64_t)h0 * hd, H)) ||
        (rc = gen_scale(D, L.sqkv + rq, rk, T + NL_T_SK, (uint64_t)kv0 * hd, H)) ||
        (rc = gen_scale(D, L.sqkv + rq + rk, rk, T + NL_T_SV, (uint64_t)kv0 * hd, H)) ||
        (rc = gen_ternary(D, L.wo, H, rq, T + NL_T_WO, 0, qd, (uint64_t)h0 * hd)) ||
        (rc = gen_scale(D, L.so, H, T + NL_T_SO, 0, qd)) ||
        (rc = gen_ternary(D, L.wgu, D->fr, H, T + NL_T_WGATE, f0, H, 0)) ||
        (rc = gen_ternary(D, L.wgu + (size_t)D->fr * (H / 16), D->fr, H, T + NL_T_WUP, f0, H, 0)) ||
        (rc = gen_scale(D, L.sgu, D->fr, T + NL_T_SGATE, f0, H)) ||
        (rc = gen_scale(D, L.sgu + D->fr, D->fr, T + NL_T_SUP, f0, H)) ||
        (rc = gen_ternary(D, L.wd, H, D->fr, T + NL_T_WDOWN, 0, c.ffn, f0)) ||
        (rc = gen_scale(D, L.sd, H, T + NL_T_SDOWN, 0, c.ffn)) ||
        (rc = gen_norm(D, L.gattn, H, T + NL_T_ATTN_NORM)) ||
        (rc = gen_norm(D, L.gffn, H, T + NL_T_FFN_NORM)))
      return rc;
    (void)kvd;
  }
  const size_t en = (size_t)c.vocab * H;
  DALLOC(D->embed, en * 4);
  DALLOC(D->gfinal, (size_t)H * 4);
  int rc;
  if (const nl_decoder_weights *w = D->src) {
    if ((rc = copy_block(D, D->embed, w->embed, c.vocab, H, 0, c.vocab, 0, H, "embed")) ||
        (rc = copy_block(D, D->gfinal, w->final_norm, H, 1, 0, H, 0, 1, "final_norm")))
      return rc;
  } else {
    gen_embed_kernel<<<grid_for(en, 256), 256, 0, D->stream>>>(
        D->embed, en, nl_tensor_key(c.seed, NL_T_EMBED));
    if ((rc = cuda_status(cudaPeekAtLastError(), "decoder: embedding"))) return rc;
    if ((rc = gen_norm(D, D->gfinal, H, NL_T_FINAL_NORM))) return rc;
  }
  wb += (size_t)D->vr * H * 4 + (size_t)H * 4;
  D->weight_bytes = wb;
  const uint32_t B = c.max_batch;
  DALLOC(D->h, (size_t)B * H * 4);
  DALLOC(D->x, (size_t)B * H * 4);
  DALLOC(D->qkv, (size_t)B * D->qkv_rows * 4);
  DALLOC(D->ctx, (size_t)B * D->hr * hd * 4);
  DALLOC(D->o, (size_t)B * H * 4);
  DALLOC(D->gu, (size_t)B * 2 * D->fr * 4);
  DALLOC(D->a, (size_t)B * D->fr * 4);
  DALLOC(D->d, (size_t)B * H * 4);
  DALLOC(D->posf, 16);
  DALLOC(D->rope, (size_t)c.max_seq * (hd / 2) * sizeof(float2));
  if ((e = rope_table_launch(D->rope, c.max_seq, hd, c.rope_base, D->stream)) != cudaSuccess)
    return cuda_status(e, "decoder: rope table");
  DALLOC(D->pos, 16);
  DALLOC(D->tok, (size_t)B * 4);
  DALLOC(D->keys, (size_t)B * 8);
  DALLOC(D->ep, 8);
  DALLOC(D->err, 4);
  DALLOC(D->attn_ctr, (size_t)B * 4);
  if ((e = cudaMemsetAsync(D->ep, 0, 8, D->stream)) != cudaSuccess ||
      (e = cudaMemsetAsync(D->err, 0, 4, D->stream)) != cudaSuccess ||
      (e = cudaMemsetAsync(D->attn_ctr, 0, (size_t)B * 4, D->stream)) != cudaSuccess)
    return cuda_status(e, "decoder: counters");
  DALLOC(D->prompt, (size_t)B * c.max_seq * 4);
  DALLOC(D->out_tok, (size_t)B * c.max_seq * 4);
  DALLOC(D->ws_qkv, ternary_ws_bytes(1, B, H));
  DALLOC(D->ws_gu, ternary_ws_bytes(1, B, H));
  DALLOC(D->ws_o, ternary_ws_bytes(1, B, D->hr * hd));
  DALLOC(D->ws_d, ternary_ws_bytes(1, B, D->fr));
  size_t scr = 0;   // the split count grows as the batch shrinks: size for every batch
  for (uint32_t bb = 1; bb <= B; bb++) {
    const AttnGeom g = attn_geom(bb, D->hr * hd, D->hr, D->kvr, c.max_seq,
                                 (uint64_t)B * c.max_seq * D->kvr * hd);
    if (attn_rope_scratch_bytes(g) > scr) scr = attn_rope_scratch_bytes(g);
  }
  DALLOC(D->attn_scr, scr + 256);
  // The one-kernel step (TP = 1, batch <= 8, the head sizes and widths it covers).
  D->step_ok = step_supported(1, H, hd, D->hr, D->kvr, D->fr, D->size);
  if (D->step_ok) {
    std::vector<StepLayer> sl(c.layers);
    for (uint32_t l = 0; l < c.layers; l++) {
      const Layer &L = D->layers[l];
      sl[l] = StepLayer{L.wqkv, L.wo, L.wgu, L.wd, L.sqkv, L.so, L.sgu, L.sd, L.gattn, L.gffn,
                        L.ck, L.cv};
    }
    const uint32_t SB = B < kStepMaxB ? B : kStepMaxB;
    DALLOC(D->step_layers, sizeof(StepLayer) * c.layers);
    DALLOC(D->step_h, (size_t)2 * SB * H * 4);
    DALLOC(D->step_acnt, (size_t)SB * D->kvr * 4);
    DALLOC(D->step_amax, (size_t)SB * 4);
    DALLOC(D->step_dpart, step_dpart_bytes(SB, H, D->fr));
    DALLOC(D->step_bar, 16);
    if ((e = cudaMemcpyAsync(D->step_layers, sl.data(), sizeof(StepLayer) * c.layers,
                             cudaMemcpyHostToDevice, D->stream)) != cudaSuccess ||
        (e = cudaMemsetAsync(D->step_acnt, 0, (size_t)SB * D->kvr * 4, D->stream)) !=
            cudaSuccess ||
        (e = cudaMemsetAsync(D->step_bar, 0, 16, D->stream)) != cudaSuccess)
      return cuda_status(e, "decoder: step buffers");
    if ((e = cudaStreamSynchronize(D->stream)) != cudaSuccess)
      return cuda_status(e, "decoder: step buffers");
  }
  if (D->keep_logits) DALLOC(D->logits, (size_t)c.max_seq * B * D->vr * 4);
  if ((rc = set_smem_limits(D))) return rc;
  return cuda_status(cudaStreamSynchronize(D->stream), "decoder: build");
}

// Map every rank's peer block into this process (CUDA IPC handles exchanged
// with an NCCL all-gather) and agree, with an NCCL min-reduction, on whether
// every rank managed it; otherwise every rank keeps the NCCL all-reduces.
// NELISP_DECODER_ALLREDUCE=nccl keeps them too.
static int setup_peer_allreduce(nl_decoder *D) {
  Nccl *n = nccl();
  if (D->size <= 1 || D->size > 8 || !n || !n->AllGather) return NL_OK;
  const char *v = getenv("NELISP_DECODER_ALLREDUCE");
  const bool want = !(v && strcmp(v, "nccl") == 0);   // same on every rank
  if (!want) return NL_OK;
  cudaStream_t st = D->stream;
  int ok = 1;
  const size_t bytes = par_bytes(D);
  if (cudaMalloc(&D->par_local, bytes) != cudaSuccess) { D->par_local = nullptr; ok = 0; }
  cudaGetLastError();
  if (ok && cudaMemset(D->par_local, 0, bytes) != cudaSuccess) ok = 0;
  // What each rank publishes: its block's IPC handle and its device's UUID
  // (ranks that wait on one another must not share a GPU).
  struct Pub {
    cudaIpcMemHandle_t h;
    char uuid[16];
    char pad[16];
  };
  Pub mine;
  memset(&mine, 0, sizeof(mine));
  if (ok && cudaIpcGetMemHandle(&mine.h, D->par_local) != cudaSuccess) ok = 0;
  cudaGetLastError();
  {
    int devn = 0;
    cudaDeviceProp prop;
    if (cudaGetDevice(&devn) == cudaSuccess && cudaGetDeviceProperties(&prop, devn) == cudaSuccess)
      memcpy(mine.uuid, &prop.uuid, 16);
    else
      ok = 0;
    cudaGetLastError();
  }
  char *dev = nullptr;
  int *flag = nullptr;
  if (cudaMalloc(&dev, (size_t)D->size * sizeof(Pub)) != cudaSuccess ||
      cudaMalloc(&flag, sizeof(int)) != cudaSuccess) {
    if (dev) cudaFree(dev);
    return set_error(NL_ERROR, "decoder: peer setup buffers");
  }
  std::vector<Pub> all(D->size);
  ncclResult_t r = 0;
  cudaError_t e = cudaMemcpy(dev + (size_t)D->rank * sizeof(Pub), &mine, sizeof(Pub),
                             cudaMemcpyHostToDevice);
  if (e == cudaSuccess)
    r = n->AllGather(dev + (size_t)D->rank * sizeof(Pub), dev, sizeof(Pub), kNcclInt8, D->comm,
                     st);
  if (e == cudaSuccess && r == 0) e = cudaStreamSynchronize(st);
  if (e == cudaSuccess && r == 0)
    e = cudaMemcpy(all.data(), dev, (size_t)D->size * sizeof(Pub), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess || r != 0) {
    cudaFree(dev);
    cudaFree(flag);
    return set_error(NL_ERROR, "decoder: peer handle exchange failed");
  }
  for (int a = 0; a < D->size; a++)
    for (int b = a + 1; b < D->size; b++)
      if (memcmp(all[a].uuid, all[b].uuid, 16) == 0) ok = 0;   // two ranks on one GPU
  for (int q = 0; q < D->size && ok; q++) {
    if (q == D->rank) {
      D->par_peer[q] = D->par_local;
      continue;
    }
    void *ptr = nullptr;
    if (cudaIpcOpenMemHandle(&ptr, all[q].h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
      cudaGetLastError();
      ok = 0;
      break;
    }
    D->par_peer[q] = static_cast<char *>(ptr);
  }
  // every rank takes the same path
  cudaMemcpy(flag, &ok, sizeof(int), cudaMemcpyHostToDevice);
  r = n->AllReduce(flag, flag, 1, kNcclInt32, kNcclMin, D->comm, st);
  int agreed = 0;
  if (r == 0 && cudaStreamSynchronize(st) == cudaSuccess)
    cudaMemcpy(&agreed, flag, sizeof(int), cudaMemcpyDeviceToHost);
  cudaFree(dev);
  cudaFree(flag);
  if (!agreed) {
    for (int q = 0; q < D->size; q++)
      if (q != D->rank && D->par_peer[q]) cudaIpcCloseMemHandle(D->par_peer[q]);
    for (int q = 0; q < 8; q++) D->par_peer[q] = nullptr;
    if (D->par_local) cudaFree(D->par_local);
    D->par_local = nullptr;
    cudaGetLastError();
    return r == 0 ? NL_OK : set_error(NL_ERROR, "decoder: peer setup agreement failed");
  }
  D->par = true;
  return NL_OK;
}

static int decoder_create(const nl_decoder_config *cfg, const nl_decoder_weights *w, int tp_rank,
                          int tp_size, const void *nccl_id, int keep_logits, nl_decoder **out);

extern "C" int nl_decoder_create(const nl_decoder_config *cfg, int tp_rank, int tp_size,
                                 const void *nccl_id, int keep_logits, nl_decoder **out) {
  return decoder_create(cfg, nullptr, tp_rank, tp_size, nccl_id, keep_logits, out);
}

extern "C" int nl_decoder_create_from_weights(const nl_decoder_config *cfg,
                                              const nl_decoder_weights *w, int tp_rank,
                                              int tp_size, const void *nccl_id, int keep_logits,
                                              nl_decoder **out) {
  if (out) *out = nullptr;
  if (!w) return set_error(NL_ERROR, "decoder: no weights");
  return decoder_create(cfg, w, tp_rank, tp_size, nccl_id, keep_logits, out);
}

static int decoder_create(const nl_decoder_config *cfg, const nl_decoder_weights *w, int tp_rank,
                          int tp_size, const void *nccl_id, int keep_logits, nl_decoder **out) {
  *out = nullptr;
  int rc = nl_init(-1);
  if (rc) return rc;
  const nl_decoder_config &c = *cfg;
  if ((rc = check_config(c))) return rc;
  Shard sh;                      // refuses a rank left without heads, FFN blocks or vocab
  if ((rc = plan_shard(c, tp_rank, tp_size, &sh))) return rc;
  nl_decoder *D = new nl_decoder();
  D->cfg = c;
  D->rank = tp_rank;
  D->size = tp_size;
  D->keep_logits = keep_logits != 0;
  D->src = w;
  if (tp_size > 1) {
    Nccl *n = nccl();
    if (!n) { delete D; return set_error(NL_ERROR, "libnccl.so.2 not available"); }
    ncclUniqueId id;
    memcpy(&id, nccl_id, sizeof(id));
    ncclResult_t r = n->CommInitRank(&D->comm, tp_size, id, tp_rank);
    if (r != 0) {
      delete D;
      return set_error(NL_ERROR, "ncclCommInitRank: %s", n->GetErrorString ? n->GetErrorString(r) : "?");
    }
  }
  if ((rc = decoder_build(D)) || (rc = setup_peer_allreduce(D))) {
    nl_decoder_destroy(D);
    return rc;
  }
  D->src = nullptr;   // the caller's handles are not needed after the copies
  *out = D;
  return NL_OK;
}

// Buffers for a batched prefill of ROWS rows (reallocated when larger).
static int prefill_buffers(nl_decoder *D, uint32_t rows) {
  if (rows <= D->pf_cap) return NL_OK;
  cudaStreamSynchronize(D->stream);
  for (void *p : D->pf_allocs) cudaFree(p);
  D->pf_allocs.clear();
  D->pf_cap = 0;
  const nl_decoder_config &c = D->cfg;
  const size_t R = rows, H = c.hidden, hq = (size_t)D->hr * c.head_dim;
  size_t ws = ternary_ws_bytes_best(1, rows, c.hidden, false);
  if (ternary_ws_bytes_best(1, rows, (uint32_t)hq, false) > ws)
    ws = ternary_ws_bytes_best(1, rows, (uint32_t)hq, false);
  if (ternary_ws_bytes_best(1, rows, D->fr, false) > ws)
    ws = ternary_ws_bytes_best(1, rows, D->fr, false);
  struct {
    void **p;
    size_t bytes;
  } want[] = {{(void **)&D->pf_tok, R * 4},          {(void **)&D->pf_h, R * H * 4},
              {(void **)&D->pf_x, R * H * 4},          {(void **)&D->pf_qkv, R * D->qkv_rows * 4},
              {(void **)&D->pf_q, R * hq * 4},         {(void **)&D->pf_ctx, R * hq * 4},
              {(void **)&D->pf_o, R * H * 4},          {(void **)&D->pf_gu, R * 2 * D->fr * 4},
              {(void **)&D->pf_a, R * D->fr * 4},      {(void **)&D->pf_d, R * H * 4},
              {&D->pf_ws, ws}};
  for (auto &w : want) {
    cudaError_t e = cudaMalloc(w.p, w.bytes ? w.bytes : 16);
    if (e != cudaSuccess) {
      for (void *p : D->pf_allocs) cudaFree(p);
      D->pf_allocs.clear();
      return cuda_status(e, "prefill: cudaMalloc");
    }
    D->pf_allocs.push_back(*w.p);
  }
  D->pf_ws_bytes = ws;
  D->pf_cap = rows;
  return NL_OK;
}

// Positions 0 .. P-2 of BATCH sequences in one pass per layer (see k_pf_tokens).
static int run_prefill(nl_decoder *D, uint32_t B, uint32_t P) {
  const nl_decoder_config &c = D->cfg;
  const uint32_t n = P - 1, rows = B * n, H = c.hidden, hd = c.head_dim, hq = D->hr * hd;
  const float eps = c.rms_eps;
  cudaStream_t st = D->stream;
  int rc;
  if ((rc = prefill_buffers(D, rows))) return rc;
  cudaError_t e;
  k_pf_tokens<<<grid_for(rows, 256), 256, 0, st>>>(D->prompt, P, n, B, D->pf_tok);
  const dim3 gnorm(rows * kRowCluster);
  const size_t smem_h = (size_t)row_slice_cols(H) * sizeof(float);
  k_norm<kNormGather><<<gnorm, kNormThreads, smem_h, st>>>(
      D->pf_tok, D->embed, D->pf_h, nullptr, D->layers[0].gattn, D->pf_x, nullptr, rows, H, eps,
      PeerIn{});
  count_launches(2);
  if ((e = cudaPeekAtLastError()) != cudaSuccess) return cuda_status(e, "prefill: embed");
  auto gemm = [&](const float *X, const uint32_t *W, const float *S, float *Y, uint32_t out,
                  uint32_t cols) {
    return ternary_gemv_launch(1, X, 0, W, 0, S, 0, nullptr, Y, 0, rows, out, cols, cols / 128,
                               cols / 16, false, UINT64_MAX, D->pf_ws, D->pf_ws_bytes, st);
  };
  for (uint32_t l = 0; l < c.layers; l++) {
    Layer &L = D->layers[l];
    if ((e = gemm(D->pf_x, L.wqkv, L.sqkv, D->pf_qkv, D->qkv_rows, H)) != cudaSuccess)
      return cuda_status(e, "prefill: qkv");
    const uint64_t nrope = (uint64_t)rows * (D->hr + 2 * D->kvr) * (hd / 2);
    k_pf_rope<<<grid_for(nrope, 256), 256, 0, st>>>(D->pf_qkv, D->pf_q, L.ck, L.cv, D->rope, B, n,
                                                    D->hr, D->kvr, hd, c.max_seq);
    count_launches(1);
    if ((e = cudaPeekAtLastError()) != cudaSuccess) return cuda_status(e, "prefill: rope");
    if ((e = attn_causal_prefill_launch(D->pf_q, L.ck, L.cv, D->pf_ctx, B, n, D->hr, D->kvr, hd,
                                        (uint64_t)n * hq, (uint64_t)c.max_seq * D->kvr * hd,
                                        st)) != cudaSuccess)
      return cuda_status(e, "prefill: attention");
    if ((e = gemm(D->pf_ctx, L.wo, L.so, D->pf_o, H, hq)) != cudaSuccess)
      return cuda_status(e, "prefill: o");
    if ((rc = allreduce(D, D->pf_o, (size_t)rows * H, kNcclFloat32, kNcclSum))) return rc;
    if (l + 1 == c.layers) break;   // the last layer's FFN feeds no cache
    // Enough rows to fill the GPU: a CTA per row; else the row clusters.
    const bool by_row = rows >= 2u * 148u && H % 4u == 0 && D->fr % 4u == 0;
    auto add_norm = [&](const float *delta, const float *g) {
      if (by_row)
        k_rows_add_norm<<<rows, kRowThreads, 0, st>>>(D->pf_h, delta, g, D->pf_x, H, eps);
      else
        k_norm<kNormAdd><<<gnorm, kNormThreads, smem_h, st>>>(nullptr, nullptr, D->pf_h, delta, g,
                                                               D->pf_x, nullptr, rows, H, eps,
                                                               PeerIn{});
      count_launches(1);
    };
    add_norm(D->pf_o, L.gffn);
    if ((e = gemm(D->pf_x, L.wgu, L.sgu, D->pf_gu, 2 * D->fr, H)) != cudaSuccess)
      return cuda_status(e, "prefill: gate/up");
    if (by_row)
      k_rows_silu<<<rows, kRowThreads, 0, st>>>(D->pf_gu, D->pf_a, D->fr);
    else
      k_silu_prep<<<gnorm, kNormThreads, (size_t)row_slice_cols(D->fr) * sizeof(float), st>>>(
          D->pf_gu, D->pf_a, nullptr, rows, D->fr);
    count_launches(1);
    if ((e = gemm(D->pf_a, L.wd, L.sd, D->pf_d, H, D->fr)) != cudaSuccess)
      return cuda_status(e, "prefill: down");
    if ((rc = allreduce(D, D->pf_d, (size_t)rows * H, kNcclFloat32, kNcclSum))) return rc;
    add_norm(D->pf_d, D->layers[l + 1].gattn);
    if ((e = cudaPeekAtLastError()) != cudaSuccess) return cuda_status(e, "prefill: norms");
  }
  k_pf_init<<<1, 32, 0, st>>>(D->prompt, P, D->tok, D->par ? nullptr : D->keys, D->pos, D->posf, B);
  count_launches(1);
  return cuda_status(cudaPeekAtLastError(), "prefill: init");
}

extern "C" int nl_decoder_generate(nl_decoder *D, uint32_t batch, uint32_t prompt_len,
                                   const int32_t *prompt, uint32_t steps, int32_t *out_tokens,
                                   double *prefill_ms, double *decode_ms) {
  const nl_decoder_config &c = D->cfg;
  if (batch == 0 || batch > c.max_batch || prompt_len == 0 || steps == 0 ||
      prompt_len + steps - 1 > c.max_seq)
    return set_error(NL_ERROR, "generate: batch %u (max %u), prompt %u + steps %u - 1 > max_seq %u",
                     batch, c.max_batch, prompt_len, steps, c.max_seq);
  for (uint64_t i = 0; i < (uint64_t)batch * prompt_len; i++)
    if (prompt[i] < 0 || (uint32_t)prompt[i] >= c.vocab)
      return set_error(NL_ERROR, "generate: token %d out of range", prompt[i]);
  cudaStream_t st = D->stream;
  cudaError_t e =
      cudaMemcpyAsync(D->prompt, prompt, (size_t)batch * prompt_len * 4, cudaMemcpyHostToDevice, st);
  if (e != cudaSuccess) return cuda_status(e, "generate: prompt");
  D->last_positions = prompt_len;
  int rc;
  auto it = D->graphs.find(batch * 100000u + prompt_len);
  if (it == D->graphs.end()) {
    // One eager step first (kernel attributes, NCCL connections), then capture.
    k_init<<<1, 32, 0, st>>>(D->prompt, prompt_len, D->tok, D->par ? nullptr : D->keys, D->pos,
                             D->posf, batch);
    if ((rc = enqueue_step(D, batch))) return rc;
    if ((rc = cuda_status(cudaStreamSynchronize(st), "generate: warm-up"))) return rc;
    uint64_t before = nl_launch_count();
    cudaGraph_t graph;
    if ((e = cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal)) != cudaSuccess)
      return cuda_status(e, "generate: capture");
    rc = enqueue_step(D, batch);
    e = cudaStreamEndCapture(st, &graph);
    if (rc) return rc;
    if (e != cudaSuccess) return cuda_status(e, "generate: end capture");
    D->kernels_per_step = nl_launch_count() - before;
    cudaGraphExec_t exec;
    e = cudaGraphInstantiate(&exec, graph, 0);
    cudaGraphDestroy(graph);
    if (e != cudaSuccess) return cuda_status(e, "generate: instantiate");
    it = D->graphs.emplace(batch * 100000u + prompt_len, exec).first;
  }
  cudaGraphExec_t exec = it->second;
  // Prompts of more than 16 rows in all: the batched prefill; shorter ones
  // step through the prompt with the decode graph (teacher forcing).
  const bool batched = prompt_len >= 2 && (uint64_t)batch * (prompt_len - 1) > 16;
  if (batched && (rc = prefill_buffers(D, batch * (prompt_len - 1)))) return rc;
  if (!batched)
    k_init<<<1, 32, 0, st>>>(D->prompt, prompt_len, D->tok, D->par ? nullptr : D->keys, D->pos,
                             D->posf, batch);
  cudaEvent_t e0, e1, e2;
  cudaEventCreate(&e0);
  cudaEventCreate(&e1);
  cudaEventCreate(&e2);
  cudaEventRecord(e0, st);
  if (batched) {
    if ((rc = run_prefill(D, batch, prompt_len))) {
      cudaEventDestroy(e0);
      cudaEventDestroy(e1);
      cudaEventDestroy(e2);
      return rc;
    }
  } else {
    for (uint32_t i = 0; i + 1 < prompt_len; i++) cudaGraphLaunch(exec, st);
  }
  cudaEventRecord(e1, st);
  for (uint32_t i = 0; i < steps; i++) cudaGraphLaunch(exec, st);
  cudaEventRecord(e2, st);
  rc = cuda_status(cudaStreamSynchronize(st), "generate");
  float a = 0.0f, b = 0.0f;
  cudaEventElapsedTime(&a, e0, e1);
  cudaEventElapsedTime(&b, e1, e2);
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  cudaEventDestroy(e2);
  if (rc) return rc;
  {
    int herr = 0;
    if ((rc = cuda_status(cudaMemcpy(&herr, D->err, 4, cudaMemcpyDeviceToHost), "generate: err")))
      return rc;
    if (herr)
      return set_error(NL_ERROR, D->par ? "generate: a tensor-parallel peer exchange timed out"
                                        : "generate: a bounded wait of the decode step timed out");
  }
  count_launches(D->kernels_per_step * ((batched ? 0u : prompt_len - 1) + steps));
  if (prefill_ms) *prefill_ms = a;
  if (decode_ms) *decode_ms = b;
  D->last_batch = batch;
  std::vector<int32_t> tmp((size_t)steps * batch);
  e = cudaMemcpy(tmp.data(), D->out_tok, tmp.size() * 4, cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_status(e, "generate: tokens");
  for (uint32_t i = 0; i < steps; i++)
    for (uint32_t bb = 0; bb < batch; bb++) out_tokens[(size_t)bb * steps + i] = tmp[(size_t)i * batch + bb];
  return NL_OK;
}

extern "C" int nl_decoder_logits(nl_decoder *D, float *out, uint64_t nfloats) {
  if (!D->keep_logits) return set_error(NL_ERROR, "decoder created without keep_logits");
  uint64_t have = (uint64_t)D->cfg.max_seq * D->cfg.max_batch * D->vr;
  if (nfloats > have) nfloats = have;
  return cuda_status(cudaMemcpy(out, D->logits, nfloats * 4, cudaMemcpyDeviceToHost), "logits");
}

extern "C" int nl_decoder_shard(const nl_decoder_config *cfg, int tp_rank, int tp_size,
                                uint32_t *shard) {
  if (!cfg || !shard) return set_error(NL_ERROR, "decoder shard: null argument");
  int rc = check_config(*cfg);
  if (rc) return rc;
  Shard sh;
  if ((rc = plan_shard(*cfg, tp_rank, tp_size, &sh))) return rc;
  shard[0] = sh.kvh.begin;
  shard[1] = sh.kvh.count;
  shard[2] = sh.ffb.begin * 128;
  shard[3] = sh.ffb.count * 128;
  shard[4] = sh.voc.begin;
  shard[5] = sh.voc.count;
  return NL_OK;
}

extern "C" int nl_decoder_info(nl_decoder *D, uint32_t *shard, uint64_t *weight_bytes,
                               uint64_t *kernels_per_step) {
  if (shard) {
    shard[0] = D->kvh.begin;
    shard[1] = D->kvh.count;
    shard[2] = D->ffb.begin * 128;
    shard[3] = D->fr;
    shard[4] = D->v0;
    shard[5] = D->vr;
  }
  if (weight_bytes) *weight_bytes = D->weight_bytes;
  if (kernels_per_step) *kernels_per_step = D->kernels_per_step;
  return NL_OK;
}

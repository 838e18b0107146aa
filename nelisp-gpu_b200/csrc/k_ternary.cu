// k_ternary.cu -- ternary (two-bit) linear kernels for sm_100a.
//
// Reference operators (lisp/nelisp-gpu-kernels.el):
//   ternary-rows       :713-746   Y = BIAS + sum_b BETA[o,b] * sum_{i in b} t(o,i) X[s,i]
//   ternary-rows-t     :750-772   X = W^T (BETA o G)
//   bitlinear-packed   :998-1016  base-4 codes in the integer value of an f32, BETA[0]
//   bitlinear-packed-v :1022-1040 the same with BETA[o]
//
// The ternary GEMV is HBM-bound (2 bits of weight per multiply-add) and the
// CUDA-core formulation -- unpack a field, convert, FMA -- costs more issue
// slots per weight than HBM delivers weights.  The fast path therefore moves
// the arithmetic onto the tensor cores in exact integer form:
//
//  * prep: every activation row s is scaled by a power of two 2^e_s so that
//    max|x| lands in [2^(8L-3), 2^(8L-2)), rounded to an integer xq and split
//    into L balanced int8 limbs, xq = l0 + 256 l1 + 65536 l2 (+ 2^24 l3):
//    L = 4 (30 bits) for up to four sequence rows, whose limb columns fit
//    the n-tiles three would take, else L = 3 (22 bits).  The rounding is the
//    only inexact step (half a unit of 2^-(8L-2) of the row maximum).  Limbs
//    are written straight into mma B-fragment order, so the main loop loads
//    one uint2 per MMA.
//  * main: each warp owns 16 weight rows.  Lanes load the packed words
//    (8 bytes per row per 128-column block, 4 lanes per row), turn the
//    two-bit codes into int8 operands with a shift and a mask per four codes
//    (a code in the top two bits of a byte is 64 times its trit:
//    00->0, 01->+1, 10->-2, 11->-1, the reference's sign-extending decode)
//    and issue mma.m16n8k32.s8 with int32 accumulation: the dot products are
//    exact.  N carries (sequence, limb) pairs: n = L s + l.
//  * epilogue: the L limb sums of (row, s) are combined in int64,
//    converted once and scaled by 2^-e_s and the row's scale (per-row mode),
//    or flushed per 128-column block against BETA[o,b] (ternary-rows mode).
//
// The K order inside a block is permuted identically in the A (weights) and
// B (activations) fragments, which a dot product does not observe.
// Rows whose activations are non-finite or below 2^-104 cannot be scaled into
// int8 limbs; prep flags them and the epilogue recomputes those outputs on
// the CUDA cores with the generic kernel's arithmetic.

#include <cuda.h>
#include <cooperative_groups.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>


#include "nl_internal.h"
#include "ternary_mma.cuh"
#include "ternary_prep.cuh"

namespace nl {
namespace cg = cooperative_groups;
namespace {

constexpr int kDepth = 8;        // 128-column blocks in flight per warp

// One warp per (problem z, output row o), sequences in chunks of 8.
__global__ void __launch_bounds__(256)
ternary_generic_kernel(const float *__restrict__ X, uint64_t x_stride,
                       const uint32_t *__restrict__ WP, uint64_t w_stride,
                       const float *__restrict__ SCALE, uint64_t s_stride,
                       const float *__restrict__ BIAS, float *__restrict__ Y,
                       uint64_t y_stride, uint32_t seq, uint32_t out,
                       uint32_t cols, uint32_t nblk, uint32_t wng,
                       int per_block, uint64_t limit) {
  const int warps = blockDim.x >> 5;
  const uint32_t o = blockIdx.x * warps + (threadIdx.x >> 5);
  const uint32_t z = blockIdx.y;
  if (o >= out) return;
  const float *Xz = X + z * x_stride;
  const uint32_t *Wrow = WP + z * w_stride + (uint64_t)o * wng;
  const float *Sz = SCALE + z * s_stride;
  const float *beta_row = per_block ? Sz + (uint64_t)o * nblk : nullptr;
  float row_scale = per_block ? 1.0f : __ldg(Sz + o);
  float bias = BIAS ? __ldg(BIAS + o) : 0.0f;
  float *Yz = Y + z * y_stride;
  for (uint32_t s0 = 0; s0 < seq; s0 += 8) {
    int ns = (int)min(8u, seq - s0);
    float acc[8];
    ternary_row_generic<8>(Xz, Wrow, beta_row, per_block != 0, row_scale,
                           (int)s0, ns, cols, nblk, wng, acc);
    if ((threadIdx.x & 31) == 0) {
      for (int s = 0; s < ns; s++) {
        uint64_t idx = (uint64_t)(s0 + s) * out + o;
        if (idx < limit) Yz[idx] = bias + acc[s];
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Fast path, step 1: activations -> int8 limbs in mma B-fragment order.
// ---------------------------------------------------------------------------
// The fragment format and the activation prep live in ternary_prep.cuh, shared
// with the decoder's fused normalisation kernels.

// grid (kRowCluster * seq, count), kPrepThreads threads, clusters of
// kRowCluster CTAs.  Cluster s handles sequence row s of problem z; each CTA
// takes a column slice, and the row maximum is combined through distributed
// shared memory in rank order, so every CTA scales the row by the same power
// of two.  The padding columns n >= 3*seq of the last n-tile are not written:
// an MMA output column depends only on its own B column, and the GEMV's
// epilogue never reads the padding columns' outputs.
constexpr int kPrepThreads = 128;
__global__ void __cluster_dims__(kRowCluster, 1, 1) __launch_bounds__(kPrepThreads)
ternary_prep_kernel(const float *__restrict__ X, uint64_t x_stride,
                    uint32_t seq, uint32_t cols, void *ws) {
  pdl_trigger();                  // the GEMV may start streaming its weights
  pdl_wait();                     // X may come from the preceding kernel
  __shared__ float red[32];
  __shared__ float s_max;
  __shared__ int s_bad;
  cg::cluster_group cl = cg::this_cluster();
  const uint32_t rank = cl.block_rank();
  const uint32_t s = blockIdx.x / kRowCluster, z = blockIdx.y;
  const RowSlice sl = row_slice(cols, rank);
  const bool live = s < seq;
  const float *xr = X + z * x_stride + (size_t)s * cols;
  float m = 0.0f;
  int bad = 0;
  if (live) {
    for (uint32_t i = sl.c0 + threadIdx.x; i < sl.c1; i += blockDim.x) {
      const float v = xr[i];
      m = fmaxf(m, fabsf(v));
      bad |= !isfinite(v);        // NaN is dropped by fmaxf; catch it here
    }
  }
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  bad = __syncthreads_or(bad);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    float r = 0.0f;
    for (int i = 0; i < (int)(blockDim.x >> 5); i++) r = fmaxf(r, red[i]);
    s_max = r;
    s_bad = bad;
  }
  cl.sync();
  float mm = 0.0f;
  int anybad = 0;
#pragma unroll
  for (int k = 0; k < kRowCluster; k++) {
    mm = fmaxf(mm, *cl.map_shared_rank(&s_max, k));
    anybad |= *cl.map_shared_rank(&s_bad, k);
  }
  quantize_slice(xr + sl.c0, sl, mm, anybad != 0, live, rank, s, seq,
                 prep_at(ws, (int)seq, cols, z));
  cl.sync();                      // no CTA leaves while its maximum is read
}

// Many rows (count * seq >= kPrepRowsMin): one CTA per (row s, problem z),
// no cluster and no cluster barrier (prep_row_cta).  Needs X 16-byte
// aligned, x_stride % 4 == 0 and cols % 16 == 0.
constexpr int kPrepRowThreads = 256;
constexpr uint32_t kPrepRowsMin = 32;
__global__ void __launch_bounds__(kPrepRowThreads)
ternary_prep_rows_kernel(const float *__restrict__ X, uint64_t x_stride, uint32_t seq,
                         uint32_t cols, void *ws) {
  pdl_trigger();                  // the GEMV may start streaming its weights
  pdl_wait();                     // X may come from the preceding kernel
  __shared__ float red[32];
  __shared__ long long xred[32];
  const uint32_t s = blockIdx.x, z = blockIdx.y;
  prep_row_cta(X + z * x_stride + (size_t)s * cols, cols, s, seq, prep_at(ws, (int)seq, cols, z),
               red, xred);
}

// The GEMV's prep launch: the one-CTA-per-row kernel for many aligned rows,
// else the clustered one.
cudaError_t launch_prep_any(const float *X, uint64_t x_stride, uint32_t count, uint32_t seq,
                            uint32_t cols, void *ws, cudaStream_t st, bool pdl) {
  if ((uint64_t)count * seq >= kPrepRowsMin && ((uintptr_t)X & 15u) == 0 && x_stride % 4u == 0 &&
      cols % 16u == 0)
    return launch_k(ternary_prep_rows_kernel, dim3(seq, count), dim3(kPrepRowThreads), 0, st,
                    pdl, X, x_stride, seq, cols, ws);
  return launch_k(ternary_prep_kernel, dim3(kRowCluster * seq, count), dim3(kPrepThreads), 0, st,
                  pdl, X, x_stride, seq, cols, ws);
}

// ---------------------------------------------------------------------------
// Fast path, step 2: the tensor-core GEMV.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void cp_async16(void *smem, const void *gmem) {
  unsigned s = (unsigned)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gmem));
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;\n" ::);
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}

// Blocks per shared-memory chunk of activation fragments; also the depth of
// the per-warp weight prefetch (one chunk ahead).
constexpr int kChunk = kDepth;

__host__ __device__ inline size_t mma_smem_bytes(int NT) {
  return (size_t)2 * kChunk * NT * 128 * sizeof(uint2);   // double-buffered chunk
}

// XSUM of a problem's rows spread over a warp: in pass p, lane l holds
// partial l % 8 of row 4p + l / 8 (zero past SEQ).  The loads are issued
// early, one or a few per lane, and combined late: total() leaves row l's
// sum in lane l.  NT n-tiles hold at most 8 NT / 3 rows.
template <int NT>
struct XsumLanes {
  static constexpr int kPasses = (8 * NT / 3 + 3) / 4;
  long long v[kPasses];
  __device__ __forceinline__ void load(const PrepOut &P, uint32_t seq, int lane) {
#pragma unroll
    for (int p = 0; p < kPasses; p++) {
      const uint32_t s = 4u * p + (uint32_t)(lane >> 3);
      v[p] = s < seq ? __ldcg(P.xsum + s * kRowCluster + (lane & 7)) : 0ll;
    }
  }
  __device__ __forceinline__ void zero() {
#pragma unroll
    for (int p = 0; p < kPasses; p++) v[p] = 0ll;
  }
  // All 32 lanes call it.
  __device__ __forceinline__ long long total(int lane) const {
    long long mine = 0;
#pragma unroll
    for (int p = 0; p < kPasses; p++) {
      long long t = v[p];
      t += __shfl_xor_sync(0xffffffffu, t, 1);
      t += __shfl_xor_sync(0xffffffffu, t, 2);
      t += __shfl_xor_sync(0xffffffffu, t, 4);
      const long long r = __shfl_sync(0xffffffffu, t, (lane & 3) * 8);   // row 4p + lane % 4
      if ((lane >> 2) == p) mine = r;
    }
    return mine;
  }
};

// One chunk of kChunk blocks for one warp: consume the weight registers,
// refill them with the blocks kChunk further on, run the MMAs against the
// staged fragments.  PRED guards a partial chunk and the last refill; whole
// chunks run without any per-block test.
template <int NT, bool PER_BLOCK, bool PRED>
__device__ __forceinline__ void mma_chunk(int (&acc)[NT][2][4], float (&yf)[NT][4],
                                          uint2 (&wa)[kChunk], uint2 (&wb)[kChunk],
                                          const uint2 *fb, const uint2 *pa, const uint2 *pb,
                                          uint32_t blk0, uint32_t nblk, const float *Sz,
                                          uint32_t rA, uint32_t rB) {
#pragma unroll
  for (int u = 0; u < kChunk; u++) {
    if (PRED && blk0 + u >= nblk) break;
    const uint2 a = wa[u], c = wb[u];
    if (!PRED || blk0 + u + kChunk < nblk) {
      wa[u] = __ldcs(pa + 4 * (u + kChunk));
      wb[u] = __ldcs(pb + 4 * (u + kChunk));
    }
    uint32_t A[4][4];
    unpack_signed(a, c, A);
    const uint2 *fu = fb + u * NT * 128;
    // Two accumulator chains per n-tile, so consecutive MMAs do not wait on
    // each other's results.
#pragma unroll
    for (int t = 0; t < NT; t++) {
      const uint4 f01 = *reinterpret_cast<const uint4 *>(fu + t * 128);
      const uint4 f23 = *reinterpret_cast<const uint4 *>(fu + t * 128 + 64);
      mma_s8(acc[t][0], A[0][0], A[0][1], A[0][2], A[0][3], lo2(f01));
      mma_s8(acc[t][1], A[1][0], A[1][1], A[1][2], A[1][3], hi2(f01));
      mma_s8(acc[t][0], A[2][0], A[2][1], A[2][2], A[2][3], lo2(f23));
      mma_s8(acc[t][1], A[3][0], A[3][1], A[3][2], A[3][3], hi2(f23));
    }
    if (PER_BLOCK) {
      // BETA is per (row, 128-column block): flush the exact block sums.
      const uint32_t blk = blk0 + u;
      const float bA = __ldg(Sz + (uint64_t)rA * nblk + blk);
      const float bB = __ldg(Sz + (uint64_t)rB * nblk + blk);
#pragma unroll
      for (int t = 0; t < NT; t++) {
#pragma unroll
        for (int r = 0; r < 4; r++) {
          yf[t][r] = fmaf((float)(acc[t][0][r] + acc[t][1][r]), r < 2 ? bA : bB, yf[t][r]);
          acc[t][0][r] = acc[t][1][r] = 0;
        }
      }
    }
  }
}

// One CTA = `blockDim.x / 32` warps over consecutive 16-row groups of one
// problem z.  The warps share the problem's activation fragments: chunks of
// kChunk blocks are copied into shared memory with cp.async (double
// buffered), while each warp streams its own weight rows kChunk blocks ahead
// through registers.
template <int NT, bool PER_BLOCK>
__global__ void __launch_bounds__(256)
ternary_mma_kernel(const float *__restrict__ X, uint64_t x_stride,
                   const uint32_t *__restrict__ WP, uint64_t w_stride,
                   const float *__restrict__ SCALE, uint64_t s_stride,
                   const float *__restrict__ BIAS, float *__restrict__ Y,
                   uint64_t y_stride, uint32_t seq, uint32_t out,
                   uint32_t cols, uint64_t limit, void *ws) {
  extern __shared__ __align__(16) uint2 smem[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nwarps = blockDim.x >> 5;
  const int g = lane >> 2, q = lane & 3;
  const uint32_t z = blockIdx.y;
  const uint32_t rg = blockIdx.x * nwarps + warp;          // 16-row group
  const bool active = rg * 16u < out;
  const uint32_t nblk = cols / 128u, wng = cols / 16u;
  const uint32_t nchunk = (nblk + kChunk - 1) / kChunk;
  PrepOut P = prep_at(ws, (int)seq, cols, z);
  const uint32_t rA = active ? min(rg * 16u + (uint32_t)g, out - 1u) : 0u;
  const uint32_t rB = active ? min(rg * 16u + (uint32_t)g + 8u, out - 1u) : 0u;
  const uint32_t *Wz = WP + z * w_stride;
  const uint2 *pA = reinterpret_cast<const uint2 *>(Wz + (uint64_t)rA * wng) + q;
  const uint2 *pB = reinterpret_cast<const uint2 *>(Wz + (uint64_t)rB * wng) + q;
  const float *Sz = SCALE + z * s_stride;
  constexpr int kChunkU2 = kChunk * NT * 128;              // uint2 per chunk

  // Stage chunk c of the fragments into buffer b.
  auto stage = [&](uint32_t c, int b) {
    const uint32_t nb = min((uint32_t)kChunk, nblk - c * kChunk);
    const uint32_t n16 = nb * NT * 64;                       // 16-byte pieces
    const char *src = reinterpret_cast<const char *>(P.frag + (size_t)c * kChunkU2);
    char *dst = reinterpret_cast<char *>(smem + b * kChunkU2);
    for (uint32_t i = threadIdx.x; i < n16; i += blockDim.x) cp_async16(dst + 16 * i, src + 16 * i);
    cp_async_commit();
  };

  int acc[NT][2][4];
  float yf[NT][4];
#pragma unroll
  for (int t = 0; t < NT; t++)
#pragma unroll
    for (int r = 0; r < 4; r++) { acc[t][0][r] = acc[t][1][r] = 0; yf[t][r] = 0.0f; }

  uint2 wa[kChunk], wb[kChunk];
  if (active) {
#pragma unroll
    for (int u = 0; u < kChunk; u++) {
      if ((uint32_t)u < nblk) {
        wa[u] = __ldcs(pA + 4u * u);
        wb[u] = __ldcs(pB + 4u * u);
      }
    }
  }
  stage(0, 0);
  for (uint32_t c = 0; c < nchunk; c++) {
    if (c + 1 < nchunk) {
      stage(c + 1, (c + 1) & 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    if (active) {
      const uint2 *fb = smem + (c & 1) * kChunkU2 + 2 * lane;
      const uint32_t blk0 = c * kChunk;
      if (blk0 + 2 * kChunk <= nblk)   // this chunk and the next are whole
        mma_chunk<NT, PER_BLOCK, false>(acc, yf, wa, wb, fb, pA + 4u * blk0, pB + 4u * blk0,
                                        blk0, nblk, Sz, rA, rB);
      else
        mma_chunk<NT, PER_BLOCK, true>(acc, yf, wa, wb, fb, pA + 4u * blk0, pB + 4u * blk0,
                                       blk0, nblk, Sz, rA, rB);
    }
    __syncthreads();   // the buffer is restaged two chunks later
  }
  if (!active) return;

  // Epilogue: stage per-(row, n) results in shared memory (reusing the
  // fragment buffers), then combine the limbs of each (row, s).
  // Per-block results are float sums; they travel as bit patterns.
  int(*s_acc)[8 * NT + 1] =
      reinterpret_cast<int(*)[8 * NT + 1]>(reinterpret_cast<int *>(smem) + warp * 16 * (8 * NT + 1));
#pragma unroll
  for (int t = 0; t < NT; t++) {
    const int v0 = PER_BLOCK ? __float_as_int(yf[t][0]) : acc[t][0][0] + acc[t][1][0];
    const int v1 = PER_BLOCK ? __float_as_int(yf[t][1]) : acc[t][0][1] + acc[t][1][1];
    const int v2 = PER_BLOCK ? __float_as_int(yf[t][2]) : acc[t][0][2] + acc[t][1][2];
    const int v3 = PER_BLOCK ? __float_as_int(yf[t][3]) : acc[t][0][3] + acc[t][1][3];
    s_acc[g][8 * t + 2 * q] = v0;
    s_acc[g][8 * t + 2 * q + 1] = v1;
    s_acc[g + 8][8 * t + 2 * q] = v2;
    s_acc[g + 8][8 * t + 2 * q + 1] = v3;
  }
  __syncwarp();
  float *Yz = Y + z * y_stride;
  bool any_flag = false;
  for (uint32_t s = 0; s < seq; s++) any_flag |= (P.rowflag[s] != 0);
  const int L = n_limbs((int)seq);
  for (uint32_t idx = lane; idx < 16u * seq; idx += 32u) {
    const uint32_t r = idx & 15u, s = idx >> 4;
    const uint32_t o = rg * 16u + r;
    if (o >= out) continue;
    float y;
    if (PER_BLOCK) {
      y = limb_total_f(s_acc[r], s, L) * P.rowinv[s];
    } else {
      long long tot = limb_total(s_acc[r], s, L);
      tot >>= 6;                               // the operands carried 64 * t: exact
      y = ((float)tot * P.rowinv[s]) * __ldg(Sz + o);
    }
    if (BIAS) y = __ldg(BIAS + o) + y;
    uint64_t oi = (uint64_t)s * out + o;
    if (oi < limit && !P.rowflag[s]) Yz[oi] = y;
  }
  if (any_flag) {
    // Rows the limbs cannot represent: the generic arithmetic, per row.
    const float *Xz = X + z * x_stride;
    for (uint32_t r = 0; r < 16u; r++) {
      const uint32_t o = rg * 16u + r;
      if (o >= out) break;
      float acc8[8];
      const uint32_t *Wrow = Wz + (uint64_t)o * wng;
      for (uint32_t s0 = 0; s0 < seq; s0 += 8) {
        int ns = (int)min(8u, seq - s0);
        ternary_row_generic<8>(Xz, Wrow, PER_BLOCK ? Sz + (uint64_t)o * nblk : nullptr,
                               PER_BLOCK, PER_BLOCK ? 1.0f : __ldg(Sz + o),
                               (int)s0, ns, cols, nblk, wng, acc8);
        if (lane == 0) {
          for (int k = 0; k < ns; k++) {
            uint32_t s = s0 + k;
            uint64_t oi = (uint64_t)s * out + o;
            if (P.rowflag[s] && oi < limit)
              Yz[oi] = (BIAS ? __ldg(BIAS + o) : 0.0f) + acc8[k];
          }
        }
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Fast path, step 2 (TMA): the same GEMV with the weight tiles streamed by the
// Tensor Memory Accelerator.  One producer warp issues, per chunk of four
// 128-column blocks, a 2-D tensor copy of the CTA's rows (128 bytes per row,
// 128B-swizzled so the consumers' 8-byte reads are bank-conflict free) and a
// 1-D bulk copy of the matching activation fragments, both completing on
// the stage's mbarrier.  Consumer warps wait on it, unpack and issue the
// MMAs, and release the stage.  Every wait is bounded: on timeout the warp
// records an error and returns.
// ---------------------------------------------------------------------------
constexpr int kTmaBlocks = 4;                 // 128-column blocks per stage
// Zero activation fragments for the blocks past the row end of a partial
// stage (at most kTmaBlocks - 1 blocks of 6 n-tiles).
__device__ __align__(128) unsigned char g_zero_frags[(kTmaBlocks - 1) * 6 * 1024];


__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(smem_u32(bar)),
               "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(smem_u32(bar)) : "memory");
}
// Bounded wait for the phase of parity PARITY to complete.  Each try_wait
// suspends the thread in hardware until the phase completes or kSuspendNs
// pass, so a waiting warp takes no issue slots; after kWaitRounds rounds
// (seconds) the wait gives up and records it in the host-visible flag ERR.
constexpr uint32_t kSuspendNs = 1000000;
constexpr uint32_t kWaitRounds = 4096;
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, int *err) {
  const uint32_t a = smem_u32(bar);
  for (uint32_t i = 0; i < kWaitRounds; i++) {
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done) : "r"(a), "r"(parity), "r"(kSuspendNs) : "memory");
    if (done) return true;
  }
  report_wait_timeout(err);
  return false;
}
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int x, int y,
                                            uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];\n" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void bulk_load(void *dst, const void *src, uint32_t bytes,
                                          uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n"
      ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ uint4 lds128(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];\n"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
  return v;
}
__device__ __forceinline__ uint2 lds64(uint32_t addr) {
  uint2 v;
  asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];\n" : "=r"(v.x), "=r"(v.y) : "r"(addr));
  return v;
}

// 16-row groups a consumer warp multiplies per item.  One or two n-tiles (up
// to 4 sequence rows) take two: both groups' MMAs use each activation
// fragment load, and the ring wait, the stage release and the loop cost are
// paid once per two groups' weights.  Such a CTA fills an SM alone (ring up
// to 200 KB, the register file for 9 warps).  Measured, 64 x 4096^2: batch 1
// 0.73 -> 0.81 of HBM, batch 4 4073 -> 4300 GB/s.  Other paths take one
// group, two CTAs an SM.
__host__ __device__ constexpr int tma_groups(int NT, bool per_block) {
  return (!per_block && NT <= 2) ? 2 : 1;
}
__host__ __device__ inline int tma_stages(int NT, int nw, int rg) {
  int per = 2048 * nw * rg + NT * kTmaBlocks * 1024;
  int st = ((rg == 1 ? 112 : nw >= 8 ? 200 : 100) * 1024) / per;
  return st < 2 ? 2 : (st > 6 ? 6 : st);
}
__host__ __device__ inline size_t tma_smem_bytes(int NT, int nw, int rg) {
  int S = tma_stages(NT, nw, rg);
  return 1024 /* alignment slack */ + (size_t)S * (2048 * nw * rg + NT * kTmaBlocks * 1024) +
         (size_t)2 * S * 8 + (size_t)nw * 16 * rg * (8 * NT + 1) * 4;
}

// Persistent: a grid of at most (resident CTAs per SM) x 148 CTAs walks the
// work items -- (problem z, tile of 16*RG*nw rows) -- round-robin.  The producer
// warp streams the (item, chunk) sequence through the S-stage ring without a
// break between items, so the copies of a CTA's next item are in flight while
// the consumers finish the current one and run its epilogue.
template <int NT, bool PER_BLOCK>
__global__ void __launch_bounds__(288, (NT <= 3 && tma_groups(NT, PER_BLOCK) == 1) ? 2 : 1)
ternary_tma_kernel(const __grid_constant__ CUtensorMap tmW, const float *__restrict__ X,
                   uint64_t x_stride, const uint32_t *__restrict__ WP, uint64_t w_stride,
                   const float *__restrict__ SCALE, uint64_t s_stride,
                   const float *__restrict__ BIAS, float *__restrict__ Y, uint64_t y_stride,
                   uint32_t seq, uint32_t out, uint32_t cols, uint64_t limit, void *ws,
                   uint32_t count, int *err) {
  extern __shared__ uint8_t smem_raw[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nw = (blockDim.x >> 5) - 1;            // consumer warps; warp nw produces
  constexpr int RG = tma_groups(NT, PER_BLOCK);
  constexpr uint32_t R = 16u * RG;                 // rows of one warp's item
  static_assert(RG == 1 || !PER_BLOCK, "per-block scales take one row group");
  const int S = tma_stages(NT, nw, RG);
  const uint32_t wbytes = 2048u * nw * RG;         // weight tile per stage
  const uint32_t fstage = NT * kTmaBlocks * 128;   // fragment uint2 per stage
  uint8_t *base = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  uint8_t *wbuf = base;                                                // S x wbytes
  uint2 *fbuf = reinterpret_cast<uint2 *>(base + (size_t)S * wbytes);  // S x fstage
  uint64_t *full = reinterpret_cast<uint64_t *>(fbuf + (size_t)S * fstage);
  uint64_t *empty = full + S;
  int *epi = reinterpret_cast<int *>(empty + S);

  const uint32_t nblk = cols / 128u, wng = cols / 16u;
  const uint32_t nchunk = (nblk + kTmaBlocks - 1) / kTmaBlocks;
  const uint32_t tpp = (out + R * nw - 1) / (R * nw);       // tiles per problem
  const uint32_t items = tpp * count;

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; i++) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], (uint32_t)nw);
    }
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  __syncthreads();

  if (warp == nw) {
    // ---- producer ----
    if (lane == 0) {
      // This CTA's chunks k = 0 .. total-1 are chunk k % nchunk of item
      // blockIdx.x + (k / nchunk) * gridDim.x.  The weights of the first
      // `pre` chunks are requested before waiting for the kernel that wrote
      // the fragments (launch_pdl); the weights are not written by it.
      const uint32_t mine = items > blockIdx.x ? (items - blockIdx.x + gridDim.x - 1) / gridDim.x
                                               : 0u;
      const uint32_t total = mine * nchunk;
      const uint32_t pre = total < (uint32_t)S ? total : (uint32_t)S;
      int st = 0;
      uint32_t ph = 0;                             // parity of the current lap
      uint32_t g = 0;
      for (; g < total; g++) {
        if (g >= (uint32_t)S && !mbar_wait(&empty[st], ph ^ 1u, err)) break;
        const uint32_t it = blockIdx.x + (g / nchunk) * gridDim.x, c = g % nchunk;
        const uint32_t z = it / tpp, tile = it % tpp;
        const uint32_t nb = min((uint32_t)kTmaBlocks, nblk - c * kTmaBlocks);
        mbar_expect_tx(&full[st], wbytes + (uint32_t)kTmaBlocks * NT * 1024u);
        tma_load_2d(wbuf + (size_t)st * wbytes, &tmW, (int)(c * 32u),
                    (int)(z * out + tile * R * nw), &full[st]);
        if (nb < (uint32_t)kTmaBlocks)             // the blocks past the row end
          bulk_load(fbuf + (size_t)st * fstage + (size_t)nb * NT * 128u, g_zero_frags,
                    ((uint32_t)kTmaBlocks - nb) * NT * 1024u, &full[st]);
        if (g >= pre) {
          bulk_load(fbuf + (size_t)st * fstage, prep_at(ws, (int)seq, cols, z).frag +
                    (size_t)c * fstage, nb * NT * 1024u, &full[st]);
        } else if (g + 1 == pre) {
          pdl_wait();
          for (uint32_t k = 0; k < pre; k++) {
            const uint32_t itk = blockIdx.x + (k / nchunk) * gridDim.x, ck = k % nchunk;
            const uint32_t nbk = min((uint32_t)kTmaBlocks, nblk - ck * kTmaBlocks);
            bulk_load(fbuf + (size_t)k * fstage,
                      prep_at(ws, (int)seq, cols, itk / tpp).frag + (size_t)ck * fstage,
                      nbk * NT * 1024u, &full[k]);
          }
        }
        if (++st == S) {
          st = 0;
          ph ^= 1u;
        }
      }
      // Leave only when the last copies have landed (bounded).
      for (uint32_t k = g > (uint32_t)S ? g - S : 0; k < g; k++)
        mbar_wait(&full[k % S], (k / S) & 1, err);
    }
    return;
  }

  // ---- consumers ----
  // One n-tile (one or two sequence rows) takes the one-LOP3 offset operands;
  // more n-tiles keep the signed ones, whose extra chains would not fit the
  // register budget of two CTAs per SM without spilling.
  constexpr bool OFF = !PER_BLOCK && NT == 1;
  pdl_wait();                                      // the epilogue reads the prep's flags
  const uint32_t xkey = offset_key();
  const int gq = lane >> 2, q = lane & 3;
  // Byte offsets of this lane's 8-byte words in a stage's weight tile: row r
  // of the tile holds 128 bytes; the 16-byte chunk k of row r sits at chunk
  // k ^ (r % 8) (128B swizzle).  Block b, words 2q..2q+1 -> chunk 2b + q/2.
  // Row group g of the warp adds 16 g rows: 2048 g bytes, same swizzle.
  const uint32_t rowA = (uint32_t)warp * R + gq, rowB = rowA + 8u;
  uint32_t offA[kTmaBlocks], offB[kTmaBlocks];
#pragma unroll
  for (int b = 0; b < kTmaBlocks; b++) {
    const uint32_t k = 2u * b + (q >> 1), in = (q & 1) * 8u;
    offA[b] = rowA * 128u + ((k ^ (rowA & 7u)) << 4) + in;
    offB[b] = rowB * 128u + ((k ^ (rowB & 7u)) << 4) + in;
  }
  int(*s_acc)[8 * NT + 1] = reinterpret_cast<int(*)[8 * NT + 1]>(epi + warp * R * (8 * NT + 1));

  const uint32_t wsm = smem_u32(wbuf), fsm = smem_u32(fbuf);
  int cst = 0;                                     // ring stage and lap parity
  uint32_t cph = 0;
  for (uint32_t it = blockIdx.x; it < items; it += gridDim.x) {
    const uint32_t z = it / tpp, tile = it % tpp;
    const uint32_t rbase = (tile * nw + warp) * R;  // this warp's first row in problem z
    const bool active = rbase < out;
    const uint32_t rA = active ? min(rbase + (uint32_t)gq, out - 1u) : 0u;
    const uint32_t rB = active ? min(rbase + (uint32_t)gq + 8u, out - 1u) : 0u;
    const float *Sz = SCALE + z * s_stride;
    PrepOut P = prep_at(ws, (int)seq, cols, z);
    // The epilogue's operands, requested now so their latency hides behind
    // the chunk loop: lane l holds the scale and bias of row l % R of the
    // warp's rows and the inverse scale and flag of sequence row l.
    const uint32_t erow = active ? min(rbase + (uint32_t)lane % R, out - 1u) : 0u;
    const float e_scale = PER_BLOCK ? 0.0f : __ldg(Sz + erow);
    const float e_bias = BIAS ? __ldg(BIAS + erow) : 0.0f;
    const float e_rinv = (uint32_t)lane < seq ? P.rowinv[lane] : 0.0f;
    const int e_flag = (uint32_t)lane < seq ? P.rowflag[lane] : 0;
    XsumLanes<NT> xl;
    if (OFF)
      xl.load(P, seq, lane);
    else
      xl.zero();

    int acc[RG][NT][4][4];                // [group][n-tile][k-step][reg]: independent chains
    float yf[NT][4];
#pragma unroll
    for (int t = 0; t < NT; t++)
#pragma unroll
      for (int r = 0; r < 4; r++) {
        yf[t][r] = 0.0f;
#pragma unroll
        for (int g = 0; g < RG; g++)
#pragma unroll
          for (int j = 0; j < 4; j++) acc[g][t][j][r] = 0;
      }

    // Chunks run without a per-block test: in the row's last chunk, when
    // nblk is not a multiple of kTmaBlocks, the blocks past the row end hold
    // TMA's zero fill and zero fragments (the producer copies them), so they
    // add an exact 0 with either operand form.
    for (uint32_t c = 0; c < nchunk; c++) {
      if (!mbar_wait(&full[cst], cph, err)) return;
      const uint32_t wt = wsm + (uint32_t)cst * wbytes;
      const uint32_t fb = fsm + (uint32_t)cst * (fstage * 8u) + (uint32_t)lane * 16u;
#pragma unroll
      for (int b = 0; b < kTmaBlocks; b++) {
        uint32_t A[RG][4][4];
#pragma unroll
        for (int g = 0; g < RG; g++) {
          const uint2 a = lds64(wt + offA[b] + 2048u * g);
          const uint2 cw = lds64(wt + offB[b] + 2048u * g);
          if (OFF)
            unpack_offset(a, cw, xkey, A[g]);
          else
            unpack_signed(a, cw, A[g]);
        }
#pragma unroll
        for (int t = 0; t < NT; t++) {
          const uint32_t ft = fb + (uint32_t)(b * NT + t) * 1024u;
          const uint4 f01 = lds128(ft), f23 = lds128(ft + 512u);
#pragma unroll
          for (int g = 0; g < RG; g++) {
            mma_s8(acc[g][t][0], A[g][0][0], A[g][0][1], A[g][0][2], A[g][0][3], lo2(f01));
            mma_s8(acc[g][t][1], A[g][1][0], A[g][1][1], A[g][1][2], A[g][1][3], hi2(f01));
            mma_s8(acc[g][t][2], A[g][2][0], A[g][2][1], A[g][2][2], A[g][2][3], lo2(f23));
            mma_s8(acc[g][t][3], A[g][3][0], A[g][3][1], A[g][3][2], A[g][3][3], hi2(f23));
          }
        }
        if (PER_BLOCK) {
          const uint32_t blk = c * kTmaBlocks + b;
          if (blk < nblk) {
            const float bA = __ldg(Sz + (uint64_t)rA * nblk + blk);
            const float bB = __ldg(Sz + (uint64_t)rB * nblk + blk);
#pragma unroll
            for (int t = 0; t < NT; t++) {
#pragma unroll
              for (int r = 0; r < 4; r++) {
                int(&a0)[4][4] = acc[0][t];
                const int v = a0[0][r] + a0[1][r] + a0[2][r] + a0[3][r];
                yf[t][r] = fmaf((float)v, r < 2 ? bA : bB, yf[t][r]);
                a0[0][r] = a0[1][r] = a0[2][r] = a0[3][r] = 0;
              }
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[cst]);
      if (++cst == S) {
        cst = 0;
        cph ^= 1u;
      }
    }
    if (!active) continue;

#pragma unroll
    for (int g = 0; g < RG; g++)
#pragma unroll
      for (int t = 0; t < NT; t++) {
        const int(&a)[4][4] = acc[g][t];
        int v[4];
#pragma unroll
        for (int r = 0; r < 4; r++)
          v[r] = PER_BLOCK ? __float_as_int(yf[t][r])
                   : OFF ? offset_combine(a[0][r], a[1][r], a[2][r], a[3][r])
                         : a[0][r] + a[1][r] + a[2][r] + a[3][r];
        s_acc[16 * g + gq][8 * t + 2 * q] = v[0];
        s_acc[16 * g + gq][8 * t + 2 * q + 1] = v[1];
        s_acc[16 * g + gq + 8][8 * t + 2 * q] = v[2];
        s_acc[16 * g + gq + 8][8 * t + 2 * q + 1] = v[3];
      }
    __syncwarp();
    const uint32_t *Wz = WP + z * w_stride;
    float *Yz = Y + z * y_stride;
    const bool any_flag = __any_sync(0xffffffffu, e_flag != 0);
    const long long e_xsum = OFF ? xl.total(lane) : 0ll;
    const int L = n_limbs((int)seq);
    for (uint32_t k = 0; k * 32u < R * seq; k++) {       // uniform trip count: shuffles
      const uint32_t idx = (uint32_t)lane + 32u * k;
      const uint32_t r = idx % R, s = min(idx / R, 31u);
      const float sc = __shfl_sync(0xffffffffu, e_scale, (int)r);
      const float bi = __shfl_sync(0xffffffffu, e_bias, (int)r);
      const float ri = __shfl_sync(0xffffffffu, e_rinv, (int)s);
      const int fl = __shfl_sync(0xffffffffu, e_flag, (int)s);
      const long long xs2 = OFF ? 2ll * __shfl_sync(0xffffffffu, e_xsum, (int)s) : 0ll;
      const uint32_t o = rbase + r;
      if (idx >= R * seq || o >= out || fl) continue;
      float yv;
      if (PER_BLOCK) {
        yv = limb_total_f(s_acc[r], s, L) * ri;
      } else {
        long long tot = limb_total(s_acc[r], s, L);
        if (OFF)
          tot -= xs2;                            // the offset operands' 2 sum x
        else
          tot >>= 6;                             // the operands carried 64 * t: exact
        yv = ((float)tot * ri) * sc;
      }
      if (BIAS) yv = bi + yv;
      const uint64_t oi = (uint64_t)s * out + o;
      if (oi < limit) Yz[oi] = yv;
    }
    if (any_flag) {
      const float *Xz = X + z * x_stride;
      for (uint32_t r = 0; r < R; r++) {
        const uint32_t o = rbase + r;
        if (o >= out) break;
        float acc8[8];
        const uint32_t *Wrow = Wz + (uint64_t)o * wng;
        for (uint32_t s0 = 0; s0 < seq; s0 += 8) {
          int ns = (int)min(8u, seq - s0);
          ternary_row_generic<8>(Xz, Wrow, PER_BLOCK ? Sz + (uint64_t)o * nblk : nullptr,
                                 PER_BLOCK, PER_BLOCK ? 1.0f : __ldg(Sz + o),
                                 (int)s0, ns, cols, nblk, wng, acc8);
          if (lane == 0) {
            for (int k = 0; k < ns; k++) {
              uint32_t s = s0 + k;
              uint64_t oi = (uint64_t)s * out + o;
              if (P.rowflag[s] && oi < limit)
                Yz[oi] = (BIAS ? __ldg(BIAS + o) : 0.0f) + acc8[k];
            }
          }
        }
      }
    }
    __syncwarp();                 // s_acc is rewritten by the next item
  }
}

// ---------------------------------------------------------------------------
// Fast path, step 2 for few rows: the latency-bound decode GEMV.
// ---------------------------------------------------------------------------
// A CTA takes RT 16-row tiles (RT = 1, 2, 4 or 8, chosen by the launcher so
// the grid is one wave); the kDecWarps / RT warps of a tile split its
// 128-column blocks (warp k of a tile takes blocks k, k + kDecWarps/RT, ...),
// each with the same exact int8 MMAs as the streaming kernels, and the int32
// partial sums are added across the tile's warps in shared memory -- exact,
// so the result does not depend on the split.  Weights go straight to
// registers (the first batch is requested before the programmatic-launch
// wait: weights are not written by the preceding kernel); fragments come
// from L2.
constexpr int kDecWarps = 8;
constexpr uint32_t kDecMaxTiles = 2048;   // above this, the persistent TMA kernel

template <int NT, bool SMW>
__global__ void __launch_bounds__(kDecWarps * 32, 2)
ternary_dec_kernel(const float *__restrict__ X, uint64_t x_stride,
                   const uint32_t *__restrict__ WP, uint64_t w_stride,
                   const float *__restrict__ SCALE, uint64_t s_stride,
                   const float *__restrict__ BIAS, float *__restrict__ Y, uint64_t y_stride,
                   uint32_t seq, uint32_t out, uint32_t cols, uint64_t limit, void *ws,
                   uint32_t tiles, uint32_t count, int rt_log2, PeerOut po, uint32_t wpre) {
  constexpr int KB = NT == 1 ? 4 : (NT <= 4 ? 2 : 1);   // blocks per warp in flight
  extern __shared__ __align__(16) uint2 wsm[];        // [warp][wpre][row A, row B][lane]
  constexpr int CH = NT <= 2 ? 4 : 1;                   // accumulator chains per n-tile
  constexpr bool OFF = CH == 4;                         // a chain per step: offset operands
  constexpr int kMaxRT = NT >= 5 ? 4 : 8;
  __shared__ int red[kDecWarps][NT * 4][32];
  __shared__ int s_acc[kMaxRT][16][8 * NT + 1];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gq = lane >> 2, q = lane & 3;
  const int RT = 1 << rt_log2, wpt = kDecWarps >> rt_log2;   // tiles per CTA, warps per tile
  const int tl = warp / wpt, kw = warp % wpt;
  const uint32_t ct = blockIdx.x * (uint32_t)RT + (uint32_t)tl;   // tile over all problems
  const bool live = ct < tiles * count;
  const uint32_t z = live ? ct / tiles : 0u, rt = live ? ct % tiles : 0u;
  const uint32_t nblk = cols / 128u, wng = cols / 16u;
  const uint32_t rA = min(rt * 16u + (uint32_t)gq, out - 1u);
  const uint32_t rB = min(rt * 16u + (uint32_t)gq + 8u, out - 1u);
  const uint32_t *Wz = WP + z * w_stride;
  // words 2q, 2q+1 of block b of a row: uint2 index 4b + q
  const uint2 *pa = reinterpret_cast<const uint2 *>(Wz + (uint64_t)rA * wng) + q;
  const uint2 *pb = reinterpret_cast<const uint2 *>(Wz + (uint64_t)rB * wng) + q;
  const uint32_t bstep = (uint32_t)wpt, step = (uint32_t)KB * bstep;
  const uint32_t nb = live ? nblk : 0u;

  // SMW: every weight word this warp multiplies (WPRE blocks) is requested
  // into shared memory now -- the weights are not written by the preceding
  // kernel -- by cp.async, each lane reading back only its own copies, so
  // the whole tile streams in while the preceding kernel runs.  Otherwise
  // the first KB blocks go to registers and the rest stream after the wait.
  uint2 *wslot = wsm + (size_t)warp * wpre * 64 + lane;
  if constexpr (SMW) {
    for (uint32_t j = 0; j < wpre; j++) {
      const uint32_t b = (uint32_t)kw + j * bstep;
      const unsigned n = b < nb ? 8u : 0u;
      asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;\n"
                   ::"r"((unsigned)__cvta_generic_to_shared(wslot + j * 64)),
                   "l"(b < nb ? pa + 4u * b : pa), "r"(n) : "memory");
      asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;\n"
                   ::"r"((unsigned)__cvta_generic_to_shared(wslot + j * 64 + 32)),
                   "l"(b < nb ? pb + 4u * b : pb), "r"(n) : "memory");
    }
    asm volatile("cp.async.commit_group;\n" ::: "memory");
  }
  // block b of this warp is slot j = (b - kw) / bstep
  auto wload = [&](uint32_t b, uint32_t j, bool second) -> uint2 {
    if constexpr (SMW) return b < nb ? wslot[j * 64 + (second ? 32 : 0)] : make_uint2(0u, 0u);
    return b < nb ? __ldcs((second ? pb : pa) + 4u * b) : make_uint2(0u, 0u);
  };
  uint2 wa[KB], wb[KB];
  if constexpr (!SMW) {
#pragma unroll
    for (int u = 0; u < KB; u++) {
      const uint32_t b = (uint32_t)kw + (uint32_t)u * bstep;
      wa[u] = wload(b, (uint32_t)u, false);
      wb[u] = wload(b, (uint32_t)u, true);
    }
  }
  // The epilogue's immutable operands, also before the wait.
  const uint32_t erow = min(rt * 16u + (uint32_t)(lane & 15), out - 1u);
  const float e_scale = __ldg(SCALE + z * s_stride + erow);
  const float e_bias = BIAS ? __ldg(BIAS + erow) : 0.0f;
  pdl_wait();                                  // fragments, flags and X come after this
  if constexpr (SMW) {
    asm volatile("cp.async.wait_all;\n" ::: "memory");
#pragma unroll
    for (int u = 0; u < KB; u++) {
      const uint32_t b = (uint32_t)kw + (uint32_t)u * bstep;
      wa[u] = wload(b, (uint32_t)u, false);
      wb[u] = wload(b, (uint32_t)u, true);
    }
  }
  const PrepOut P = prep_at(ws, (int)seq, cols, z);
  const uint2 *fr = P.frag + 2 * lane;
  const float e_rinv = (uint32_t)lane < seq ? __ldcg(P.rowinv + lane) : 0.0f;
  const int e_flag = (uint32_t)lane < seq ? __ldcg(P.rowflag + lane) : 0;
  XsumLanes<NT> xl;
  if (OFF)
    xl.load(P, seq, lane);
  else
    xl.zero();
  const uint32_t xkey = offset_key();

  int acc[NT][CH][4];
#pragma unroll
  for (int t = 0; t < NT; t++)
#pragma unroll
    for (int j = 0; j < CH; j++)
#pragma unroll
      for (int r = 0; r < 4; r++) acc[t][j][r] = 0;

  uint32_t jn = KB;                            // slot of the next iteration's first block
  for (uint32_t b0 = (uint32_t)kw; b0 < nb; b0 += step, jn += KB) {
    uint2 f[KB][NT][4];
#pragma unroll
    for (int u = 0; u < KB; u++) {
      const uint32_t b = b0 + (uint32_t)u * bstep;
#pragma unroll
      for (int t = 0; t < NT; t++) {
        uint4 f01 = make_uint4(0u, 0u, 0u, 0u), f23 = f01;
        if (b < nb) {
          f01 = __ldcg(reinterpret_cast<const uint4 *>(fr + (b * NT + t) * 128u));
          f23 = __ldcg(reinterpret_cast<const uint4 *>(fr + (b * NT + t) * 128u + 64u));
        }
        f[u][t][0] = lo2(f01);
        f[u][t][1] = hi2(f01);
        f[u][t][2] = lo2(f23);
        f[u][t][3] = hi2(f23);
      }
    }
    uint2 na[KB], nb2[KB];
#pragma unroll
    for (int u = 0; u < KB; u++) {
      const uint32_t b = b0 + step + (uint32_t)u * bstep;
      na[u] = wload(b, jn + (uint32_t)u, false);
      nb2[u] = wload(b, jn + (uint32_t)u, true);
    }
#pragma unroll
    for (int u = 0; u < KB; u++) {
      uint32_t A[4][4];
      // words past nblk are zero and so are their fragments: they add 0
      if (OFF)
        unpack_offset(wa[u], wb[u], xkey, A);
      else
        unpack_signed(wa[u], wb[u], A);
#pragma unroll
      for (int t = 0; t < NT; t++)
#pragma unroll
        for (int j = 0; j < 4; j++)
          mma_s8(acc[t][j % CH], A[j][0], A[j][1], A[j][2], A[j][3], f[u][t][j]);
    }
#pragma unroll
    for (int u = 0; u < KB; u++) {
      wa[u] = na[u];
      wb[u] = nb2[u];
    }
  }

  // Exact sum over each tile's warps into the [row][column] layout.
#pragma unroll
  for (int t = 0; t < NT; t++)
#pragma unroll
    for (int r = 0; r < 4; r++) {
      int v = 0;
      if (OFF) {
        v = offset_combine(acc[t][0][r], acc[t][1 % CH][r], acc[t][2 % CH][r], acc[t][3 % CH][r]);
      } else {
#pragma unroll
        for (int j = 0; j < CH; j++) v += acc[t][j][r];
      }
      red[warp][t * 4 + r][lane] = v;
    }
  __syncthreads();
  for (int i = threadIdx.x; i < RT * NT * 4 * 32; i += blockDim.x) {
    const int ti = i / (NT * 4 * 32), rem = i % (NT * 4 * 32);
    const int tr = rem >> 5, ln = rem & 31, t = tr >> 2, r = tr & 3;
    int v = 0;
    for (int w = 0; w < wpt; w++) v += red[ti * wpt + w][tr][ln];
    s_acc[ti][(ln >> 2) + (r >= 2 ? 8 : 0)][8 * t + 2 * (ln & 3) + (r & 1)] = v;
  }
  __syncthreads();

  // Epilogue: warp kw of tile tl covers outputs kw*32 + lane, step wpt*32.
  // With peer outputs every value goes to each rank's slot.
  const unsigned long long tag =
      po.n ? (unsigned long long)(uint32_t)(*po.ep * po.tmul + po.tadd) << 32 : 0ull;
  auto store = [&](uint64_t oi, float v) {
    if (po.n == 0) {
      Y[z * y_stride + oi] = v;
    } else {
      const unsigned long long word = tag | __float_as_uint(v);
#pragma unroll
      for (int r = 0; r < 8; r++)        // constant indices: PeerOut stays in parameter space
        if (r < po.n) po.dst[r][z * y_stride + oi] = word;
    }
  };
  if (live) {
    const bool any_flag = __any_sync(0xffffffffu, e_flag != 0);
    const long long e_xsum = OFF ? xl.total(lane) : 0ll;
    const int L = n_limbs((int)seq);
    for (uint32_t k = (uint32_t)kw; k * 32u < 16u * seq; k += (uint32_t)wpt) {   // warp-uniform
      const uint32_t idx = (uint32_t)lane + 32u * k;
      const uint32_t r = idx & 15u, s = min(idx >> 4, 31u);
      const float sc = __shfl_sync(0xffffffffu, e_scale, (int)r);
      const float bi = __shfl_sync(0xffffffffu, e_bias, (int)r);
      const float ri = __shfl_sync(0xffffffffu, e_rinv, (int)s);
      const int fl = __shfl_sync(0xffffffffu, e_flag, (int)s);
      const long long xs2 = OFF ? 2ll * __shfl_sync(0xffffffffu, e_xsum, (int)s) : 0ll;
      const uint32_t o = rt * 16u + r;
      if (idx >= 16u * seq || o >= out || fl) continue;
      long long tot = limb_total(s_acc[tl][r], s, L);
      if (OFF)
        tot -= xs2;                                // the offset operands' 2 sum x
      else
        tot >>= 6;                                 // the operands carried 64 * t: exact
      float yv = ((float)tot * ri) * sc;
      if (BIAS) yv = bi + yv;
      const uint64_t oi = (uint64_t)s * out + o;
      if (oi < limit) store(oi, yv);
    }
    // Rows the prep flagged (non-finite or unrepresentable) on the CUDA cores.
    if (kw == 0 && any_flag) {
      const float *Xz = X + z * x_stride;
      const float *Sz = SCALE + z * s_stride;
      for (uint32_t r = 0; r < 16u; r++) {
        const uint32_t o = rt * 16u + r;
        if (o >= out) break;
        float acc8[8];
        const uint32_t *Wrow = Wz + (uint64_t)o * wng;
        for (uint32_t s0 = 0; s0 < seq; s0 += 8) {
          const int ns = (int)min(8u, seq - s0);
          ternary_row_generic<8>(Xz, Wrow, nullptr, false, __ldg(Sz + o), (int)s0, ns, cols,
                                 nblk, wng, acc8);
          if (lane == 0) {
            for (int k = 0; k < ns; k++) {
              const uint32_t s = s0 + k;
              const uint64_t oi = (uint64_t)s * out + o;
              if (__ldcg(P.rowflag + s) && oi < limit)
                store(oi, (BIAS ? __ldg(BIAS + o) : 0.0f) + acc8[k]);
            }
          }
        }
      }
    }
  }
}

// Launch the decode GEMV when the problem has few row tiles; false when the
// streaming kernels should run instead.
// Tiles per CTA (log 2) of the decode GEMV: the fewest that keep the grid
// within one wave of the resident CTAs (2 per SM), at least two warps a tile.
int dec_rt_log2(uint32_t total, int NTs) {
  const uint32_t wave = 2u * 148u;
  int lg = 0;
  while (lg < (NTs >= 5 ? 2 : 3) && (total + (1u << lg) - 1) >> lg > wave) lg++;
  return lg;
}

bool try_launch_dec(uint32_t count, const float *X, uint64_t xs, const uint32_t *WP,
                    uint64_t wst, const float *S, uint64_t ss, const float *B, float *Y,
                    uint64_t ys, uint32_t seq, uint32_t out, uint32_t cols, bool per_block,
                    uint64_t limit, void *ws, cudaStream_t st, cudaError_t *err,
                    const PeerOut *po = nullptr) {
  static const int mode = [] {
    const char *v = getenv("NELISP_TERNARY_PATH");
    return v && (strcmp(v, "ring") == 0 || strcmp(v, "tma") == 0) ? 0 : 1;
  }();
  const uint32_t tiles = (out + 15u) / 16u;
  if (!mode || per_block || (uint64_t)tiles * count > kDecMaxTiles) return false;
  const int NTs = n_tiles((int)seq);
  const uint32_t total = tiles * count;
  const int lg = dec_rt_log2(total, NTs);
  const dim3 grid((total + (1u << lg) - 1) >> lg), block(kDecWarps * 32);
  PeerOut pov = {};
  if (po) pov = *po;
  // the weight prefetch into shared memory: blocks per warp, up to 40 KB a CTA
  const uint32_t wpt = (uint32_t)kDecWarps >> lg, nblk = cols / 128u;
  const uint32_t bpw = (nblk + wpt - 1) / wpt;
  const size_t wsmem = (size_t)kDecWarps * bpw * 64 * sizeof(uint2);
  // with two or more n-tiles (batch 8 decode 1.92 -> 1.84 ms), and at one
  // n-tile where more than 6 blocks a warp would leave most of the weights to
  // stream after the wait (batch 1: 1.324 -> 1.315 ms); otherwise the first
  // blocks held in registers measured faster
  const uint32_t wpre = (wsmem <= (40u << 10) && (NTs >= 2 || bpw > 6u)) ? bpw : 0u;
  switch (NTs) {
#define NL_DEC(N)                                                                            \
  case N:                                                                                    \
    {                                                                                      \
      static bool set = false;                                                             \
      if (wpre && !set) {                                                                  \
        *err = cudaFuncSetAttribute(ternary_dec_kernel<N, true>,                           \
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, 40 << 10); \
        if (*err != cudaSuccess) return true;                                              \
        set = true;                                                                        \
      }                                                                                    \
    }                                                                                      \
    if (wpre)                                                                              \
      *err = launch_pdl(ternary_dec_kernel<N, true>, grid, block, wsmem, st, X, xs, WP, wst, S, \
                        ss, B, Y, ys, seq, out, cols, limit, ws, tiles, count, lg, pov, wpre); \
    else                                                                                   \
      *err = launch_pdl(ternary_dec_kernel<N, false>, grid, block, (size_t)0, st, X, xs, WP,  \
                        wst, S, ss, B, Y, ys, seq, out, cols, limit, ws, tiles, count, lg, pov, \
                        0u);                                                                \
    return true;
    NL_DEC(1) NL_DEC(2) NL_DEC(3) NL_DEC(4) NL_DEC(5) NL_DEC(6)
#undef NL_DEC
    default: return false;
  }
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                  const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                  const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_tiled() {
  static EncodeTiledFn fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess && q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
    cudaGetLastError();
  }
  return fn;
}

// The weight rows of all problems as one [rows x wng] u32 tensor, box
// [16*nw rows x 32 words], 128B swizzle.  False when TMA cannot describe it.
bool make_weight_map(CUtensorMap *map, const uint32_t *WP, uint64_t rows, uint32_t wng, int nw) {
  EncodeTiledFn fn = encode_tiled();
  if (!fn || ((uintptr_t)WP & 15u) || (wng * 4u) % 16u || rows == 0) return false;
  cuuint64_t dims[2] = {wng, rows};
  cuuint64_t strides[1] = {(cuuint64_t)wng * 4u};
  cuuint32_t box[2] = {32u, 16u * (uint32_t)nw};
  cuuint32_t estr[2] = {1u, 1u};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<uint32_t *>(WP), dims, strides,
            box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int NT, bool PB>
cudaError_t launch_tma_nt(const CUtensorMap &map, uint32_t items, int nw, cudaStream_t st,
                          const float *X, uint64_t xs, const uint32_t *WP, uint64_t wst,
                          const float *S, uint64_t ss, const float *B, float *Y, uint64_t ys,
                          uint32_t seq, uint32_t out, uint32_t cols, uint64_t limit, void *ws,
                          uint32_t count) {
  static int configured = 0;
  static int per_sm[9] = {0};                  // resident CTAs per SM, by nw
  constexpr int RG = tma_groups(NT, PB);
  size_t smem = tma_smem_bytes(NT, 2, RG);     // the largest CTA this instance runs
  if (tma_smem_bytes(NT, 4, RG) > smem) smem = tma_smem_bytes(NT, 4, RG);
  if (tma_smem_bytes(NT, 8, RG) > smem) smem = tma_smem_bytes(NT, 8, RG);
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(ternary_tma_kernel<NT, PB>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    configured = 1;
  }
  if (!per_sm[nw]) {
    int n = 0;
    cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(
        &n, ternary_tma_kernel<NT, PB>, 32 * (nw + 1), tma_smem_bytes(NT, nw, RG));
    if (e != cudaSuccess) return e;
    per_sm[nw] = n > 0 ? n : 1;
  }
  int sms = 148;
  {
    int dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess)
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    cudaGetLastError();
  }
  const uint32_t cap = (uint32_t)(per_sm[nw] * sms);
  const uint32_t grid = items < cap ? items : cap;
  // The preceding kernel in the stream is always this GEMV's own prep (or a
  // kernel with the prep fused in), launched without the attribute.
  return launch_pdl(ternary_tma_kernel<NT, PB>, dim3(grid), dim3(32 * (nw + 1)),
                    tma_smem_bytes(NT, nw, RG), st, map, X, xs, WP, wst, S, ss, B, Y, ys, seq,
                    out, cols, limit, ws, count, wait_flag_device());
}

// Launch the TMA variant when the weights of all COUNT problems form one
// row-major [count*out x wng] tensor; returns false when it does not apply.
bool try_launch_tma(uint32_t count, const float *X, uint64_t xs, const uint32_t *WP, uint64_t wst,
                    const float *S, uint64_t ss, const float *B, float *Y, uint64_t ys,
                    uint32_t seq, uint32_t out, uint32_t cols, bool per_block, uint64_t limit,
                    void *ws, cudaStream_t st, cudaError_t *err) {
  // NELISP_TERNARY_PATH=ring selects the register-ring kernel instead (and
  // =tma this kernel even where the decode kernel would run).
  static const int use_tma = [] {
    const char *v = getenv("NELISP_TERNARY_PATH");
    return (v && strcmp(v, "ring") == 0) ? 0 : 1;
  }();
  const uint32_t wng = cols / 16u;
  if (!use_tma || (count > 1 && wst != (uint64_t)out * wng)) return false;
  const int NT = n_tiles((int)seq);
  const int rg = tma_groups(NT, per_block);
  // warps of RG 16-row groups; enough items for every resident CTA
  const int groups = ceil_div((int)out, 16 * rg);
  const uint64_t want = rg == 1 ? 2u * 148u : 148u;
  int nw = 8;
  while (nw > 2 && (uint64_t)ceil_div(groups, nw) * count < want) nw >>= 1;
  CUtensorMap map;
  if (!make_weight_map(&map, WP, (uint64_t)count * out, wng, nw * rg)) return false;
  const uint32_t items = (uint32_t)ceil_div(groups, nw) * count;
#define NL_CASE(N)                                                                         \
  case N:                                                                                  \
    *err = per_block ? launch_tma_nt<N, true>(map, items, nw, st, X, xs, WP, wst, S, ss, B, \
                                              Y, ys, seq, out, cols, limit, ws, count)     \
                     : launch_tma_nt<N, false>(map, items, nw, st, X, xs, WP, wst, S, ss,  \
                                               B, Y, ys, seq, out, cols, limit, ws, count); \
    return true;
  switch (NT) {
    NL_CASE(1) NL_CASE(2) NL_CASE(3) NL_CASE(4) NL_CASE(5) NL_CASE(6)
    default: return false;
  }
#undef NL_CASE
}

template <int NT, bool PB>
cudaError_t launch_mma_nt(dim3 grid, int threads, cudaStream_t st, const float *X,
                          uint64_t xs, const uint32_t *WP, uint64_t wst, const float *S,
                          uint64_t ss, const float *B, float *Y, uint64_t ys, uint32_t seq,
                          uint32_t out, uint32_t cols, uint64_t limit, void *ws) {
  static bool configured = false;
  const size_t smem = mma_smem_bytes(NT);
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(ternary_mma_kernel<NT, PB>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    configured = true;
  }
  ternary_mma_kernel<NT, PB><<<grid, threads, smem, st>>>(X, xs, WP, wst, S, ss, B, Y, ys, seq,
                                                          out, cols, limit, ws);
  return cudaPeekAtLastError();
}

template <bool PB>
cudaError_t launch_mma(int NT, dim3 grid, int threads, cudaStream_t st, const float *X,
                       uint64_t xs, const uint32_t *WP, uint64_t wst, const float *S,
                       uint64_t ss, const float *B, float *Y, uint64_t ys, uint32_t seq,
                       uint32_t out, uint32_t cols, uint64_t limit, void *ws) {
#define NL_CASE(N)                                                                  \
  case N:                                                                           \
    return launch_mma_nt<N, PB>(grid, threads, st, X, xs, WP, wst, S, ss, B, Y, ys, \
                                seq, out, cols, limit, ws);
  switch (NT) {
    NL_CASE(1) NL_CASE(2) NL_CASE(3) NL_CASE(4) NL_CASE(5) NL_CASE(6)
    default: return cudaErrorInvalidValue;
  }
#undef NL_CASE
}

}  // namespace

bool ternary_fast_shape(uint32_t cols, uint32_t nblk, uint32_t wng,
                        bool per_block) {
  if (cols == 0 || cols % 128u != 0) return false;
  if (wng != cols / 16u) return false;
  if (per_block && nblk != cols / 128u) return false;
  return true;
}

uint32_t ternary_dec_ctas(uint32_t count, uint32_t out, uint32_t cols, uint32_t seq) {
  const uint32_t tiles = (out + 15u) / 16u, total = tiles * count;
  if (seq == 0 || seq > (uint32_t)kMaxFastSeq || total > kDecMaxTiles || cols % 128u) return 0;
  const int lg = dec_rt_log2(total, n_tiles((int)seq));
  return (total + (1u << lg) - 1) >> lg;
}

size_t ternary_ws_bytes_best(uint32_t count, uint32_t seq, uint32_t cols, bool per_block) {
  size_t b = ternary_ws_bytes(count, seq, cols);
  if (ternary_tc_applies(1, seq, 1, cols, per_block, 0)) {   // the shapes the tcgen05 GEMV takes
    const size_t t = ternary_tc_ws_bytes(count, seq, cols);
    if (t > b) b = t;
  }
  if (ternary_umma_applies(count, seq, cols, per_block)) {
    const size_t u = ternary_umma_ws_bytes(seq, cols);
    if (u > b) b = u;
  }
  return b;
}

size_t ternary_ws_bytes(uint32_t count, uint32_t seq, uint32_t cols) {
  int s = (int)(seq < (uint32_t)kMaxFastSeq ? seq : (uint32_t)kMaxFastSeq);
  if (s < 1) s = 1;
  return (size_t)count * prep_bytes(s, cols);
}

cudaError_t ternary_gemv_launch(uint32_t count, const float *X,
                                uint64_t x_stride, const uint32_t *WP,
                                uint64_t w_stride, const float *SCALE,
                                uint64_t s_stride, const float *BIAS,
                                float *Y, uint64_t y_stride, uint32_t seq,
                                uint32_t out, uint32_t cols, uint32_t nblk,
                                uint32_t wng, bool per_block, uint64_t limit,
                                void *ws, size_t ws_bytes,
                                cudaStream_t stream) {
  if (count == 0 || seq == 0 || out == 0) return cudaSuccess;
  bool fast = ternary_fast_shape(cols, nblk, wng, per_block) && ws != nullptr &&
              ws_bytes >= ternary_ws_bytes(count, seq, cols) &&
              aligned16(X) && (x_stride % 4u) == 0 && (w_stride % 2u) == 0 &&
              ((uintptr_t)WP & 7u) == 0;
  if (!fast) {
    dim3 grid(ceil_div((int)out, 8), count);
    ternary_generic_kernel<<<grid, 256, 0, stream>>>(
        X, x_stride, WP, w_stride, SCALE, s_stride, BIAS, Y, y_stride, seq,
        out, cols, nblk, wng, per_block ? 1 : 0, limit);
    count_launches(1);
    return cudaPeekAtLastError();
  }
  // Streaming shapes (more 16-row tiles than the decode kernel takes): the
  // tcgen05 GEMV with the weights expanded into tensor memory.
  if (ternary_tc_applies(count, seq, out, cols, per_block, w_stride) &&
      ternary_dec_ctas(count, out, cols, seq) == 0) {
    bool launched = false;
    cudaError_t e = ternary_tc_launch(count, X, x_stride, WP, w_stride, SCALE, s_stride, BIAS, Y,
                                      y_stride, seq, out, cols, limit, ws, ws_bytes, stream,
                                      &launched);
    if (launched || e != cudaSuccess) return e;
  }
  // Many sequence rows of one problem: the tcgen05 GEMM, when the workspace
  // holds its int8 limb matrix.
  static const bool umma_on = [] {
    const char *v = getenv("NELISP_TERNARY_PATH");   // ring / tma: the chunked kernels
    return !(v && (strcmp(v, "ring") == 0 || strcmp(v, "tma") == 0));
  }();
  if (umma_on && seq > (uint32_t)kMaxFastSeq && limit == UINT64_MAX &&
      ternary_umma_applies(count, seq, cols, per_block)) {
    bool launched = false;
    cudaError_t e = ternary_umma_launch(X, WP, SCALE, BIAS, Y, seq, out, cols, ws, ws_bytes,
                                        stream, &launched);
    if (launched || e != cudaSuccess) return e;
  }
  // Sequences in chunks of 16 (one prep + one main launch per chunk); the
  // workspace is reused chunk to chunk, ordered by the stream.  Past 16 rows
  // no chunk is left with four rows or fewer (the last two share the rest
  // evenly): every row then gets the three-limb precision that the tcgen05
  // GEMM gives such calls, whichever kernel runs.
  for (uint32_t s0 = 0, ns = 0; s0 < seq; s0 += ns) {
    ns = min((uint32_t)kMaxFastSeq, seq - s0);
    if (seq > (uint32_t)kMaxFastSeq && seq - s0 > ns && seq - s0 - ns <= 4u)
      ns = (seq - s0 + 1u) / 2u;
    int NT = n_tiles((int)ns);
    // Programmatic launch: the prep's blocks become resident while the
    // preceding kernel drains and wait (griddepcontrol.wait) before they
    // read X or write the workspace.
    cudaError_t e = launch_prep_any(X + (uint64_t)s0 * cols, x_stride, count, ns, cols, ws,
                                    stream, true);
    if (e == cudaSuccess) e = cudaPeekAtLastError();
    if (e != cudaSuccess) return e;
    {
      // The short-grid limit is an index into the whole Y; shift it per chunk.
      uint64_t b0 = (uint64_t)s0 * out;
      uint64_t l0 = limit > b0 ? limit - b0 : 0;
      if (try_launch_dec(count, X + (uint64_t)s0 * cols, x_stride, WP, w_stride, SCALE,
                         s_stride, BIAS, Y + (uint64_t)s0 * out, y_stride, ns, out, cols,
                         per_block, l0, ws, stream, &e) ||
          try_launch_tma(count, X + (uint64_t)s0 * cols, x_stride, WP, w_stride, SCALE,
                         s_stride, BIAS, Y + (uint64_t)s0 * out, y_stride, ns, out, cols,
                         per_block, l0, ws, stream, &e)) {
        count_launches(2);
        if (e != cudaSuccess) return e;
        continue;
      }
    }
    // Warps per CTA: as many as keep the grid at two or more CTAs per SM.
    const int groups16 = ceil_div((int)out, 16);
    int nw = 8;
    while (nw > 2 && (uint64_t)ceil_div(groups16, nw) * count < 2u * 148u) nw >>= 1;
    dim3 grid(ceil_div(groups16, nw), count);
    // The short-grid limit is an index into the whole Y; shift it per chunk.
    uint64_t base = (uint64_t)s0 * out;
    uint64_t lim = limit > base ? limit - base : 0;
    if (per_block)
      e = launch_mma<true>(NT, grid, nw * 32, stream, X + (uint64_t)s0 * cols, x_stride,
                           WP, w_stride, SCALE, s_stride, BIAS,
                           Y + (uint64_t)s0 * out, y_stride, ns, out, cols, lim, ws);
    else
      e = launch_mma<false>(NT, grid, nw * 32, stream, X + (uint64_t)s0 * cols, x_stride,
                            WP, w_stride, SCALE, s_stride, BIAS,
                            Y + (uint64_t)s0 * out, y_stride, ns, out, cols, lim, ws);
    count_launches(2);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

cudaError_t ternary_prep_launch(const float *X, uint64_t x_stride, uint32_t count,
                                uint32_t seq, uint32_t cols, void *ws, cudaStream_t stream,
                                bool pdl) {
  if (count == 0 || seq == 0) return cudaSuccess;
  cudaError_t e = launch_prep_any(X, x_stride, count, seq, cols, ws, stream, pdl);
  count_launches(1);
  return e != cudaSuccess ? e : cudaPeekAtLastError();
}

cudaError_t ternary_main_launch(uint32_t count, const float *X, uint64_t x_stride,
                                const uint32_t *WP, uint64_t w_stride, const float *SCALE,
                                uint64_t s_stride, const float *BIAS, float *Y,
                                uint64_t y_stride, uint32_t seq, uint32_t out, uint32_t cols,
                                bool per_block, void *ws, cudaStream_t stream,
                                const PeerOut *po) {
  if (count == 0 || seq == 0 || out == 0) return cudaSuccess;
  const uint32_t nblk = (cols + 127) / 128, wng = (cols + 15) / 16;
  if (po && po->n) {
    // Peer outputs exist only on the decode kernel.
    cudaError_t e = cudaErrorNotSupported;
    if (ws && seq <= (uint32_t)kMaxFastSeq && ternary_fast_shape(cols, nblk, wng, per_block) &&
        try_launch_dec(count, X, x_stride, WP, w_stride, SCALE, s_stride, BIAS, Y, y_stride, seq,
                       out, cols, per_block, UINT64_MAX, ws, stream, &e, po)) {
      count_launches(1);
      return e;
    }
    return cudaErrorNotSupported;
  }
  if (!ws || seq > (uint32_t)kMaxFastSeq || !ternary_fast_shape(cols, nblk, wng, per_block)) {
    dim3 grid(ceil_div((int)out, 8), count);
    ternary_generic_kernel<<<grid, 256, 0, stream>>>(X, x_stride, WP, w_stride, SCALE, s_stride,
                                                     BIAS, Y, y_stride, seq, out, cols, nblk,
                                                     wng, per_block ? 1 : 0, UINT64_MAX);
    count_launches(1);
    return cudaPeekAtLastError();
  }
  cudaError_t e;
  if (try_launch_dec(count, X, x_stride, WP, w_stride, SCALE, s_stride, BIAS, Y, y_stride, seq,
                     out, cols, per_block, UINT64_MAX, ws, stream, &e) ||
      try_launch_tma(count, X, x_stride, WP, w_stride, SCALE, s_stride, BIAS, Y, y_stride, seq,
                     out, cols, per_block, UINT64_MAX, ws, stream, &e)) {
    count_launches(1);
    return e;
  }
  const int groups16 = ceil_div((int)out, 16);
  int nw = 8;
  while (nw > 2 && (uint64_t)ceil_div(groups16, nw) * count < 2u * 148u) nw >>= 1;
  dim3 grid(ceil_div(groups16, nw), count);
  e = per_block ? launch_mma<true>(n_tiles((int)seq), grid, nw * 32, stream, X, x_stride, WP,
                                   w_stride, SCALE, s_stride, BIAS, Y, y_stride, seq, out, cols,
                                   UINT64_MAX, ws)
                : launch_mma<false>(n_tiles((int)seq), grid, nw * 32, stream, X, x_stride, WP,
                                    w_stride, SCALE, s_stride, BIAS, Y, y_stride, seq, out, cols,
                                    UINT64_MAX, ws);
  count_launches(1);
  return e;
}

// ---------------------------------------------------------------------------
// ternary-rows-t (kernels.el:750-772): one thread per (column i), all
// sequence rows, summing over o in the reference's order.
// ---------------------------------------------------------------------------
namespace {
__global__ void ternary_rows_t_kernel(const uint32_t *__restrict__ WP,
                                      const float *__restrict__ BETA,
                                      const float *__restrict__ G,
                                      float *__restrict__ Xo, uint32_t out,
                                      uint32_t cols, uint32_t nblk,
                                      uint32_t wng, uint32_t seq,
                                      uint64_t limit) {
  uint64_t idx = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (uint64_t)seq * cols || idx >= limit) return;
  uint32_t p = (uint32_t)(idx / cols), i = (uint32_t)(idx % cols);
  uint32_t b = i / 128u, wi = i / 16u, fd = i % 16u;
  uint32_t gb = p * out;
  float acc = 0.0f;
  for (uint32_t o = 0; o < out; o++) {
    float sv = trit_of(__ldg(WP + (uint64_t)o * wng + wi), fd);
    float bg = __fmul_rn(__ldg(BETA + (uint64_t)o * nblk + b), __ldg(G + gb + o));
    acc = __fadd_rn(acc, __fmul_rn(sv, bg));
  }
  Xo[idx] = acc;
}

// bitlinear-packed(-v) (kernels.el:998-1040): one warp per output; lanes
// take packed floats, reduced across the warp.
__global__ void bitlinear_packed_kernel(const float *__restrict__ X,
                                        const float *__restrict__ WPK,
                                        const float *__restrict__ BIAS,
                                        const float *__restrict__ BETA,
                                        float *__restrict__ Y, uint32_t seq,
                                        uint32_t in, uint32_t out, uint32_t pk,
                                        uint32_t fcount, int per_row,
                                        uint64_t limit) {
  uint64_t wid = ((uint64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  int lane = threadIdx.x & 31;
  if (wid >= (uint64_t)seq * out || wid >= limit) return;
  uint32_t s = (uint32_t)(wid / out), o = (uint32_t)(wid % out);
  float beta = per_row ? __ldg(BETA + o) : __ldg(BETA);
  const float *xr = X + (uint64_t)s * in;
  float acc = 0.0f;
  for (uint32_t f = lane; f < fcount; f += 32) {
    float pf = __ldg(WPK + (uint64_t)o * fcount + f);
    uint32_t packed = __float2uint_rz(pf);
    uint32_t i0 = f * pk;
    for (uint32_t zz = 0; zz < pk; zz++) {
      uint32_t i = i0 + zz;
      if (i < in) {
        float tern = (float)(packed % 4u) - 1.0f;
        acc = fmaf(__ldg(xr + i), __fmul_rn(beta, tern), acc);
      }
      packed /= 4u;
    }
  }
  for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  if (lane == 0) Y[wid] = __ldg(BIAS + o) + acc;
}

// ---- registry glue ------------------------------------------------------

const char *chk_ternary_rows(const OpArgs &a) {
  // (X WP BIAS BETA Y) push (seq out cols nblk wng)
  uint64_t seq = a.push[0], out = a.push[1], cols = a.push[2], nblk = a.push[3], wng = a.push[4];
  const char *m;
  if ((m = need_words(a, 0, seq * cols, "X"))) return m;
  if ((m = need_words(a, 1, out * wng, "WP"))) return m;
  if ((m = need_words(a, 2, out, "BIAS"))) return m;
  if ((m = need_words(a, 3, out * nblk, "BETA"))) return m;
  if ((m = need_words(a, 4, seq * out, "Y"))) return m;
  if (wng * 16 < cols && wng < 8 * nblk)
    return fmt_msg("ternary-rows: cols %llu needs %llu words per row, wng is %llu",
                   (unsigned long long)cols, (unsigned long long)((cols + 15) / 16),
                   (unsigned long long)wng);
  return nullptr;
}
size_t scr_ternary_rows(const OpArgs &a) {
  return ternary_fast_shape(a.push[2], a.push[3], a.push[4], true)
             ? ternary_ws_bytes(1, a.push[0], a.push[2])
             : 0;
}
cudaError_t run_ternary_rows(const OpArgs &a) {
  return ternary_gemv_launch(1, (const float *)a.buf[0], 0,
                             (const uint32_t *)a.buf[1], 0,
                             (const float *)a.buf[3], 0,
                             (const float *)a.buf[2], (float *)a.buf[4], 0,
                             a.push[0], a.push[1], a.push[2], a.push[3],
                             a.push[4], true, invocations(a.groups, 64),
                             a.scratch, a.scratch_bytes, a.stream);
}

const char *chk_ternary_rows_t(const OpArgs &a) {
  // (WP BETA G X) push (out cols nblk wng seq)
  uint64_t out = a.push[0], cols = a.push[1], nblk = a.push[2], wng = a.push[3], seq = a.push[4];
  const char *m;
  if (cols && ((cols - 1) / 16) >= wng)
    return fmt_msg("ternary-rows-t: column %llu is past word %llu of a row",
                   (unsigned long long)(cols - 1), (unsigned long long)wng);
  if (cols && ((cols - 1) / 128) >= nblk && out)
    return fmt_msg("ternary-rows-t: column %llu is past block %llu",
                   (unsigned long long)(cols - 1), (unsigned long long)nblk);
  if ((m = need_words(a, 0, out * wng, "WP"))) return m;
  if ((m = need_words(a, 1, out * nblk, "BETA"))) return m;
  if ((m = need_words(a, 2, seq * out, "G"))) return m;
  if ((m = need_words(a, 3, seq * cols, "X"))) return m;
  return nullptr;
}
cudaError_t run_ternary_rows_t(const OpArgs &a) {
  uint64_t n = (uint64_t)a.push[4] * a.push[1];
  if (n == 0) return cudaSuccess;
  ternary_rows_t_kernel<<<(unsigned)ceil_div64(n, 128), 128, 0, a.stream>>>(
      (const uint32_t *)a.buf[0], (const float *)a.buf[1],
      (const float *)a.buf[2], (float *)a.buf[3], a.push[0], a.push[1],
      a.push[2], a.push[3], a.push[4], invocations(a.groups, 64));
  count_launches(1);
  return cudaPeekAtLastError();
}

template <int PER_ROW>
const char *chk_bitlinear_packed(const OpArgs &a) {
  // (X WPK BIAS BETA Y) push (seq in out pk fcount); X is read at s*in + i
  // for i < min(in, fcount*pk).
  uint64_t seq = a.push[0], in = a.push[1], out = a.push[2], fcount = a.push[4];
  uint64_t used = fcount * a.push[3] < in ? fcount * a.push[3] : in;
  uint64_t xneed = (seq && out && used) ? (seq - 1) * in + used : 0;
  const char *m;
  if ((m = need_words(a, 0, xneed, "X"))) return m;
  if ((m = need_words(a, 1, out * fcount, "WPK"))) return m;
  if ((m = need_words(a, 2, out, "BIAS"))) return m;
  if ((m = need_words(a, 3, PER_ROW ? out : (seq && out ? 1 : 0), "BETA"))) return m;
  if ((m = need_words(a, 4, seq * out, "Y"))) return m;
  return nullptr;
}
template <int PER_ROW>
cudaError_t run_bitlinear_packed(const OpArgs &a) {
  uint64_t n = (uint64_t)a.push[0] * a.push[2];
  if (n == 0) return cudaSuccess;
  bitlinear_packed_kernel<<<(unsigned)ceil_div64(n * 32, 256), 256, 0, a.stream>>>(
      (const float *)a.buf[0], (const float *)a.buf[1],
      (const float *)a.buf[2], (const float *)a.buf[3], (float *)a.buf[4],
      a.push[0], a.push[1], a.push[2], a.push[3], a.push[4], PER_ROW,
      invocations(a.groups, 64));
  count_launches(1);
  return cudaPeekAtLastError();
}

size_t no_scratch(const OpArgs &) { return 0; }

}  // namespace

const OpSpec kTernaryOps[] = {
    {"ternary-rows", 5, 5, chk_ternary_rows, scr_ternary_rows, run_ternary_rows},
    {"ternary-rows-t", 4, 5, chk_ternary_rows_t, no_scratch, run_ternary_rows_t},
    {"bitlinear-packed", 5, 5, chk_bitlinear_packed<0>, no_scratch, run_bitlinear_packed<0>},
    {"bitlinear-packed-v", 5, 5, chk_bitlinear_packed<1>, no_scratch, run_bitlinear_packed<1>},
};
const int kTernaryOpsCount = sizeof(kTernaryOps) / sizeof(kTernaryOps[0]);

}  // namespace nl

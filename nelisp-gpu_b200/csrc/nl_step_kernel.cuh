// nl_step_kernel.cuh -- the step kernel of nl_step.cu: all layers of one
// decode step of the ternary decoder in one persistent, cooperative kernel.
// Included by nl_step_h128.cu and nl_step_h64.cu, one head size each (the
// instantiations compile in parallel).
//
// A decode step at batch 1..8 moves about 20 MB of packed weights and a few
// MB of KV cache per layer: each of the nine kernels a layer takes as
// separate launches is too small to reach HBM bandwidth, and the step was a
// chain of latency-bound launches.  Here one grid of one CTA per SM runs the
// whole step:
//
//  * a producer warp streams every weight tile the CTA will need, in the
//    order it will need them, through a ring of shared-memory stages
//    (cp.async.bulk, one copy per row into rows padded for conflict-free
//    operand loads, completing on the stage's mbarrier).  Weights do not
//    depend on the activations, so the ring runs ahead across phase
//    boundaries: when a phase starts, its first tiles are already on chip;
//  * eight compute warps walk the phases of each layer, separated by grid
//    barriers (a counter in global memory, bounded waits):
//      Q  RMSNorm of the residual row (gathered from the embedding at layer
//         0), its activation prep, the Q|K|V GEMV;
//      A  RoPE, cache append and split-K attention (the decoder's fused
//         attention); the last split of a head merges the partials;
//      O  prep of the context rows, the O GEMV;
//      G  residual add, RMSNorm, prep, the gate|up GEMV with SwiGLU in its
//         epilogue (the gate and up rows of the same columns in one task)
//         and the row maximum of the result (atomicMax);
//      D  prep of this CTA's column chunk of the SwiGLU row, the down GEMV
//         split along K into exact int64 partial sums per chunk;
//    after the last layer CTA 0 forms the final normalised rows for the LM
//    head, which runs as the next (bandwidth-bound) launch;
//  * every CTA prepares the activation rows it multiplies itself, in shared
//    memory (the int8 limbs and scales of the GEMV's prep kernels), so no
//    phase needs a prep launch or an extra barrier.
//
// The GEMV arithmetic (exact int8 limb MMAs, int32 / int64 sums, the
// epilogue's f32 operations), the attention (split geometry, fold order,
// merge) and the SwiGLU are those of the separate kernels, so those results
// are the same bits; the RMSNorm sum of squares is reduced in a different
// (fixed) order.  Rows whose activations are non-finite (or whose scale
// leaves the f32 normals) give NaN outputs here, where the separate kernels
// recompute them with the reference's CUDA-core arithmetic.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include "nl_internal.h"
#include "nl_step.h"
#include "ternary_mma.cuh"
#include "ternary_prep.cuh"

namespace nl {
namespace {

constexpr int kCW = 8;                    // compute warps
constexpr int kCT = kCW * 32;             // compute threads
constexpr int kThreads = kCT + 32;        // and the producer warp
constexpr uint32_t kSuspendNs = 200000;   // a try_wait suspends at most this long
constexpr uint64_t kWaitNs = 1000000000ull;   // any wait gives up after one second
constexpr int kAW = 4;                    // warps per attention task (half a CTA)
constexpr uint32_t kNaN = 0x7fc00000u;

// ---- synchronisation ------------------------------------------------------------
__device__ __forceinline__ uint32_t sa(const void *p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}
// The compute warps only (the producer never joins).
__device__ __forceinline__ void csync() { asm volatile("bar.sync 1, 256;\n" ::: "memory"); }
// One half of the compute warps (an attention task).
__device__ __forceinline__ void hsync(int h) {
  asm volatile("bar.sync %0, 128;\n" ::"r"(2 + h) : "memory");
}
__device__ __forceinline__ void mb_init(uint64_t *b, uint32_t n) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(sa(b)), "r"(n));
}
__device__ __forceinline__ void mb_expect(uint64_t *b, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(sa(b)),
               "r"(bytes) : "memory");
}
__device__ __forceinline__ void mb_arrive(uint64_t *b) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(sa(b)) : "memory");
}
__device__ __forceinline__ uint64_t gtime() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;\n" : "=l"(t));
  return t;
}
__device__ __forceinline__ bool mb_try(uint32_t a, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(done) : "r"(a), "r"(parity), "r"(kSuspendNs) : "memory");
  return done != 0;
}
// Bounded wait for the phase of parity PARITY: each try_wait suspends in
// hardware until the phase completes or kSuspendNs pass.  Off the fast path
// the wait gives up at once if a wait anywhere in the grid already gave up
// (ERR set), else after kWaitNs, and records it in ERR.
__device__ __forceinline__ bool mb_wait(uint64_t *b, uint32_t parity, int *err) {
  const uint32_t a = sa(b);
  if (mb_try(a, parity)) return true;
  const uint64_t t0 = gtime();
  while (!*reinterpret_cast<volatile int *>(err)) {
    if (mb_try(a, parity)) return true;
    if (gtime() - t0 > kWaitNs) {
      report_wait_timeout(err);
      return false;
    }
  }
  return false;
}
__device__ __forceinline__ void bulk_row(uint32_t dst, const void *src, uint32_t bytes,
                                         uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n"
      ::"r"(dst), "l"(src), "r"(bytes), "r"(sa(bar)) : "memory");
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
__device__ __forceinline__ unsigned long long ld_acquire_gpu(const unsigned long long *p) {
  unsigned long long v;
  asm volatile("ld.acquire.gpu.global.u64 %0, [%1];\n" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// Grid barrier of the compute warps: every CTA's writes before it are
// visible to every CTA after it (data other CTAs wrote in this launch is
// read with L1-bypassing loads).  Bounded: a wait that gives up sets ERR and
// later barriers no longer wait (the step's outputs are then invalid and
// the host reports it).
__device__ __forceinline__ void grid_sync(unsigned long long *bar, unsigned long long target,
                                          int *err) {
  csync();
  if (threadIdx.x == 0) {
    __threadfence();
    asm volatile("red.relaxed.gpu.global.add.u64 [%0], 1;\n" ::"l"(bar) : "memory");
    const uint64_t t0 = gtime();
    for (uint32_t i = 1; ld_acquire_gpu(bar) < target; i++) {
      if ((i & 63u) == 0u) {           // now and then: a wait elsewhere gave up, or time is out
        if (*reinterpret_cast<volatile int *>(err)) break;
        if (gtime() - t0 > kWaitNs) {
          report_wait_timeout(err);
          break;
        }
      }
    }
    __threadfence();
  }
  csync();
}

// ---- the work of one step ----------------------------------------------------------
// A balanced share [lo, hi) of N items for part I of PARTS.
struct Range {
  uint32_t lo, hi;
};
__device__ __forceinline__ Range share(uint32_t n, uint32_t parts, uint32_t i) {
  return {(uint32_t)((uint64_t)n * i / parts), (uint32_t)((uint64_t)n * (i + 1) / parts)};
}

// One weight stage: 16 rows of W (row stride WNG words) from row ROW0, words
// [W0, W0 + NBW) of each, into a ring stage (row stride NBW + pad words).
struct StageSrc {
  const uint32_t *W;
  uint32_t row0, wng, w0, nbw;
};

struct Ring {
  uint64_t *full, *empty;
  uint32_t base, nst;
  uint32_t it;   // stages consumed (or produced) so far
  __device__ __forceinline__ uint32_t slot() const { return it % nst; }
  __device__ __forceinline__ uint32_t parity() const { return (it / nst) & 1u; }
  __device__ __forceinline__ uint32_t addr() const { return base + slot() * kStepStageBytes; }
};

// Producer: issue one stage, lanes 0..15 one row each.
__device__ __forceinline__ void produce(Ring &r, const StageSrc &s, int lane, int *err) {
  const uint32_t slot = r.slot();
  if (lane == 0) {
    mb_wait(&r.empty[slot], r.parity() ^ 1u, err);
    mb_expect(&r.full[slot], 16u * s.nbw * 4u);
  }
  __syncwarp();
  if (lane < 16) {
    const uint32_t dst = r.addr() + (uint32_t)lane * (s.nbw + kStepRowPad) * 4u;
    bulk_row(dst, s.W + (uint64_t)(s.row0 + (uint32_t)lane) * s.wng + s.w0, s.nbw * 4u,
             &r.full[slot]);
  }
  r.it++;
}

template <int NT>
struct TileT {
  static constexpr int CH = NT <= 2 ? 4 : 1;   // accumulator chains per n-tile
  static constexpr bool OFF = CH == 4;         // one-LOP3 offset operands
};

// Consumer: this warp's 128-column blocks (warp, warp + 8, ...) of the stage
// against the staged fragments (the decode GEMV's MMA sequence); the stage
// is released when every warp is done with it.
template <int NT>
__device__ __forceinline__ void consume(Ring &r, uint32_t nbw, uint32_t frag, int warp, int lane,
                                       uint32_t xkey, int (&acc)[NT][TileT<NT>::CH][4],
                                       int *err) {
  constexpr int CH = TileT<NT>::CH;
  const uint32_t slot = r.slot();
  mb_wait(&r.full[slot], r.parity(), err);
  const uint32_t stride = nbw + kStepRowPad;
  const int gq = lane >> 2, q = lane & 3;
  const uint32_t ra = r.addr() + ((uint32_t)gq * stride + 2u * (uint32_t)q) * 4u;
  const uint32_t rb = ra + 8u * stride * 4u;
  const uint32_t nb = nbw / 8u;
  for (uint32_t b = (uint32_t)warp; b < nb; b += kCW) {
    const uint2 wa = lds64(ra + b * 32u), wb = lds64(rb + b * 32u);
    uint32_t A[4][4];
    if (TileT<NT>::OFF)
      unpack_offset(wa, wb, xkey, A);
    else
      unpack_signed(wa, wb, A);
#pragma unroll
    for (int t = 0; t < NT; t++) {
      const uint32_t fa = frag + (((b * NT + (uint32_t)t) * 2u) * 32u + (uint32_t)lane) * 16u;
      const uint4 f01 = lds128(fa), f23 = lds128(fa + 32u * 16u);
      mma_s8(acc[t][0 % CH], A[0][0], A[0][1], A[0][2], A[0][3], lo2(f01));
      mma_s8(acc[t][1 % CH], A[1][0], A[1][1], A[1][2], A[1][3], hi2(f01));
      mma_s8(acc[t][2 % CH], A[2][0], A[2][1], A[2][2], A[2][3], lo2(f23));
      mma_s8(acc[t][3 % CH], A[3][0], A[3][1], A[3][2], A[3][3], hi2(f23));
    }
  }
  __syncwarp();
  if (lane == 0) mb_arrive(&r.empty[slot]);
  r.it++;
}

// One tile: the stage's MMAs, then the exact sum of the eight warps'
// partials into SACC[16][8 NT + 1] (row, n = 3 s + limb) as the decode GEMV
// lays it out.
template <int NT>
__device__ __forceinline__ void tile(Ring &r, uint32_t nbw, uint32_t frag, int warp, int lane,
                                     uint32_t xkey, int *red, int *sacc, int *err) {
  constexpr int CH = TileT<NT>::CH;
  int acc[NT][CH][4];
#pragma unroll
  for (int t = 0; t < NT; t++)
#pragma unroll
    for (int j = 0; j < CH; j++)
#pragma unroll
      for (int k = 0; k < 4; k++) acc[t][j][k] = 0;
  consume<NT>(r, nbw, frag, warp, lane, xkey, acc, err);
#pragma unroll
  for (int t = 0; t < NT; t++)
#pragma unroll
    for (int k = 0; k < 4; k++) {
      int v;
      if (TileT<NT>::OFF)
        v = offset_combine(acc[t][0][k], acc[t][1 % CH][k], acc[t][2 % CH][k], acc[t][3 % CH][k]);
      else
        v = acc[t][0][k];
      red[((warp * NT + t) * 4 + k) * 32 + lane] = v;
    }
  csync();
  for (int i = (int)threadIdx.x; i < NT * 4 * 32; i += kCT) {
    const int tr = i >> 5, ln = i & 31, t = tr >> 2, k = tr & 3;
    int v = 0;
#pragma unroll
    for (int w = 0; w < kCW; w++) v += red[(w * NT * 4 + tr) * 32 + ln];
    sacc[((ln >> 2) + (k >= 2 ? 8 : 0)) * (8 * NT + 1) + 8 * t + 2 * (ln & 3) + (k & 1)] = v;
  }
  csync();
}

// Row statistics of the prep, per sequence row.
struct RowStat {
  float rinv[kStepMaxB];     // RMSNorm's 1/rms
  float mul[kStepMaxB];      // 2^e of the quantisation
  float inv[kStepMaxB];      // 2^-e
  int flag[kStepMaxB];       // not representable: NaN outputs
  long long xs[kStepMaxB];   // sum of xq over fields 0..2
  float dinv[kStepMaxB];     // the previous down GEMV's 2^-e
  int dflag[kStepMaxB];      // ... and its flag
};

// Exact integer dot product of tile row R, sequence row S, from SACC.
template <int NT>
__device__ __forceinline__ long long tile_tot(const int *sacc, int r, int s, long long xs, int L) {
  const int *row = sacc + r * (8 * NT + 1) + L * s;
  long long tot = (long long)row[0] + 256ll * row[1] + 65536ll * row[2];
  if (L == 4) tot += 16777216ll * row[3];
  if (TileT<NT>::OFF)
    tot -= 2ll * xs;                 // the offset operands' 2 sum xq
  else
    tot >>= 6;                       // the signed operands carried 64 t
  return tot;
}

// The scale of the rows a down GEMV ran with: from the SwiGLU row maximum.
__device__ __forceinline__ void given_scale(float mm, int L, float *mul, float *inv, int *flag) {
  float m, i;
  const bool ok = row_scale(mm, !isfinite(mm), &m, &i, L);
  *mul = m;
  *inv = i;
  *flag = !ok;
}

// The prep of B activation rows of K columns in this CTA, into shared
// memory.  LOAD(b, W, v) gives the 16 values of packed word W of row b,
// which are staged in XS ([B][K] floats).  NORM: x = (v * rinv) * G, rinv
// from the row's sum of squares (per-word partials, then a fixed order per
// row); then the row maximum, its power-of-two scale and the int8 limbs of
// every value (quantize_word, the prep kernels' format) into FRAG.  GIVEN:
// the scale comes from MAXB[b] (float bits of the row maximum).  HDST (may
// be null): v is stored there too.
enum { kPrepPlain = 0, kPrepNorm = 1, kPrepGiven = 2 };
template <int MODE, int NT, class Load>
__device__ __forceinline__ void prep_rows(const Load &load, uint32_t B, uint32_t K,
                                          const float *G, float eps, const unsigned *maxb,
                                          float *hdst, void *frag, float *xs, float *pss,
                                          float *pmx, int *pbad, RowStat *st, int warp,
                                          int lane) {
  const uint32_t nw = K / 16u, n = B * nw;
  const int tid = (int)threadIdx.x;
#pragma unroll 1
  for (uint32_t k = (uint32_t)tid; k < n; k += kCT) {
    const uint32_t b = k / nw, W = k % nw;
    float v[16];
    load(b, W, v);
    float4 *x4 = reinterpret_cast<float4 *>(xs + (size_t)b * K + 16u * W);
#pragma unroll
    for (int e = 0; e < 4; e++)
      x4[e] = make_float4(v[4 * e], v[4 * e + 1], v[4 * e + 2], v[4 * e + 3]);
    if (hdst) {
      float4 *d4 = reinterpret_cast<float4 *>(hdst + (size_t)b * K + 16u * W);
#pragma unroll
      for (int e = 0; e < 4; e++)
        __stcg(d4 + e, make_float4(v[4 * e], v[4 * e + 1], v[4 * e + 2], v[4 * e + 3]));
    }
    if (MODE == kPrepNorm) {
      float ss = 0.0f;
#pragma unroll
      for (int e = 0; e < 16; e++) ss = fmaf(v[e], v[e], ss);
      pss[k] = ss;
    }
  }
  if (MODE == kPrepNorm) {
    csync();
    if ((uint32_t)warp < B) {          // row b = warp
      float s = 0.0f;
      for (uint32_t W = (uint32_t)lane; W < nw; W += 32u) s += pss[warp * nw + W];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
      if (lane == 0) st->rinv[warp] = 1.0f / sqrtf(s / (float)K + eps);
    }
  }
  csync();
  if (MODE != kPrepGiven) {
#pragma unroll 1
    for (uint32_t k = (uint32_t)tid; k < n; k += kCT) {
      const uint32_t b = k / nw, W = k % nw;
      float4 *x4 = reinterpret_cast<float4 *>(xs + (size_t)b * K + 16u * W);
      float mm = 0.0f;
      int bad = 0;
#pragma unroll
      for (int e = 0; e < 4; e++) {
        float4 f = x4[e];
        if (MODE == kPrepNorm) {
          const float ri = st->rinv[b];
          const float4 gv = __ldg(reinterpret_cast<const float4 *>(G + 16u * W) + e);
          f.x = __fmul_rn(__fmul_rn(f.x, ri), gv.x);
          f.y = __fmul_rn(__fmul_rn(f.y, ri), gv.y);
          f.z = __fmul_rn(__fmul_rn(f.z, ri), gv.z);
          f.w = __fmul_rn(__fmul_rn(f.w, ri), gv.w);
          x4[e] = f;
        }
        mm = fmaxf(fmaxf(mm, fabsf(f.x)), fmaxf(fmaxf(fabsf(f.y), fabsf(f.z)), fabsf(f.w)));
        bad |= !isfinite(f.x) | !isfinite(f.y) | !isfinite(f.z) | !isfinite(f.w);
      }
      pmx[k] = mm;
      pbad[k] = bad;
    }
    csync();
    if ((uint32_t)warp < B) {
      float mm = 0.0f;
      int bad = 0;
      for (uint32_t W = (uint32_t)lane; W < nw; W += 32u) {
        mm = fmaxf(mm, pmx[warp * nw + W]);
        bad |= pbad[warp * nw + W];
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) mm = fmaxf(mm, __shfl_xor_sync(0xffffffffu, mm, o));
      bad = __any_sync(0xffffffffu, bad);
      if (lane == 0) {
        float mul, inv;
        const bool ok = row_scale(mm, bad != 0, &mul, &inv, n_limbs((int)B));
        st->mul[warp] = mul;
        st->inv[warp] = inv;
        st->flag[warp] = !ok;
      }
    }
  } else if (tid < (int)B) {
    given_scale(__uint_as_float(__ldcg(maxb + tid)), n_limbs((int)B), &st->mul[tid], &st->inv[tid],
                &st->flag[tid]);
  }
  csync();
  PrepOut P;
  P.frag = reinterpret_cast<uint2 *>(frag);
  long long *pxs = reinterpret_cast<long long *>(pss);   // the word partials are dead now
#pragma unroll 1
  for (uint32_t k = (uint32_t)tid; k < n; k += kCT) {
    const uint32_t b = k / nw, W = k % nw;
    const float4 *x4 = reinterpret_cast<const float4 *>(xs + (size_t)b * K + 16u * W);
    float v[16];
#pragma unroll
    for (int e = 0; e < 4; e++) {
      const float4 f = x4[e];
      v[4 * e] = f.x; v[4 * e + 1] = f.y; v[4 * e + 2] = f.z; v[4 * e + 3] = f.w;
    }
    pxs[k] = quantize_word(v, st->mul[b], st->flag[b] == 0, W, b, NT, n_limbs((int)B), P);
  }
  csync();
  if ((uint32_t)warp < B) {            // the row's offset sum (exact: any order)
    long long x = 0;
    for (uint32_t W = (uint32_t)lane; W < nw; W += 32u) x += pxs[warp * nw + W];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
    if (lane == 0) st->xs[warp] = x;
  }
  csync();
}

// ---- attention (one task on half a CTA) ----------------------------------------------
struct AttnCtx {
  const float *qkv;
  const float2 *rope;
  float *ck, *cv, *apart, *ctx;
  unsigned *acnt;
  uint32_t kvr, hr, grp, maxseq, chunk, nsplit, qkv_rows, p;
  uint64_t cache_words;
  float coef;
};

// The decoder's fused attention for one (split, sequence b, kv head) with the
// operation order of attn_rope_partial_kernel, one query head of the group
// at a time (the heads never interact, so the bits are the same): the head
// rotated at position P in registers, the split's cached keys folded four
// rows in flight per warp, the new key and value (rotated; written to the
// cache row P by the split that holds it) folded last, the four warps
// merged.  The last split of a (b, kv head) to finish merges all splits
// into the context rows (attn_combine's order).
template <int HD>
__device__ __forceinline__ void attn_task(const AttnCtx &C, uint32_t split, uint32_t bkv,
                                          float *scr, int h, int *s_last) {
  constexpr int DPL = HD / 32;
  constexpr int U = 4;
  const int hl = (int)threadIdx.x & 127, lane = hl & 31, warp = hl >> 5;
  const uint32_t bb = bkv / C.kvr, kvh = bkv % C.kvr, p = C.p;
  float *s_m = scr, *s_l = scr + kAW, *s_o = scr + 2 * kAW;   // [kAW], [kAW], [kAW][HD]
  const uint32_t len = min(p + 1u, C.maxseq);
  const uint32_t p0 = split * C.chunk;
  const uint32_t p1 = min(p0 + C.chunk, len);
  const bool has_p = p < C.maxseq && p >= p0 && p < p1;
  const uint32_t kvdim = C.kvr * HD;
  const float *row = C.qkv + (uint64_t)bb * C.qkv_rows;

  float cs[DPL], sn[DPL];
#pragma unroll
  for (int d = 0; d < DPL; d++) {
    const uint32_t m = (uint32_t)(lane * DPL + d) % (HD / 2);
    const float2 r = __ldg(C.rope + (uint64_t)min(p, C.maxseq - 1u) * (HD / 2) + m);
    cs[d] = r.x;
    sn[d] = r.y;
  }
  const bool first_half = lane < 16;
  auto rotate = [&](const float *src, float (&out)[DPL]) {
#pragma unroll
    for (int d = 0; d < DPL; d++) {
      const float own = __ldcg(src + lane * DPL + d);
      const float other = __shfl_xor_sync(0xffffffffu, own, 16);
      const float a0 = first_half ? own : other, a1 = first_half ? other : own;
      out[d] = first_half ? __fsub_rn(__fmul_rn(a0, cs[d]), __fmul_rn(a1, sn[d]))
                          : __fadd_rn(__fmul_rn(a1, cs[d]), __fmul_rn(a0, sn[d]));
    }
  };
  float kn[DPL], vn[DPL];
  const uint64_t cbase = (uint64_t)bb * C.maxseq * kvdim + (uint64_t)kvh * HD + lane * DPL;
  if (has_p) {
    rotate(row + (uint64_t)(C.hr + kvh) * HD, kn);
    const float *vs = row + (uint64_t)(C.hr + C.kvr + kvh) * HD + lane * DPL;
#pragma unroll
    for (int d = 0; d < DPL; d++) vn[d] = __ldcg(vs + d);
    const uint64_t off = cbase + (uint64_t)p * kvdim;
    if (warp == 0 && off + DPL <= C.cache_words) {
#pragma unroll
      for (int d = 0; d < DPL; d++) {
        C.ck[off + d] = kn[d];
        C.cv[off + d] = vn[d];
      }
    }
  }
  const uint32_t pc = has_p ? p : p1;   // cached keys: [p0, pc)
  for (uint32_t hh = 0; hh < C.grp; hh++) {
    const uint32_t hq = kvh * C.grp + hh;
    float q[DPL];
    rotate(row + (uint64_t)hq * HD, q);
    float m = -INFINITY, l = 0.0f, o[DPL];
#pragma unroll
    for (int d = 0; d < DPL; d++) o[d] = 0.0f;
    auto fold = [&](const float (&kr)[DPL], const float (&vr)[DPL]) {
      float dot = 0.0f;
#pragma unroll
      for (int d = 0; d < DPL; d++) dot = fmaf(q[d], kr[d], dot);
      for (int off = 16; off > 0; off >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, off);
      const float sc = dot * C.coef;
      const float mn = fmaxf(m, sc);
      const float corr = expf(m - mn);   // exp(-inf) = 0 on the first key
      const float pr = expf(sc - mn);
      l = l * corr + pr;
#pragma unroll
      for (int d = 0; d < DPL; d++) o[d] = fmaf(pr, vr[d], o[d] * corr);
      m = mn;
    };
    for (uint32_t j0 = p0 + warp * U; j0 < pc; j0 += kAW * U) {
      float kr[U][DPL], vr[U][DPL];
#pragma unroll
      for (int u = 0; u < U; u++) {
        const uint32_t j = j0 + u;
        const uint64_t off = cbase + (uint64_t)j * kvdim;
        const bool ok = j < pc && off + DPL <= C.cache_words;
        if (DPL == 4) {
          const float4 k4 =
              ok ? __ldcs(reinterpret_cast<const float4 *>(C.ck + off)) : make_float4(0, 0, 0, 0);
          const float4 v4 =
              ok ? __ldcs(reinterpret_cast<const float4 *>(C.cv + off)) : make_float4(0, 0, 0, 0);
          kr[u][0] = k4.x; kr[u][1] = k4.y; kr[u][2] = k4.z; kr[u][3] = k4.w;
          vr[u][0] = v4.x; vr[u][1] = v4.y; vr[u][2] = v4.z; vr[u][3] = v4.w;
        } else {
#pragma unroll
          for (int d = 0; d < DPL; d++) {
            kr[u][d] = ok ? __ldcs(C.ck + off + d) : 0.0f;
            vr[u][d] = ok ? __ldcs(C.cv + off + d) : 0.0f;
          }
        }
      }
#pragma unroll
      for (int u = 0; u < U; u++) {
        if (j0 + u >= pc) break;
        fold(kr[u], vr[u]);
      }
    }
    if (has_p && warp == (int)(((pc - p0) / U) % kAW)) fold(kn, vn);
    if (lane == 0) {
      s_m[warp] = m;
      s_l[warp] = l;
    }
#pragma unroll
    for (int d = 0; d < DPL; d++) s_o[warp * HD + lane * DPL + d] = o[d];
    hsync(h);
    for (uint32_t d = (uint32_t)hl; d < (uint32_t)HD; d += kAW * 32) {
      float mm = -INFINITY;
      for (int w = 0; w < kAW; w++) mm = fmaxf(mm, s_m[w]);
      float ll = 0.0f, oo = 0.0f;
      if (mm > -INFINITY) {
        for (int w = 0; w < kAW; w++) {
          const float c = expf(s_m[w] - mm);
          ll += s_l[w] * c;
          oo += s_o[w * HD + d] * c;
        }
      }
      float *pp = C.apart + (((uint64_t)bb * C.hr + hq) * C.nsplit + split) * (HD + 2);
      __stcg(pp + 2 + d, oo);
      if (d == 0) {
        __stcg(pp, mm);
        __stcg(pp + 1, ll);
      }
    }
    hsync(h);   // the merge scratch is reused by the next head
  }
  __threadfence();
  hsync(h);
  if (hl == 0) *s_last = atomicAdd(C.acnt + bkv, 1u) == C.nsplit - 1u;
  hsync(h);
  if (*s_last) {
    __threadfence();
    constexpr int SB = 8;   // splits whose loads are in flight at once
    for (uint32_t e = (uint32_t)hl; e < C.grp * (uint32_t)HD; e += kAW * 32) {
      const uint32_t hq = kvh * C.grp + e / HD, d = e % HD;
      const float *pp = C.apart + ((uint64_t)bb * C.hr + hq) * C.nsplit * (HD + 2);
      float mm = -INFINITY;
      for (uint32_t s0 = 0; s0 < C.nsplit; s0 += SB) {
        float mv[SB];
#pragma unroll
        for (int u = 0; u < SB; u++)
          mv[u] = s0 + u < C.nsplit ? __ldcg(pp + (uint64_t)(s0 + u) * (HD + 2)) : -INFINITY;
#pragma unroll
        for (int u = 0; u < SB; u++) mm = fmaxf(mm, mv[u]);
      }
      float ll = 0.0f, oo = 0.0f;
      for (uint32_t s0 = 0; s0 < C.nsplit; s0 += SB) {
        float mv[SB], lv[SB], ov[SB];
#pragma unroll
        for (int u = 0; u < SB; u++) {
          const bool in = s0 + u < C.nsplit;
          const float *ps = pp + (uint64_t)(s0 + u) * (HD + 2);
          mv[u] = in ? __ldcg(ps) : -INFINITY;
          lv[u] = in ? __ldcg(ps + 1) : 0.0f;
          ov[u] = in ? __ldcg(ps + 2 + d) : 0.0f;
        }
#pragma unroll
        for (int u = 0; u < SB; u++) {      // in split order, as attn_combine
          if (mv[u] > -INFINITY) {
            const float c = expf(mv[u] - mm);
            ll += lv[u] * c;
            oo += ov[u] * c;
          }
        }
      }
      __stcg(C.ctx + (uint64_t)bb * C.hr * HD + (uint64_t)hq * HD + d, oo / ll);
    }
    if (hl == 0) C.acnt[bkv] = 0u;
  }
  hsync(h);   // s_last is reused by the next task
}

// The f32 output of the down GEMV for (b, column i): the exact sum of its
// chunks' dot products (accumulated in DSUM), scaled.
__device__ __forceinline__ float down_value(long long tot, float sd, float inv, int flag) {
  if (flag) return __uint_as_float(kNaN);
  return ((float)tot * inv) * sd;
}

// ---- the kernel ---------------------------------------------------------------------------
template <int HD, int NT>
__global__ void __launch_bounds__(kThreads, 1) step_kernel(const StepArgs A) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  __shared__ int s_last[2];
  uint8_t *sm = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 127) &
                                            ~(uintptr_t)127);
  const uint32_t grp = A.hr / A.kvr;
  const StepSmem Ls = step_layout(NT, HD, grp, A.nst);
  const uint32_t G = gridDim.x, cta = blockIdx.x;
  const int warp = (int)(threadIdx.x >> 5), lane = (int)(threadIdx.x & 31);
  Ring ring;
  ring.full = reinterpret_cast<uint64_t *>(sm);
  ring.empty = ring.full + kStepMaxStages;
  ring.base = sa(sm + Ls.ring);
  ring.nst = A.nst;
  ring.it = 0;
  if (threadIdx.x == 0) {
    for (uint32_t i = 0; i < ring.nst; i++) {
      mb_init(&ring.full[i], 1);
      mb_init(&ring.empty[i], kCW);
    }
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  __syncthreads();

  const uint32_t H = A.H, B = A.B, F = A.fr, nl = A.L;
  const uint32_t qcols = A.hr * HD;
  uint32_t dgroup = 0;                                        // this CTA's K chunk of down
  while (dgroup + 1u < A.dch && share(G, A.dch, dgroup + 1u).lo <= cta) dgroup++;
  const Range dcta = share(G, A.dch, dgroup);                 // the chunk's CTAs
  const Range dblk = share(F / 128u, A.dch, dgroup);          // its 128-column blocks
  const Range qr = share(A.qkv_rows / 16u, G, cta), orr = share(H / 16u, G, cta),
              gr = share(F / 16u, G, cta);
  const Range dr = share(H / 16u, dcta.hi - dcta.lo, cta - dcta.lo);
  const StepLayer *layers = A.layers;
  int *err = A.err;

  if (warp == kCW) {
    // ---- producer: every weight stage of the step, in consumption order ----
    for (uint32_t l = 0; l < nl; l++) {
      const StepLayer &Ly = layers[l];
      for (uint32_t t = qr.lo; t < qr.hi; t++)
        produce(ring, StageSrc{Ly.wqkv, 16u * t, H / 16u, 0u, H / 16u}, lane, err);
      for (uint32_t t = orr.lo; t < orr.hi; t++)
        produce(ring, StageSrc{Ly.wo, 16u * t, qcols / 16u, 0u, qcols / 16u}, lane, err);
      for (uint32_t t = gr.lo; t < gr.hi; t++) {
        produce(ring, StageSrc{Ly.wgu, 16u * t, H / 16u, 0u, H / 16u}, lane, err);
        produce(ring, StageSrc{Ly.wgu, F + 16u * t, H / 16u, 0u, H / 16u}, lane, err);
      }
      for (uint32_t t = dr.lo; t < dr.hi; t++)
        produce(ring, StageSrc{Ly.wd, 16u * t, F / 16u, dblk.lo * 8u, (dblk.hi - dblk.lo) * 8u},
                lane, err);
    }
    return;
  }

  // ---- compute warps ----
  uint8_t *act = sm + Ls.act;
  int *red = reinterpret_cast<int *>(sm + Ls.red);
  int *sacc = reinterpret_cast<int *>(sm + Ls.sacc);
  float *pss = reinterpret_cast<float *>(sm + Ls.pre);
  float *pmx = pss + kStepMaxB * (kStepMaxK / 16u);
  int *pbad = reinterpret_cast<int *>(pss);   // the sums of squares are consumed by then
  RowStat *st = reinterpret_cast<RowStat *>(pmx + kStepMaxB * (kStepMaxK / 16u));
  const uint32_t frag = sa(act);
  float *xsm = reinterpret_cast<float *>(act + step_frag_bytes(NT));   // staged rows
  const uint32_t xkey = offset_key();
  const unsigned long long nbar = step_barriers(nl);
  const unsigned long long base = __ldcg(A.sep) * nbar * (unsigned long long)G;
  unsigned long long bars = 0;
  const int tid = (int)threadIdx.x;
  const bool lead = cta == 0;
  const int sstride = 16 * (8 * NT + 1);

  for (uint32_t l = 0; l < nl; l++) {
    const StepLayer &Ly = layers[l];
    // ---- Q: h = E[tok] (layer 0) or h + d; x = RMSNorm(h) g_attn; Q|K|V ----
    if (l == 0) {
      const float *embed = A.embed;
      const int *tok = A.tok;
      prep_rows<kPrepNorm, NT>(
          [=](uint32_t b, uint32_t W, float (&v)[16]) {
            const float4 *e4 =
                reinterpret_cast<const float4 *>(embed + (size_t)__ldcg(tok + b) * H + 16u * W);
#pragma unroll
            for (int e = 0; e < 4; e++) {
              const float4 f = __ldg(e4 + e);
              v[4 * e] = f.x; v[4 * e + 1] = f.y; v[4 * e + 2] = f.z; v[4 * e + 3] = f.w;
            }
          },
          B, H, Ly.gattn, A.eps, nullptr, lead ? A.hbuf : nullptr, act, xsm, pss, pmx, pbad, st, warp,
          lane);
    } else {
      // the previous layer's down GEMV output, scaled as its rows were
      if (tid < (int)B) {
        float mul;
        given_scale(__uint_as_float(__ldcg(A.amax + tid)), n_limbs((int)B), &mul, &st->dinv[tid], &st->dflag[tid]);
      }
      csync();
      const float *sd = layers[l - 1].sd;
      const float *hsrc = (A.hbuf + (size_t)B * H);
      const RowStat *cst = st;
      prep_rows<kPrepNorm, NT>(
          [=](uint32_t b, uint32_t W, float (&v)[16]) {
            const float inv = cst->dinv[b];
            const int fl = cst->dflag[b];
            const float4 *h4 = reinterpret_cast<const float4 *>(hsrc + (size_t)b * H + 16u * W);
#pragma unroll
            for (int e = 0; e < 4; e++) {
              const float4 f = __ldcg(h4 + e);
              v[4 * e] = f.x; v[4 * e + 1] = f.y; v[4 * e + 2] = f.z; v[4 * e + 3] = f.w;
            }
            const long long *dp = A.dpart + (size_t)b * H + 16u * W;
            long long tot[16];
            float sc[16];
#pragma unroll
            for (int e = 0; e < 16; e++) {
              tot[e] = __ldcg(dp + e);
              sc[e] = __ldg(sd + 16u * W + (uint32_t)e);
            }
#pragma unroll
            for (int e = 0; e < 16; e++) v[e] = __fadd_rn(v[e], down_value(tot[e], sc[e], inv, fl));
          },
          B, H, Ly.gattn, A.eps, nullptr, lead ? A.hbuf : nullptr, act, xsm, pss, pmx, pbad, st, warp,
          lane);
    }
    const float *sq = Ly.sqkv;
    for (uint32_t t = qr.lo; t < qr.hi; t++) {
      // the epilogue's scale, requested before the tile's MMAs
      const float sc = tid < 16 * (int)B ? __ldg(sq + 16u * t + (uint32_t)(tid & 15)) : 0.0f;
      tile<NT>(ring, H / 16u, frag, warp, lane, xkey, red, sacc, err);
      if (tid < 16 * (int)B) {
        const int r = tid & 15, s = tid >> 4;
        const uint32_t oi = 16u * t + (uint32_t)r;
        const long long tot = tile_tot<NT>(sacc, r, s, st->xs[s], n_limbs((int)B));
        const float y = st->flag[s] ? __uint_as_float(kNaN) : ((float)tot * st->inv[s]) * sc;
        __stcg(A.qkv + (uint64_t)s * A.qkv_rows + oi, y);
      }
    }
    grid_sync(A.bar, base + (++bars) * G, err);
    // ---- A: attention; the last split of a head merges into A.ctx ----
    {
      const int h = warp >> 2;
      float *scr = reinterpret_cast<float *>(act) + h * (2 * kAW + kAW * HD);
      const uint32_t ntask = A.nsplit * B * A.kvr;
      AttnCtx ac;
      ac.qkv = A.qkv;
      ac.rope = A.rope;
      ac.apart = A.apart;
      ac.ctx = A.ctx;
      ac.acnt = A.acnt;
      ac.kvr = A.kvr;
      ac.hr = A.hr;
      ac.grp = A.hr / A.kvr;
      ac.maxseq = A.maxseq;
      ac.chunk = A.chunk;
      ac.nsplit = A.nsplit;
      ac.qkv_rows = A.qkv_rows;
      ac.p = (uint32_t)__ldcg(A.pos);
      ac.cache_words = (uint64_t)A.max_batch * A.maxseq * A.kvr * HD;
      ac.coef = A.coef;
      ac.ck = Ly.ck;
      ac.cv = Ly.cv;
      // this layer's down GEMV accumulates into A.dpart: clear it (the
      // previous layer's sums were read before the last barrier)
      {
        const Range z = share(B * H, G, cta);
        for (uint32_t i = z.lo + (uint32_t)tid; i < z.hi; i += kCT) __stcg(A.dpart + i, 0ll);
      }
      for (uint32_t t = 2u * cta + (uint32_t)h; t < ntask; t += 2u * G)
        attn_task<HD>(ac, t % A.nsplit, t / A.nsplit, scr, h, &s_last[h]);
    }
    grid_sync(A.bar, base + (++bars) * G, err);
    // ---- O: prep of the context rows; the O GEMV ----
    if (lead && tid < (int)B) A.amax[tid] = 0u;        // for this layer's SwiGLU maximum
    {
      const float *csrc = A.ctx;
      prep_rows<kPrepPlain, NT>(
          [=](uint32_t b, uint32_t W, float (&v)[16]) {
            const float4 *c4 =
                reinterpret_cast<const float4 *>(csrc + (size_t)b * qcols + 16u * W);
#pragma unroll
            for (int e = 0; e < 4; e++) {
              const float4 f = __ldcg(c4 + e);
              v[4 * e] = f.x; v[4 * e + 1] = f.y; v[4 * e + 2] = f.z; v[4 * e + 3] = f.w;
            }
          },
          B, qcols, nullptr, 0.0f, nullptr, nullptr, act, xsm, pss, pmx, pbad, st, warp, lane);
    }
    const float *so = Ly.so;
    for (uint32_t t = orr.lo; t < orr.hi; t++) {
      const float sc = tid < 16 * (int)B ? __ldg(so + 16u * t + (uint32_t)(tid & 15)) : 0.0f;
      tile<NT>(ring, qcols / 16u, frag, warp, lane, xkey, red, sacc, err);
      if (tid < 16 * (int)B) {
        const int r = tid & 15, s = tid >> 4;
        const uint32_t oi = 16u * t + (uint32_t)r;
        const long long tot = tile_tot<NT>(sacc, r, s, st->xs[s], n_limbs((int)B));
        const float y = st->flag[s] ? __uint_as_float(kNaN) : ((float)tot * st->inv[s]) * sc;
        __stcg(A.o + (uint64_t)s * H + oi, y);
      }
    }
    grid_sync(A.bar, base + (++bars) * G, err);
    // ---- G: h += A.o; x = RMSNorm(h) g_ffn; gate|up with SwiGLU ----
    {
      const float *hsrc = A.hbuf, *osrc = A.o;
      prep_rows<kPrepNorm, NT>(
          [=](uint32_t b, uint32_t W, float (&v)[16]) {
            const float4 *h4 = reinterpret_cast<const float4 *>(hsrc + (size_t)b * H + 16u * W);
            const float4 *o4 = reinterpret_cast<const float4 *>(osrc + (size_t)b * H + 16u * W);
#pragma unroll
            for (int e = 0; e < 4; e++) {
              const float4 f = __ldcg(h4 + e), g = __ldcg(o4 + e);
              v[4 * e] = __fadd_rn(f.x, g.x);
              v[4 * e + 1] = __fadd_rn(f.y, g.y);
              v[4 * e + 2] = __fadd_rn(f.z, g.z);
              v[4 * e + 3] = __fadd_rn(f.w, g.w);
            }
          },
          B, H, Ly.gffn, A.eps, nullptr, lead ? (A.hbuf + (size_t)B * H) : nullptr, act, xsm, pss, pmx, pbad, st, warp,
          lane);
    }
    const float *sgu = Ly.sgu;
    for (uint32_t t = gr.lo; t < gr.hi; t++) {
      const uint32_t c = 16u * t + (uint32_t)(tid & 15);
      const float scg = tid < 16 * (int)B ? __ldg(sgu + c) : 0.0f;
      const float scu = tid < 16 * (int)B ? __ldg(sgu + F + c) : 0.0f;
      tile<NT>(ring, H / 16u, frag, warp, lane, xkey, red, sacc, err);             // gate rows
      tile<NT>(ring, H / 16u, frag, warp, lane, xkey, red, sacc + sstride, err);   // up rows
      if (tid < 16 * (int)B) {
        const int r = tid & 15, s = tid >> 4;
        float av;
        if (st->flag[s]) {
          av = __uint_as_float(kNaN);
        } else {
          const long long tg = tile_tot<NT>(sacc, r, s, st->xs[s], n_limbs((int)B));
          const long long tu = tile_tot<NT>(sacc + sstride, r, s, st->xs[s], n_limbs((int)B));
          const float gv = ((float)tg * st->inv[s]) * scg;
          const float uv = ((float)tu * st->inv[s]) * scu;
          const float sg = 1.0f / (1.0f + expf(-gv));
          av = __fmul_rn(__fmul_rn(gv, sg), uv);
        }
        __stcg(A.a + (uint64_t)s * F + c, av);
        // the row maximum for the down GEMV's scale (a NaN's bits exceed inf's)
        atomicMax(A.amax + s, __float_as_uint(fabsf(av)));
      }
    }
    grid_sync(A.bar, base + (++bars) * G, err);
    // ---- D: prep of this CTA's chunk of a; the down GEMV (exact partial sums) ----
    {
      const uint32_t c0 = dblk.lo * 128u, kc = (dblk.hi - dblk.lo) * 128u;
      const float *asrc = A.a;
      prep_rows<kPrepGiven, NT>(
          [=](uint32_t b, uint32_t W, float (&v)[16]) {
            const float4 *a4 =
                reinterpret_cast<const float4 *>(asrc + (size_t)b * F + c0 + 16u * W);
#pragma unroll
            for (int e = 0; e < 4; e++) {
              const float4 f = __ldcg(a4 + e);
              v[4 * e] = f.x; v[4 * e + 1] = f.y; v[4 * e + 2] = f.z; v[4 * e + 3] = f.w;
            }
          },
          B, kc, nullptr, 0.0f, A.amax, nullptr, act, xsm, pss, pmx, pbad, st, warp, lane);
      for (uint32_t t = dr.lo; t < dr.hi; t++) {
        tile<NT>(ring, kc / 16u, frag, warp, lane, xkey, red, sacc, err);
        if (tid < 16 * (int)B) {
          const int r = tid & 15, s = tid >> 4;
          const uint32_t oi = 16u * t + (uint32_t)r;
          atomicAdd(reinterpret_cast<unsigned long long *>(A.dpart + (uint64_t)s * H + oi),
                    (unsigned long long)tile_tot<NT>(sacc, r, s, st->xs[s], n_limbs((int)B)));
        }
      }
    }
    grid_sync(A.bar, base + (++bars) * G, err);
  }

  // ---- CTA 0: x = RMSNorm(h + d) g_final, the LM head's input ----
  if (!lead) return;
  {
    if (tid < (int)B) {
      float mul;
      given_scale(__uint_as_float(__ldcg(A.amax + tid)), n_limbs((int)B), &mul, &st->dinv[tid], &st->dflag[tid]);
    }
    csync();
    const float *sd = layers[nl - 1].sd;
    float *xrow = reinterpret_cast<float *>(act);
    for (uint32_t b = 0; b < B; b++) {
      const float inv = st->dinv[b];
      const int fl = st->dflag[b];
      for (uint32_t W = (uint32_t)tid; W < H / 16u; W += kCT) {   // per-word partials
        float ss = 0.0f;
        for (uint32_t e = 0; e < 16; e++) {
          const uint32_t i = 16u * W + e;
          const float v = __fadd_rn(__ldcg((A.hbuf + (size_t)B * H) + (size_t)b * H + i),
                                    down_value(__ldcg(A.dpart + (size_t)b * H + i),
                                               __ldg(sd + i), inv, fl));
          xrow[i] = v;
          ss = fmaf(v, v, ss);
        }
        pss[W] = ss;
      }
      csync();
      if (warp == 0) {
        float s = 0.0f;
        for (uint32_t W = (uint32_t)lane; W < H / 16u; W += 32u) s += pss[W];
#pragma unroll
        for (int k = 16; k > 0; k >>= 1) s += __shfl_xor_sync(0xffffffffu, s, k);
        if (lane == 0) st->rinv[0] = 1.0f / sqrtf(s / (float)H + A.eps);
      }
      csync();
      const float ri = st->rinv[0];
      for (uint32_t i = (uint32_t)tid; i < H; i += kCT)
        __stcg(A.x_final + (size_t)b * H + i,
               __fmul_rn(__fmul_rn(xrow[i], ri), __ldg(A.gfinal + i)));
      csync();
    }
  }
  if (tid == 0) *A.sep = *A.sep + 1ull;   // every CTA read it before its first barrier
}

// Launch for one (head size, n-tiles): cooperative (all CTAs resident), one
// CTA per SM, as many ring stages as the shared memory holds.
template <int HD, int NT>
cudaError_t step_launch_one(const StepArgs &a, cudaStream_t st) {
  static int sms = 0;
  static uint32_t budget = 0;
  if (!budget) {
    int dev = 0, optin = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e == cudaSuccess)
      e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return e;
    const uint32_t b = (uint32_t)optin - 1024u;   // static shared memory and alignment slack
    e = cudaFuncSetAttribute(step_kernel<HD, NT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)b + 128);
    if (e != cudaSuccess) return e;
    int per = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per, step_kernel<HD, NT>, kThreads,
                                                      (size_t)b + 128u);
    if (e != cudaSuccess) return e;
    if (per < 1) return cudaErrorInvalidConfiguration;
    budget = b;
  }
  StepArgs args = a;
  args.nst = step_stages(NT, HD, a.hr / a.kvr, budget);
  if (args.nst < 2) return cudaErrorInvalidConfiguration;
  const uint32_t smem = step_layout(NT, HD, a.hr / a.kvr, args.nst).total + 128u;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)sms);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeCooperative;
  at[0].val.cooperative = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, step_kernel<HD, NT>, args);
}

template <int HD>
cudaError_t step_launch_hd(const StepArgs &a, cudaStream_t st) {
  switch (n_tiles((int)a.B)) {
    case 1: return step_launch_one<HD, 1>(a, st);
    case 2: return step_launch_one<HD, 2>(a, st);
    case 3: return step_launch_one<HD, 3>(a, st);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace
}  // namespace nl

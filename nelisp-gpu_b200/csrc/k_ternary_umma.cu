// k_ternary_umma.cu -- the ternary GEMM for many sequence rows (prefill) on
// the 5th-generation tensor cores (tcgen05, accumulators in TMEM).
//
// Y[s, o] = S[o] * sum_k t(o, k) X[s, k] (+ BIAS[o]) for seq > 16 rows, the
// per-row-scale form of ternary-rows (lisp/nelisp-gpu-kernels.el:713-746)
// computed exactly: every activation row is scaled by a power of two and
// split into three int8 limbs (as in the GEMV's prep), the products are
// summed in int32 by tcgen05.mma.kind::i8, and the limbs are recombined in
// int64 -- so the result is the exact sum rounded once per row scale.
//
// One CTA computes a tile of 128 MH output rows x 64 or 80 sequence rows
// (N = 3 x the rows: one column per limb) over the whole K, 3 + 4 MH warps:
//   warp 0      TMA producer: the packed weight tile (128 MH rows x 128
//               columns, two bits each, 4 MH KB) and the int8 limb tile
//               (N x 128 B, 128-byte swizzle) per stage, S-stage mbarrier
//               ring; the weights of the first stages are requested before
//               waiting for the prep kernel (programmatic dependent launch);
//   warps 2 ..  expand the two-bit codes into the int8 A tiles in shared
//   1 + 4 MH    memory (one thread per weight row; one shift and one mask per
//               four weights, 64 * t per byte), then arrive;
//   warp 1 and  two MMA issuers, four 128xNx32 MMAs per stage each into its
//   2 + 4 MH    own TMEM accumulator (warp 1 also allocates TMEM);
//               tcgen05.commit frees the stage.  MH = 1: they take the
//               stages in turn (two partial sums of the same rows); MH = 2:
//               issuer h multiplies rows half h in every stage against the
//               same limb tile, halving the limb stream per MMA;
//   warps 2 ..  finally read the accumulators back (tcgen05.ld), recombine
//   1 + 4 MH    the limbs and write Y; rows the prep flagged are computed
//               there on the CUDA cores.
// The shift-and-mask expansion leaves the 16 codes of a packed word in the
// order P = {3,7,11,15, 2,6,10,14, 1,5,9,13, 0,4,8,12}; the limb tile is
// written in the same order, so the K index of A and B agrees.
// Every mbarrier wait is bounded; one that gives up sets the library's
// host-mapped wait flag, which the synchronising entry points report.

#include <cuda.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>
#include <stdlib.h>

#include "nl_internal.h"
#include "ternary_prep.cuh"

namespace nl {
namespace {

constexpr int kUmmaM = 128;              // output rows per CTA
constexpr int kUmmaK = 128;              // K per stage (bytes of int8)
constexpr int kUmmaStages = 4;
constexpr uint32_t kTmemCols = 512;      // two accumulators of up to 256 columns
constexpr uint32_t kWBytes = kUmmaM * kUmmaK / 4;      // packed weights per stage
constexpr uint32_t kABytes = kUmmaM * kUmmaK;           // int8 A per stage
// Sequence rows per CTA: 80 or 64 (chosen per shape, umma_tok).  MMA N is
// the (row, limb) columns, 3 * TOK <= 256, and N x 128 B of int8 B per stage.
template <int TOK>
struct UmmaTile {
  static constexpr int N = 3 * TOK;
  static constexpr uint32_t BBytes = N * kUmmaK;
  static_assert(N % 48 == 0 && N <= 256 && BBytes % 1024 == 0, "tile");
};
// Output rows per CTA: MH halves of 128.  With MH = 1 two issuers take the K
// stages in turn, each into its own accumulator (summed in the epilogue);
// with MH = 2 issuer h multiplies rows 128h .. 128h+127 in every stage
// against the same limb tile, so each limb stage staged from L2 feeds twice
// the MMA work (the limb stream is what bounds the kernel).
template <int MH>
struct UmmaRows {
  static constexpr int Stages = MH == 1 ? kUmmaStages : 3;
  static constexpr int Expanders = 4 * MH;                   // warps, one thread per A row
  static constexpr int Threads = 32 * (3 + Expanders);        // + producer, two issuers
  static constexpr uint32_t A = kABytes * MH, W = kWBytes * MH;
};
constexpr uint32_t kWaitRounds = 4096;
constexpr uint32_t kSuspendNs = 1000000;
constexpr uint32_t kTop2 = 0xC0C0C0C0u;


__device__ __forceinline__ uint32_t su32(const void *p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void bar_init(uint64_t *b, uint32_t n) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(su32(b)), "r"(n));
}
__device__ __forceinline__ void bar_expect(uint64_t *b, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(su32(b)),
               "r"(bytes) : "memory");
}
__device__ __forceinline__ void bar_arrive(uint64_t *b) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(su32(b)) : "memory");
}
__device__ __forceinline__ bool bar_wait(uint64_t *b, uint32_t parity, int *err) {
  for (uint32_t i = 0; i < kWaitRounds; i++) {
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done) : "r"(su32(b)), "r"(parity), "r"(kSuspendNs) : "memory");
    if (done) return true;
  }
  report_wait_timeout(err);
  return false;
}
__device__ __forceinline__ void tma2d(void *dst, const CUtensorMap *map, int x, int y,
                                      uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];\n" ::"r"(su32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(su32(bar))
      : "memory");
}

// Shared-memory matrix descriptor: K-major operand in the 128-byte-swizzle
// canonical layout (rows of 128 bytes, 8-row groups 1024 bytes apart).
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr) {
  return (uint64_t)((addr >> 4) & 0x3FFFu) | (1ull << 16) | ((uint64_t)(1024 >> 4) << 32) |
         (1ull << 46) | (2ull << 61);
}
// Instruction descriptor: s8 x s8 -> s32, both K-major, M = 128, N.
template <int N>
constexpr uint32_t umma_idesc() {
  return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) |
         ((uint32_t)(kUmmaM >> 4) << 24);
}

__device__ __forceinline__ void umma_i8(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                        uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}
__device__ __forceinline__ void umma_commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(
                   su32(bar)) : "memory");
}
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,"
      "%15}, [%16];\n"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
        "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]),
        "=r"(v[14]), "=r"(v[15])
      : "r"(taddr));
}

// ---- prep: activation rows -> scale, flag and the K-permuted int8 limb rows --
// Row s of X becomes rows 3s, 3s+1, 3s+2 of XB (limbs l0, l1, l2 with
// xq = l0 + 256 l1 + 65536 l2 and xq = round(x * 2^e), max|x * 2^e| in
// [2^21, 2^22)); byte p of each 16-column group holds column P[p].
__global__ void __launch_bounds__(256)
umma_prep_kernel(const float *__restrict__ X, uint32_t cols, int8_t *__restrict__ XB,
                 float *__restrict__ rowinv, int *__restrict__ rowflag) {
  pdl_trigger();                 // the GEMM may start streaming its weights
  pdl_wait();                    // X may come from the preceding kernel
  __shared__ float red[8];
  __shared__ int sbad;
  const uint32_t s = blockIdx.x;
  const float *xr = X + (size_t)s * cols;
  const float4 *x4 = reinterpret_cast<const float4 *>(xr);
  float m = 0.0f;
  int bad = 0;
  for (uint32_t i = threadIdx.x; i < cols / 4u; i += blockDim.x) {
    const float4 v = __ldg(x4 + i);
    m = fmaxf(fmaxf(m, fmaxf(fabsf(v.x), fabsf(v.y))), fmaxf(fabsf(v.z), fabsf(v.w)));
    bad |= !isfinite(v.x) | !isfinite(v.y) | !isfinite(v.z) | !isfinite(v.w);
  }
  bad = __syncthreads_or(bad);
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  if (threadIdx.x == 0) sbad = bad;
  __syncthreads();
  float mm = 0.0f;
  for (int w = 0; w < 8; w++) mm = fmaxf(mm, red[w]);
  // the exponent of the GEMV's prep (ternary_prep.cuh, row_scale)
  float mul = 0.0f, inv = 0.0f;
  const bool ok = row_scale(mm, sbad != 0, &mul, &inv, 3);
  if (threadIdx.x == 0) {
    rowinv[s] = inv;
    rowflag[s] = !ok;
  }
  // Byte p of a 16-column group holds column P[p] = 4 (p % 4) + 3 - p / 4:
  // {3,7,11,15, 2,6,10,14, 1,5,9,13, 0,4,8,12}.
  int8_t *o0 = XB + (size_t)(3 * s) * cols, *o1 = o0 + cols, *o2 = o1 + cols;
  for (uint32_t w = threadIdx.x; w < cols / 16u; w += blockDim.x) {
    float v[16];
#pragma unroll
    for (int q = 0; q < 4; q++) {
      const float4 f = ok ? __ldg(x4 + 4u * w + q) : make_float4(0.f, 0.f, 0.f, 0.f);
      v[4 * q] = f.x; v[4 * q + 1] = f.y; v[4 * q + 2] = f.z; v[4 * q + 3] = f.w;
    }
    uint32_t b0[4] = {0, 0, 0, 0}, b1[4] = {0, 0, 0, 0}, b2[4] = {0, 0, 0, 0};
#pragma unroll
    for (int p = 0; p < 16; p++) {
      const int qv = __float2int_rn(v[4 * (p % 4) + 3 - p / 4] * mul);
      const int l0 = (int)(int8_t)(qv & 0xff);
      const int r = (qv - l0) >> 8;
      const int l1 = (int)(int8_t)(r & 0xff);
      const int l2 = (r - l1) >> 8;
      b0[p >> 2] |= (uint32_t)(l0 & 0xff) << (8 * (p & 3));
      b1[p >> 2] |= (uint32_t)(l1 & 0xff) << (8 * (p & 3));
      b2[p >> 2] |= (uint32_t)(l2 & 0xff) << (8 * (p & 3));
    }
    reinterpret_cast<uint4 *>(o0)[w] = make_uint4(b0[0], b0[1], b0[2], b0[3]);
    reinterpret_cast<uint4 *>(o1)[w] = make_uint4(b1[0], b1[1], b1[2], b1[3]);
    reinterpret_cast<uint4 *>(o2)[w] = make_uint4(b2[0], b2[1], b2[2], b2[3]);
  }
}

// ---- the GEMM ------------------------------------------------------------------
// Two MMA issuers take the K stages in turn (one thread issues a tcgen05.mma
// only every ~50-170 cycles, a 128 x 240 x 32 MMA takes the tensor core ~120),
// each into its own accumulator; the epilogue adds the two exactly.
template <int TOK, int MH>
__global__ void __launch_bounds__(UmmaRows<MH>::Threads, 1)
ternary_umma_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmB,
                    const float *__restrict__ X, const uint32_t *__restrict__ WP,
                    const float *__restrict__ S, const float *__restrict__ BIAS,
                    const float *__restrict__ rowinv, const int *__restrict__ rowflag,
                    float *__restrict__ Y, uint32_t seq, uint32_t out, uint32_t cols,
                    int *err) {
  constexpr int kUmmaN = UmmaTile<TOK>::N;
  constexpr uint32_t kBBytes = UmmaTile<TOK>::BBytes;
  constexpr uint32_t kIdesc = umma_idesc<kUmmaN>();
  using RW = UmmaRows<MH>;
  constexpr int NS = RW::Stages;
  constexpr int kIssuer1 = 2 + RW::Expanders;       // the second issuer's warp
  extern __shared__ uint8_t smem_raw[];
  uint8_t *base = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  uint8_t *sA = base;                                   // stages x MH x 16 KB (1024-aligned)
  uint8_t *sB = sA + NS * RW::A;                        // stages x N x 128 B (1024-aligned)
  uint8_t *sW = sB + NS * kBBytes;                      // stages x MH x 4 KB
  uint64_t *full = reinterpret_cast<uint64_t *>(sW + NS * RW::W);
  uint64_t *aready = full + NS;
  uint64_t *empty = aready + NS;
  uint64_t *done = empty + NS;                          // one per issuer
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(done + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t m0 = blockIdx.x * (uint32_t)(kUmmaM * MH), t0 = blockIdx.y * (uint32_t)TOK;
  const uint32_t nk = cols / kUmmaK;

  if (threadIdx.x == 0) {
    for (int i = 0; i < NS; i++) {
      bar_init(&full[i], 1);
      bar_init(&aready[i], RW::Expanders);
      bar_init(&empty[i], MH);                          // one commit per issuer using it
    }
    bar_init(&done[0], 1);
    bar_init(&done[1], 1);
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(
                     su32(tmem_slot)), "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::);
  }
  asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
  const uint32_t tmem = *tmem_slot;               // accumulators at columns 0 and 256

  if (warp == 0) {
    // ---- producer: the weights of the first stages before the wait for
    // the prep kernel (launch_pdl), which does not write them ----
    if (lane == 0) {
      const uint32_t pre = nk < (uint32_t)NS ? nk : (uint32_t)NS;
      for (uint32_t kt = 0; kt < nk; kt++) {
        const int st = (int)(kt % NS);
        if (kt >= (uint32_t)NS && !bar_wait(&empty[st], ((kt / NS) - 1) & 1, err)) break;
        bar_expect(&full[st], RW::W + kBBytes);
        tma2d(sW + st * RW::W, &tmW, (int)(kt * (kUmmaK / 16)), (int)m0, &full[st]);
        if (kt >= pre) {
          tma2d(sB + st * kBBytes, &tmB, (int)(kt * kUmmaK), (int)(3 * t0), &full[st]);
        } else if (kt + 1 == pre) {
          pdl_wait();
          for (uint32_t k = 0; k < pre; k++)
            tma2d(sB + k * kBBytes, &tmB, (int)(k * kUmmaK), (int)(3 * t0), &full[k]);
        }
      }
    }
  } else if (warp == 1 || warp == kIssuer1) {
    // ---- MMA issuers: with MH = 1 issuer p takes the stages kt with
    // kt % 2 == p; with MH = 2 issuer p takes every stage for rows half p ----
    if (lane == 0) {
      const uint32_t p = warp == 1 ? 0u : 1u;
      const uint32_t acc_d = tmem + 256u * p;
      bool first = true;
      for (uint32_t kt = MH == 1 ? p : 0u; kt < nk; kt += MH == 1 ? 2u : 1u) {
        const int st = (int)(kt % NS);
        const uint32_t ph = (kt / NS) & 1;
        if (!bar_wait(&full[st], ph, err) || !bar_wait(&aready[st], ph, err)) break;
        asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
        const uint32_t a0 = su32(sA + st * RW::A + (MH == 1 ? 0u : p * kABytes));
        const uint32_t b0 = su32(sB + st * kBBytes);
#pragma unroll
        for (int k = 0; k < kUmmaK / 32; k++)
          umma_i8(acc_d, smem_desc(a0 + 32u * k), smem_desc(b0 + 32u * k), kIdesc,
                  (!first || k > 0) ? 1u : 0u);
        first = false;
        umma_commit(&empty[st]);      // the stage is free once these MMAs are done
      }
      umma_commit(&done[p]);
    }
  } else {
    // ---- expand the weights (warps 2 .. 1 + 4 MH, one thread per A row) ----
    const uint32_t r = threadIdx.x - 64;          // 0 .. 128 MH - 1
    for (uint32_t kt = 0; kt < nk; kt++) {
      const int st = (int)(kt % NS);
      if (!bar_wait(&full[st], (kt / NS) & 1, err)) break;
      const uint4 *wr = reinterpret_cast<const uint4 *>(sW + st * RW::W + r * 32u);
      const uint4 lo = wr[0], hi = wr[1];
      const uint32_t w8[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
      uint8_t *arow = sA + st * RW::A + (r >> 7) * kABytes + ((r & 127u) >> 3) * 1024u +
                      (r & 7u) * 128u;
#pragma unroll
      for (int c = 0; c < 8; c++) {
        const uint32_t w = w8[c];
        const uint4 v = make_uint4(w & kTop2, (w << 2) & kTop2, (w << 4) & kTop2, (w << 6) & kTop2);
        *reinterpret_cast<uint4 *>(arow + (((uint32_t)c ^ (r & 7u)) << 4)) = v;
      }
      // generic-proxy writes, read by the tensor cores (async proxy)
      asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
      __syncwarp();
      if (lane == 0) bar_arrive(&aready[st]);
    }
    // ---- epilogue: accumulators -> Y ----
    const uint32_t hh = MH == 1 ? 0u : (uint32_t)(warp - 2) / 4u;   // this warp's rows half
    const bool two = MH == 1 && nk >= 2;          // issuer 1 wrote a second partial sum
    if (bar_wait(&done[hh], 0, err) && (!two || bar_wait(&done[1], 0, err))) {
      asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
      const uint32_t q = (uint32_t)(warp & 3);      // TMEM lane quarter of this warp
      const uint32_t o = m0 + hh * 128u + q * 32u + (uint32_t)lane;
      const float sc = o < out ? __ldg(S + o) : 0.0f;
      const float bi = (BIAS && o < out) ? __ldg(BIAS + o) : 0.0f;
      const uint32_t lb = ((q * 32u) << 16) + 256u * hh;
      for (uint32_t c0 = 0; c0 < (uint32_t)kUmmaN; c0 += 48) {   // 16 rows per round
        uint32_t v[48], u[48];
#pragma unroll
        for (int j = 0; j < 3; j++) {
          tmem_ld16(tmem + lb + c0 + 16u * j, *reinterpret_cast<uint32_t(*)[16]>(v + 16 * j));
          if (two)
            tmem_ld16(tmem + lb + 256u + c0 + 16u * j, *reinterpret_cast<uint32_t(*)[16]>(u + 16 * j));
        }
        asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
        if (two) {
#pragma unroll
          for (int j = 0; j < 48; j++) v[j] += u[j];   // exact int32 partial sums
        }
#pragma unroll
        for (int j = 0; j < 16; j++) {
          const uint32_t s = t0 + c0 / 3u + (uint32_t)j;
          if (o >= out || s >= seq || rowflag[s]) continue;
          long long tot = (long long)(int)v[3 * j] + 256ll * (int)v[3 * j + 1] +
                          65536ll * (int)v[3 * j + 2];
          tot >>= 6;                                 // the operands carried 64 * t: exact
          float y = ((float)tot * rowinv[s]) * sc;
          if (BIAS) y = bi + y;
          Y[(size_t)s * out + o] = y;
        }
      }
      // Rows the prep flagged (non-finite or unrepresentable): the generic
      // CUDA-core arithmetic, one output row of this warp's 32 at a time.
      const uint32_t wng = cols / 16u, nblk = cols / 128u;
      for (uint32_t j = 0; j < (uint32_t)TOK; j++) {
        const uint32_t s = t0 + j;
        if (s >= seq) break;
        if (!rowflag[s]) continue;
        for (uint32_t rr = 0; rr < 32u; rr++) {
          const uint32_t orow = m0 + hh * 128u + q * 32u + rr;
          if (orow >= out) break;
          float acc1[1];
          ternary_row_generic<1>(X, WP + (size_t)orow * wng, nullptr, false, __ldg(S + orow),
                                 (int)s, 1, cols, nblk, wng, acc1);
          if (lane == 0) Y[(size_t)s * out + orow] = (BIAS ? __ldg(BIAS + orow) : 0.0f) + acc1[0];
        }
      }
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
  __syncthreads();
  if (warp == 1) {
    asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem),
                 "r"(kTmemCols));
  }
}

typedef CUresult (*EncodeFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                             const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                             const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                             CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeFn encode_fn() {
  static EncodeFn fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess && q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeFn>(p);
    cudaGetLastError();
  }
  return fn;
}

template <int TOK, int MH>
size_t umma_smem_bytes() {
  using RW = UmmaRows<MH>;
  return 1024 + (size_t)RW::Stages * (RW::A + UmmaTile<TOK>::BBytes + RW::W) +
         3 * RW::Stages * 8 + 16 + 16;
}

int umma_tok(uint32_t seq, uint32_t out, int mh);
// Output-row halves per CTA (UmmaRows): 2 when that grid still fills a wave
// of one CTA per SM, else 1 (measured, B200, 512 rows: 2560 -> 6912 58.5 vs
// 70.1 us, -> 13824 86.3 vs 131.7, -> 7680 59 vs 80; 6912 -> 2560, 70 CTAs
// with two halves, 53.5 vs 45.6).  NELISP_UMMA_MH=1 or 2 forces one.
int umma_mh(uint32_t seq, uint32_t out) {
  static const int forced = [] {
    const char *v = getenv("NELISP_UMMA_MH");
    const int m = v ? atoi(v) : 0;
    return m == 1 || m == 2 ? m : 0;
  }();
  if (forced) return forced;
  const uint32_t tok = (uint32_t)umma_tok(seq, out, 2);
  const uint64_t ctas = (uint64_t)((out + 2 * kUmmaM - 1) / (2 * kUmmaM)) * ((seq + tok - 1) / tok);
  return ctas >= 148u ? 2 : 1;
}

// Sequence rows per CTA for SEQ rows x OUT outputs: the height whose grid,
// rounded up to whole waves of one CTA per SM, costs the fewest MMA columns
// (waves x 3 TOK); ties keep 80.  NELISP_UMMA_TOK=64 or 80 forces one.
int umma_tok(uint32_t seq, uint32_t out, int mh) {
  static const int forced = [] {
    const char *v = getenv("NELISP_UMMA_TOK");
    const int t = v ? atoi(v) : 0;
    return t == 64 || t == 80 ? t : 0;
  }();
  if (forced) return forced;
  const uint64_t mt = (out + kUmmaM * mh - 1) / (kUmmaM * mh);
  auto cost = [&](uint32_t tok) {
    const uint64_t ctas = mt * ((seq + tok - 1) / tok);
    return ((ctas + 147) / 148) * tok;
  };
  return cost(64) < cost(80) ? 64 : 80;
}

uint32_t umma_cols_for(uint32_t seq, int tok) {
  return (seq + tok - 1) / tok * 3u * (uint32_t)tok;
}

}  // namespace

// Limb rows of the B operand in the workspace: enough for either tile height.
uint32_t umma_cols_padded(uint32_t seq) {
  const uint32_t a = umma_cols_for(seq, 64), b = umma_cols_for(seq, 80);
  return a > b ? a : b;
}

size_t ternary_umma_ws_bytes(uint32_t seq, uint32_t cols) {
  return align256((size_t)umma_cols_padded(seq) * cols) + align256((size_t)seq * 4) * 2;
}

bool ternary_umma_applies(uint32_t count, uint32_t seq, uint32_t cols, bool per_block) {
  return count == 1 && !per_block && seq > 16 && cols % kUmmaK == 0 && cols >= kUmmaK;
}

cudaError_t ternary_umma_launch(const float *X, const uint32_t *WP, const float *S,
                                const float *BIAS, float *Y, uint32_t seq, uint32_t out,
                                uint32_t cols, void *ws, size_t ws_bytes, cudaStream_t st,
                                bool *launched) {
  *launched = false;
  EncodeFn enc = encode_fn();
  if (!enc || !ws || ws_bytes < ternary_umma_ws_bytes(seq, cols) || ((uintptr_t)WP & 15u) ||
      ((uintptr_t)X & 15u))
    return cudaSuccess;
  const uint32_t ncol = umma_cols_padded(seq);
  int8_t *XB = reinterpret_cast<int8_t *>(ws);
  float *rowinv = reinterpret_cast<float *>((char *)ws + align256((size_t)ncol * cols));
  int *rowflag = reinterpret_cast<int *>((char *)rowinv + align256((size_t)seq * 4));
  const int mh = umma_mh(seq, out);
  const int tok = umma_tok(seq, out, mh);
  CUtensorMap mw, mb;
  {
    const cuuint64_t dims[2] = {cols / 16u, out}, strides[1] = {(cuuint64_t)cols / 16u * 4u};
    const cuuint32_t box[2] = {kUmmaK / 16, (cuuint32_t)(kUmmaM * mh)}, es[2] = {1, 1};
    if (enc(&mw, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<uint32_t *>(WP), dims, strides,
            box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return cudaSuccess;
  }
  {
    const cuuint64_t dims[2] = {cols, ncol}, strides[1] = {cols};
    const cuuint32_t box[2] = {kUmmaK, 3u * (uint32_t)tok}, es[2] = {1, 1};
    if (enc(&mb, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, XB, dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return cudaSuccess;
  }
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaSuccess;
#define NL_SMEM(T, M)                                                                     \
    if (e == cudaSuccess)                                                                 \
      e = cudaFuncSetAttribute(ternary_umma_kernel<T, M>,                                  \
                               cudaFuncAttributeMaxDynamicSharedMemorySize,                \
                               (int)umma_smem_bytes<T, M>());
    NL_SMEM(80, 1) NL_SMEM(64, 1) NL_SMEM(80, 2) NL_SMEM(64, 2)
#undef NL_SMEM
    if (e != cudaSuccess) return e;
    configured = true;
  }
  *launched = true;
  // rows 3*seq .. ncol of XB feed only MMA columns no output reads
  cudaError_t e = launch_k(umma_prep_kernel, dim3(seq), dim3(256), 0, st, false, X, cols, XB,
                           rowinv, rowflag);
  if (e != cudaSuccess) return e;
  const dim3 grid((out + kUmmaM * mh - 1) / (kUmmaM * mh), (seq + tok - 1) / tok);
#define NL_GEMM(T, M)                                                                     \
  e = launch_pdl(ternary_umma_kernel<T, M>, grid, dim3(UmmaRows<M>::Threads),              \
                 umma_smem_bytes<T, M>(), st, mw, mb, X, WP, S, BIAS, (const float *)rowinv, \
                 (const int *)rowflag, Y, seq, out, cols, wait_flag_device())
  if (mh == 2) {
    if (tok == 64) NL_GEMM(64, 2);
    else NL_GEMM(80, 2);
  } else {
    if (tok == 64) NL_GEMM(64, 1);
    else NL_GEMM(80, 1);
  }
#undef NL_GEMM
  count_launches(2);
  return e != cudaSuccess ? e : cudaPeekAtLastError();
}

}  // namespace nl

// k_ternary_tc.cu -- the streaming ternary GEMV (up to 16 sequence rows, many
// output rows) on the 5th-generation tensor cores, weights expanded straight
// into tensor memory.
//
// Y[s, o] = S[o] * sum_k t(o, k) X[s, k] (+ BIAS[o]): the per-row-scale form
// of ternary-rows (lisp/nelisp-gpu-kernels.el:713-746), computed exactly as
// an integer dot product and rounded once, bit-identical to the other fast
// paths of this library.
//
// Weight operand with one logic op per four weights.  A two-bit code c of
// the reference format (00 -> 0, 01 -> +1, 11 -> -1, 10 -> -2) XOR 0b10 is
// c' = t + 2 in {0..3}.  Field f (bits 2f..2f+1) of every byte of a packed
// word is selected by one LOP3, (w & (3 << 2f) * 0x01010101) ^
// (2 << 2f) * 0x01010101, whose bytes read as unsigned integers are
// 4^f * c'.  These bytes are the A operand (u8) of tcgen05.mma.kind::i8 as
// they are; the B operand (s8) carries, at the same K position, the balanced
// int8 limbs of xq * 4^(3-f), xq the activation scaled by a power of two
// into [2^21, 2^22) and rounded (the prep below).  Every product is then
// 64 * c' * xq, four limbs recombine exactly in int64, and
//     sum_k t * xq = (sum_k 64 c' xq) / 64 - 2 * sum_k xq,
// the last sum coming from the prep as well.  A K position inside a
// 128-column stage is 16 j + 4 f + b for byte b, field f of packed word j
// (the B rows are written in that order).
//
// One CTA per SM, persistent over (problem, 128-row tile) items, 15 or 17
// warps;
// a stage is 256 columns (8 KB of packed weights):
//   warp 0      TMA producer: the packed weight tile (128 rows x 64 bytes,
//               64-byte swizzle) and the int8 limb tile (two 128-column
//               halves, 128-byte swizzle) per stage, an 8-stage mbarrier ring;
//   warps 2-5,  two groups of four expanding warps, taking alternate stages,
//   warps 6-9   one thread per weight row: four 16-byte shared loads, 64
//               LOP3s, two tcgen05.st of 32 columns into a TMEM A stage;
//   warps 1,    four MMA issuers (two for N > 32) taking stages in turn
//   14 (15, 16) (warp 1 also allocates TMEM): eight 128 x N x 32 MMAs per
//               stage with A in TMEM and B in shared memory, each issuer
//               into its own accumulator of a double-buffered set;
//   warps 10-13 read an item's accumulators back (tcgen05.ld), add the two
//               issuers' sums, recombine the limbs and write Y while the next
//               item accumulates.
// The CUDA cores only expand weights; every MMA is issued by one thread and
// runs asynchronously.  Every mbarrier wait is bounded; one that gives up
// sets the library's host-mapped wait flag, which the synchronising entry
// points report.

#include <cooperative_groups.h>
#include <cuda.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include "nl_internal.h"
#include "ternary_prep.cuh"

namespace nl {
namespace cg = cooperative_groups;
namespace {

constexpr int kTcM = 128;                 // output rows per item
constexpr int kTcK = 256;                 // columns per stage (eight MMAs)
constexpr int kTcStages = 8;              // shared-memory ring
constexpr int kTcAStages = 4;             // TMEM A stages, 64 columns each
constexpr uint32_t kTcWBytes = kTcM * kTcK / 4;   // packed weights per stage
constexpr uint32_t kTcTmemCols = 512;     // one CTA per SM
constexpr uint32_t kTcWaitRounds = 4096;
constexpr uint32_t kTcSuspendNs = 1000000;
constexpr uint32_t kTcMaxCols = 65536;    // keeps every int32 limb sum exact
constexpr uint32_t kTcMinSeq = 6;

// ---- activation format -------------------------------------------------------
// For COUNT problems of SEQ rows: xb [count][rows_b][cols] int8 limb rows
// (row 4s + l = limb l of sequence row s, K-permuted and field-scaled as in
// the file comment), then rowinv / rowflag [count][16], then the per-CTA
// partial sums of xq, rowsum [count][16][kRowCluster] (int64).
__host__ __device__ inline uint32_t tc_rows_b(uint32_t seq) { return 8u * ((4u * seq + 7u) / 8u); }
__host__ __device__ inline uint32_t tc_mma_n(uint32_t seq) { return 16u * ((4u * seq + 15u) / 16u); }

struct TcPrep {
  int8_t *xb;
  float *rowinv;
  int *rowflag;
  long long *rowsum;
};
__host__ __device__ inline size_t tc_xb_bytes(uint32_t count, uint32_t seq, uint32_t cols) {
  return align256((size_t)count * tc_rows_b(seq) * cols);
}
__host__ __device__ inline TcPrep tc_prep_at(void *ws, uint32_t count, uint32_t seq,
                                             uint32_t cols) {
  char *b = (char *)ws;
  TcPrep p;
  p.xb = (int8_t *)b;
  b += tc_xb_bytes(count, seq, cols);
  p.rowinv = (float *)b;
  b += align256((size_t)count * 16 * 4);
  p.rowflag = (int *)b;
  b += align256((size_t)count * 16 * 4);
  p.rowsum = (long long *)b;
  return p;
}

// ---- PTX wrappers --------------------------------------------------------------
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
// Bounded wait for phase PARITY: each try_wait suspends until the phase
// completes or the hint runs out; after kTcWaitRounds rounds the wait gives
// up and records it in the host-visible flag ERR.
__device__ __forceinline__ bool bar_wait(uint64_t *b, uint32_t parity, int *err) {
  for (uint32_t i = 0; i < kTcWaitRounds; i++) {
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done) : "r"(su32(b)), "r"(parity), "r"(kTcSuspendNs) : "memory");
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
__device__ __forceinline__ uint4 lds128(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];\n"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
  return v;
}
// (a & b) ^ c in one LOP3.
__device__ __forceinline__ uint32_t and_xor(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t r;
  asm("lop3.b32 %0, %1, %2, %3, 0x6a;\n" : "=r"(r) : "r"(a), "r"(b), "r"(c));
  return r;
}
// K-major operand, 128-byte swizzle (rows of 128 bytes, 8-row groups 1024 apart).
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr) {
  return (uint64_t)((addr >> 4) & 0x3FFFu) | (1ull << 16) | ((uint64_t)(1024 >> 4) << 32) |
         (1ull << 46) | (2ull << 61);
}
__device__ __forceinline__ void mma_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc,
                                       uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::i8 [%0], [%1], %2, %3, p;\n}\n" ::"r"(tmem_d),
      "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate));
}
__device__ __forceinline__ void mma_commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(
                   su32(bar)) : "memory");
}
__device__ __forceinline__ void fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
}
__device__ __forceinline__ void fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,"
      "%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};\n" ::"r"(
          taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
      "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]),
      "r"(v[15]), "r"(v[16]), "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]),
      "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]),
      "r"(v[29]), "r"(v[30]), "r"(v[31])
      : "memory");
}
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t *v) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,"
      "%15}, [%16];\n"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
        "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]),
        "=r"(v[14]), "=r"(v[15])
      : "r"(taddr));
}

// ---- prep ------------------------------------------------------------------------
// Packed word W (16 columns) of a row: xq = round(x * mul) (zeros when !OK),
// the four field-scaled limb rows at XB (row stride COLS) in the K order of
// the file comment; returns the sum of the sixteen xq.
__device__ __forceinline__ long long tc_quantize_word(const float *xr, uint32_t W, bool ok,
                                                      float mul, int8_t *xb, uint32_t cols) {
  int q[16];
  const float4 *src = reinterpret_cast<const float4 *>(xr + 16u * W);
#pragma unroll
  for (int v4 = 0; v4 < 4; v4++) {
    const float4 f = ok ? src[v4] : make_float4(0.f, 0.f, 0.f, 0.f);
    q[4 * v4] = __float2int_rn(f.x * mul);       // exact scaling, one rounding
    q[4 * v4 + 1] = __float2int_rn(f.y * mul);
    q[4 * v4 + 2] = __float2int_rn(f.z * mul);
    q[4 * v4 + 3] = __float2int_rn(f.w * mul);
  }
  long long part = 0;
  uint32_t bw[4][4] = {};                        // [limb][byte group f]
#pragma unroll
  for (int f = 0; f < 4; f++) {
#pragma unroll
    for (int b = 0; b < 4; b++) {
      const int v = q[4 * b + f] * (1 << (2 * (3 - f)));   // |v| <= 2^28
      part += q[4 * b + f];
      const int l0 = (int)(int8_t)(v & 0xff);
      int r = (v - l0) >> 8;
      const int l1 = (int)(int8_t)(r & 0xff);
      r = (r - l1) >> 8;
      const int l2 = (int)(int8_t)(r & 0xff);
      const int l3 = (r - l2) >> 8;
      bw[0][f] |= (uint32_t)(l0 & 0xff) << (8 * b);
      bw[1][f] |= (uint32_t)(l1 & 0xff) << (8 * b);
      bw[2][f] |= (uint32_t)(l2 & 0xff) << (8 * b);
      bw[3][f] |= (uint32_t)(l3 & 0xff) << (8 * b);
    }
  }
#pragma unroll
  for (int l = 0; l < 4; l++)
    *reinterpret_cast<uint4 *>(xb + (size_t)l * cols + 16u * W) =
        make_uint4(bw[l][0], bw[l][1], bw[l][2], bw[l][3]);
  return part;
}

// Few rows: grid (kRowCluster * seq, count), clusters of kRowCluster CTAs per row (the
// row maximum is combined through distributed shared memory in rank order, as
// in the chunked kernels' prep).  Each CTA quantizes its column slice, writes
// its four limb rows and its partial sum of xq.
constexpr int kTcPrepThreads = 128;
__global__ void __cluster_dims__(kRowCluster, 1, 1) __launch_bounds__(kTcPrepThreads)
tc_prep_kernel(const float *__restrict__ X, uint64_t x_stride, uint32_t seq, uint32_t cols,
               uint32_t count, void *ws) {
  pdl_trigger();                  // the GEMV may start streaming its weights
  pdl_wait();                     // X may come from the preceding kernel
  __shared__ float red[4];
  __shared__ long long lred[4];
  __shared__ float s_max;
  __shared__ int s_bad;
  cg::cluster_group cl = cg::this_cluster();
  const uint32_t rank = cl.block_rank();
  const uint32_t s = blockIdx.x / kRowCluster, z = blockIdx.y;
  const RowSlice sl = row_slice(cols, rank);
  const float *xr = X + z * x_stride + (size_t)s * cols;
  float m = 0.0f;
  int bad = 0;
  for (uint32_t i = sl.c0 + threadIdx.x; i < sl.c1; i += blockDim.x) {
    const float v = xr[i];
    m = fmaxf(m, fabsf(v));
    bad |= !isfinite(v);          // NaN is dropped by fmaxf; catch it here
  }
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  bad = __syncthreads_or(bad);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    s_max = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
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
  float mul = 0.0f, inv = 0.0f;
  const bool ok = row_scale(mm, anybad != 0, &mul, &inv, 3);
  TcPrep P = tc_prep_at(ws, count, seq, cols);
  if (rank == 0 && threadIdx.x == 0) {
    P.rowinv[z * 16 + s] = inv;
    P.rowflag[z * 16 + s] = !ok;
  }
  int8_t *xb = P.xb + ((size_t)z * tc_rows_b(seq) + 4u * s) * cols;
  long long part = 0;
  for (uint32_t W = sl.c0 / 16u + threadIdx.x; W < sl.c1 / 16u; W += blockDim.x)
    part += tc_quantize_word(xr, W, ok, mul, xb, cols);
  for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
  if ((threadIdx.x & 31) == 0) lred[threadIdx.x >> 5] = part;
  __syncthreads();
  if (threadIdx.x == 0)
    P.rowsum[(z * 16 + s) * kRowCluster + rank] = lred[0] + lred[1] + lred[2] + lred[3];
  cl.sync();                      // no CTA leaves while its maximum is read
}

// Many rows (enough to fill the GPU without splitting a row): one CTA of
// kTcRowThreads per row, no cluster; the row's sum of xq goes to partial slot
// 0 and the other slots are zeroed, so the GEMV reads the same layout.
constexpr int kTcRowThreads = 256;
__global__ void __launch_bounds__(kTcRowThreads)
tc_prep_rows_kernel(const float *__restrict__ X, uint64_t x_stride, uint32_t seq, uint32_t cols,
                    uint32_t count, void *ws) {
  pdl_trigger();
  pdl_wait();
  __shared__ float red[kTcRowThreads / 32];
  __shared__ long long lred[kTcRowThreads / 32];
  const uint32_t s = blockIdx.x, z = blockIdx.y;
  const float *xr = X + z * x_stride + (size_t)s * cols;
  float m = 0.0f;
  int bad = 0;
  for (uint32_t i = threadIdx.x; i < cols; i += blockDim.x) {
    const float v = xr[i];
    m = fmaxf(m, fabsf(v));
    bad |= !isfinite(v);
  }
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  bad = __syncthreads_or(bad);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  float mm = 0.0f;
#pragma unroll
  for (int w = 0; w < kTcRowThreads / 32; w++) mm = fmaxf(mm, red[w]);
  float mul = 0.0f, inv = 0.0f;
  const bool ok = row_scale(mm, bad != 0, &mul, &inv, 3);
  TcPrep P = tc_prep_at(ws, count, seq, cols);
  if (threadIdx.x == 0) {
    P.rowinv[z * 16 + s] = inv;
    P.rowflag[z * 16 + s] = !ok;
  }
  int8_t *xb = P.xb + ((size_t)z * tc_rows_b(seq) + 4u * s) * cols;
  long long part = 0;
  for (uint32_t W = threadIdx.x; W < cols / 16u; W += blockDim.x)
    part += tc_quantize_word(xr, W, ok, mul, xb, cols);
  for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
  if ((threadIdx.x & 31) == 0) lred[threadIdx.x >> 5] = part;
  __syncthreads();
  if (threadIdx.x < kRowCluster) {
    long long t = 0;
    if (threadIdx.x == 0)
      for (int w = 0; w < kTcRowThreads / 32; w++) t += lred[w];
    P.rowsum[(z * 16 + s) * kRowCluster + threadIdx.x] = t;
  }
}

// ---- the GEMV ---------------------------------------------------------------------
// Issue cost, measured on B200: one thread issues a tcgen05.mma about every 52
// cycles whatever N is, while the tensor core finishes a 128 x 16 x 32 one in
// a few; two threads issuing in parallel halve the time.  A stage is
// therefore 256 columns (eight MMAs, so its waits and commits are shared by
// more MMAs), stages are issued in turn by NI issuing warps, each with its
// own accumulators, and alternate between two groups of four expanding warps.
__host__ __device__ inline size_t tc_smem_bytes(uint32_t n) {
  return 1024 + (size_t)kTcStages * (2u * n * 128u + kTcWBytes) +
         8 * (2 * kTcStages + 2 * kTcAStages + 2 * 2 + 4) + 16;
}

// NI issuing warps: 4 where four accumulator pairs fit next to the A stages
// in TMEM (N <= 32), else 2.
template <int N>
struct TcIssuers {
  static constexpr int NI = N <= 32 ? 4 : 2;
  static constexpr int kThreads = 32 * (13 + NI);
};

template <int N>
__global__ void __launch_bounds__(TcIssuers<N>::kThreads, 1)
ternary_tc_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmB,
                  const float *__restrict__ X, uint64_t x_stride, const uint32_t *__restrict__ WP,
                  uint64_t w_stride, const float *__restrict__ SCALE, uint64_t s_stride,
                  const float *__restrict__ BIAS, float *__restrict__ Y, uint64_t y_stride,
                  uint32_t seq, uint32_t out, uint32_t cols, uint64_t limit, void *ws,
                  uint32_t count, int *err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *base = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  constexpr uint32_t kBHalf = N * 128u;                       // one 128-column half of B
  uint8_t *sB = base;                                         // stages x 2 halves (1024-aligned)
  uint8_t *sW = sB + kTcStages * 2 * kBHalf;                  // stages x 8 KB
  uint64_t *full = reinterpret_cast<uint64_t *>(sW + kTcStages * kTcWBytes);
  uint64_t *empty = full + kTcStages;
  uint64_t *aready = empty + kTcStages;
  uint64_t *tfree = aready + kTcAStages;
  uint64_t *dfull = tfree + kTcAStages;
  uint64_t *dempty = dfull + 2;
  uint64_t *fin = dempty + 2;                                 // one per issuer
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(fin + 4);
  constexpr int NI = TcIssuers<N>::NI;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t tiles = (out + kTcM - 1) / kTcM;
  const uint32_t items = tiles * count;
  const uint32_t nk = (cols + kTcK - 1) / kTcK;
  const uint32_t mine = items > blockIdx.x ? (items - blockIdx.x + gridDim.x - 1) / gridDim.x : 0u;
  const uint32_t rows_b = tc_rows_b(seq);
  // u8 (A) x s8 (B) -> s32, both K-major, M = 128, N.
  const uint32_t idesc = (2u << 4) | (1u << 10) | ((uint32_t)(N >> 3) << 17) |
                         ((uint32_t)(kTcM >> 4) << 24);

  if (threadIdx.x == 0) {
    for (int i = 0; i < kTcStages; i++) {
      bar_init(&full[i], 1);
      bar_init(&empty[i], 1);      // the stage's MMAs have completed
    }
    for (int i = 0; i < kTcAStages; i++) {
      bar_init(&aready[i], 4);     // the four warps of the stage's expanding group
      bar_init(&tfree[i], 1);
    }
    for (int i = 0; i < 2; i++) {
      bar_init(&dfull[i], NI);     // every issuer
      bar_init(&dempty[i], 4);
    }
    for (int i = 0; i < NI; i++) bar_init(&fin[i], 1);
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(
                     su32(tmem_slot)), "r"(kTcTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::);
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tA = tmem;                          // A stages: 64 columns each
  const uint32_t tD = tmem + 64u * kTcAStages;       // accumulators [buffer][issuer]: N each
  const uint32_t total = mine * nk;

  if (warp == 0) {
    // ---- producer ----
    if (lane == 0) {
      // The weights of the first stages are requested before waiting for the
      // prep kernel (launch_pdl); the weights are not written by it.
      const uint32_t pre = total < (uint32_t)kTcStages ? total : (uint32_t)kTcStages;
      const uint32_t bbytes = rows_b * 128u;
      uint32_t g = 0;
      for (; g < total; g++) {
        const int st = (int)(g % kTcStages);
        if (g >= (uint32_t)kTcStages && !bar_wait(&empty[st], ((g / kTcStages) - 1) & 1, err))
          break;
        const uint32_t it = blockIdx.x + (g / nk) * gridDim.x, kt = g % nk;
        const uint32_t z = it / tiles, tile = it % tiles;
        bar_expect(&full[st], kTcWBytes + 2u * bbytes);
        tma2d(sW + st * kTcWBytes, &tmW, (int)(kt * (kTcK / 16)), (int)(z * out + tile * kTcM),
              &full[st]);
        if (g >= pre) {
          tma2d(sB + st * 2 * kBHalf, &tmB, (int)(kt * kTcK), (int)(z * rows_b), &full[st]);
          tma2d(sB + st * 2 * kBHalf + kBHalf, &tmB, (int)(kt * kTcK + 128), (int)(z * rows_b),
                &full[st]);
        } else if (g + 1 == pre) {
          pdl_wait();
          for (uint32_t k = 0; k < pre; k++) {
            const uint32_t itk = blockIdx.x + (k / nk) * gridDim.x, x = (k % nk) * kTcK;
            const int y = (int)((itk / tiles) * rows_b);
            tma2d(sB + k * 2 * kBHalf, &tmB, (int)x, y, &full[k]);
            tma2d(sB + k * 2 * kBHalf + kBHalf, &tmB, (int)(x + 128), y, &full[k]);
          }
        }
      }
      // Leave only when the last copies have landed (bounded).
      for (uint32_t k = g > (uint32_t)kTcStages ? g - kTcStages : 0; k < g; k++)
        bar_wait(&full[k % kTcStages], (k / kTcStages) & 1, err);
    }
  } else if (warp == 1 || warp >= 14) {
    // ---- MMA issuers (warps 1, 14, 15, 16): issuer p takes the stages g
    // with g % NI == p ----
    if (lane == 0) {
      const uint32_t p = warp == 1 ? 0u : (uint32_t)(warp - 13);
      bool ok = true;
      for (uint32_t i = 0; i < mine && ok; i++) {
        const uint32_t d = i & 1u;
        const uint32_t acc_d = tD + (NI * d + p) * N;
        if (i >= 2 && !bar_wait(&dempty[d], ((i >> 1) - 1) & 1, err)) break;
        fence_after();
        bool first = true;
        for (uint32_t kt = 0; kt < nk; kt++) {
          const uint32_t g = i * nk + kt;
          if (g % NI != p) continue;
          const int st = (int)(g % kTcStages), ts = (int)(g % kTcAStages);
          if (!bar_wait(&full[st], (g / kTcStages) & 1, err) ||
              !bar_wait(&aready[ts], (g / kTcAStages) & 1, err)) {
            ok = false;
            break;
          }
          fence_after();
          const uint32_t b0 = su32(sB + st * 2 * kBHalf);
#pragma unroll
          for (int k = 0; k < kTcK / 32; k++)
            mma_ts(acc_d, tA + 64u * ts + 8u * k,
                   smem_desc(b0 + (uint32_t)(k >> 2) * kBHalf + 32u * (k & 3)), idesc,
                   (!first || k > 0) ? 1u : 0u);
          first = false;
          mma_commit(&empty[st]);     // the stage's shared memory is free once these are done
          mma_commit(&tfree[ts]);     // and so is the TMEM A stage
        }
        if (ok) mma_commit(&dfull[d]);
      }
      mma_commit(&fin[p]);
      bar_wait(&fin[p], 0, err);      // every MMA of this issuer has completed
    }
  } else if (warp < 10) {
    // ---- expand the weights into TMEM: group q (warps 2-5, 6-9) takes the
    // stages g with g % 2 == q, one thread per weight row ----
    const uint32_t q = warp < 6 ? 0u : 1u;
    const uint32_t quad = (uint32_t)(warp & 3);
    const uint32_t r = quad * 32u + (uint32_t)lane;
    const uint32_t lane_base = (quad * 32u) << 16;
    // 64-byte swizzle: the 16-byte chunk c of row r sits at chunk c ^ ((r >> 1) & 3).
    const uint32_t sw = (r >> 1) & 3u;
    const uint32_t wrow = su32(sW) + r * 64u;
    for (uint32_t g = q; g < total; g += 2) {
      const int st = (int)(g % kTcStages), ts = (int)(g % kTcAStages);
      if (!bar_wait(&full[st], (g / kTcStages) & 1, err)) break;
      uint32_t w16[16];
#pragma unroll
      for (int c = 0; c < 4; c++) {
        const uint4 v = lds128(wrow + st * kTcWBytes + (((uint32_t)c ^ sw) << 4));
        w16[4 * c] = v.x; w16[4 * c + 1] = v.y; w16[4 * c + 2] = v.z; w16[4 * c + 3] = v.w;
      }
      if (g >= (uint32_t)kTcAStages && !bar_wait(&tfree[ts], ((g / kTcAStages) - 1) & 1, err))
        break;
      fence_after();
#pragma unroll
      for (int h = 0; h < 2; h++) {
        uint32_t a[32];
#pragma unroll
        for (int j = 0; j < 8; j++) {
          const uint32_t w = w16[8 * h + j];
          a[4 * j + 0] = and_xor(w, 0x03030303u, 0x02020202u);
          a[4 * j + 1] = and_xor(w, 0x0C0C0C0Cu, 0x08080808u);
          a[4 * j + 2] = and_xor(w, 0x30303030u, 0x20202020u);
          a[4 * j + 3] = and_xor(w, 0xC0C0C0C0u, 0x80808080u);
        }
        tmem_st32(tA + lane_base + 64u * ts + 32u * h, a);
      }
      asm volatile("tcgen05.wait::st.sync.aligned;\n" ::: "memory");
      fence_before();
      __syncwarp();
      if (lane == 0) bar_arrive(&aready[ts]);
    }
  } else if (warp < 14) {
    // ---- epilogue: accumulators -> Y ----
    pdl_wait();                                    // the prep's scales, flags and sums
    const uint32_t quad = (uint32_t)(warp & 3);
    const uint32_t lane_base = (quad * 32u) << 16;
    TcPrep P = tc_prep_at(ws, count, seq, cols);
    const uint32_t wng = cols / 16u, nblk = cols / 128u;
    for (uint32_t i = 0; i < mine; i++) {
      const uint32_t d = i & 1u;
      const uint32_t it = blockIdx.x + i * gridDim.x;
      const uint32_t z = it / tiles, tile = it % tiles;
      const uint32_t o = tile * kTcM + quad * 32u + (uint32_t)lane;
      const float *Sz = SCALE + z * s_stride;
      const float sc = o < out ? __ldg(Sz + o) : 0.0f;
      const float bi = (BIAS && o < out) ? __ldg(BIAS + o) : 0.0f;
      float e_rinv = 0.0f;
      int e_flag = 0;
      long long e_sum = 0;
      if ((uint32_t)lane < seq) {
        e_rinv = P.rowinv[z * 16 + lane];
        e_flag = P.rowflag[z * 16 + lane];
        const long long *rs = P.rowsum + (size_t)(z * 16 + lane) * kRowCluster;
#pragma unroll
        for (int k = 0; k < kRowCluster; k++) e_sum += rs[k];
      }
      if (!bar_wait(&dfull[d], (i >> 1) & 1, err)) break;
      fence_after();
      // Issuer p has a stage in this item unless the item is shorter than
      // NI stages and none of its stages falls to p.
      const uint32_t g0 = i * nk;
      uint32_t v[N];
#pragma unroll
      for (int c = 0; c < N; c++) v[c] = 0u;
#pragma unroll
      for (int p = 0; p < NI; p++) {
        if (nk < (uint32_t)NI && ((uint32_t)p + NI - g0 % NI) % NI >= nk) continue;
#pragma unroll
        for (int c = 0; c < N; c += 16) {
          uint32_t u[16];
          tmem_ld16(tD + lane_base + (NI * d + (uint32_t)p) * N + c, u);
          asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
#pragma unroll
          for (int j = 0; j < 16; j++) v[c + j] += u[j];   // exact int32 partial sums
        }
      }
      fence_before();
      __syncwarp();
      if (lane == 0) bar_arrive(&dempty[d]);       // the accumulators may be reused
      float *Yz = Y + z * y_stride;
#pragma unroll
      for (int s = 0; s < N / 4; s++) {
        if ((uint32_t)s >= seq) break;
        const float ri = __shfl_sync(0xffffffffu, e_rinv, s);
        const int fl = __shfl_sync(0xffffffffu, e_flag, s);
        const long long sx = __shfl_sync(0xffffffffu, e_sum, s);
        if (o >= out || fl) continue;
        const long long tot = (long long)(int)v[4 * s] + 256ll * (int)v[4 * s + 1] +
                              65536ll * (int)v[4 * s + 2] + 16777216ll * (int)v[4 * s + 3];
        const long long dot = (tot >> 6) - 2 * sx;   // exact: tot = 64 sum c' xq
        float y = ((float)dot * ri) * sc;
        if (BIAS) y = bi + y;
        const uint64_t oi = (uint64_t)s * out + o;
        if (oi < limit) Yz[oi] = y;
      }
      if (__any_sync(0xffffffffu, e_flag != 0)) {
        // Rows the limbs cannot represent: the generic arithmetic, one row of
        // this warp's 32 at a time, all lanes.
        const float *Xz = X + z * x_stride;
        const uint32_t *Wz = WP + z * w_stride;
        for (uint32_t s = 0; s < seq; s++) {
          if (!__shfl_sync(0xffffffffu, e_flag, (int)s)) continue;
          for (uint32_t rr = 0; rr < 32u; rr++) {
            const uint32_t orow = tile * kTcM + quad * 32u + rr;
            if (orow >= out) break;
            float acc1[1];
            ternary_row_generic<1>(Xz, Wz + (uint64_t)orow * wng, nullptr, false,
                                   __ldg(Sz + orow), (int)s, 1, cols, nblk, wng, acc1);
            const uint64_t oi = (uint64_t)s * out + orow;
            if (lane == 0 && oi < limit) Yz[oi] = (BIAS ? __ldg(BIAS + orow) : 0.0f) + acc1[0];
          }
        }
      }
    }
  }
  fence_before();
  __syncthreads();
  if (warp == 1) {
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem),
                 "r"(kTcTmemCols));
  }
}

typedef CUresult (*EncodeFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                             const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                             const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                             CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeFn tc_encode_fn() {
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

template <int N>
cudaError_t launch_tc_n(const CUtensorMap &mw, const CUtensorMap &mb, uint32_t items,
                        cudaStream_t st, const float *X, uint64_t xs, const uint32_t *WP,
                        uint64_t wst, const float *S, uint64_t ss, const float *B, float *Y,
                        uint64_t ys, uint32_t seq, uint32_t out, uint32_t cols, uint64_t limit,
                        void *ws, uint32_t count) {
  static int per_sm = 0;
  const size_t smem = tc_smem_bytes(N);
  if (!per_sm) {
    cudaError_t e = cudaFuncSetAttribute(ternary_tc_kernel<N>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    int n = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, ternary_tc_kernel<N>,
                                                      TcIssuers<N>::kThreads, smem);
    if (e != cudaSuccess) return e;
    // TMEM: 512 columns per SM.
    per_sm = n < 1 ? 1 : (n > (int)(512 / kTcTmemCols) ? (int)(512 / kTcTmemCols) : n);
    (void)per_sm;
  }
  int sms = 148, dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess)
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  cudaGetLastError();
  const uint32_t cap = (uint32_t)(per_sm * sms);
  const uint32_t grid = items < cap ? items : cap;
  return launch_pdl(ternary_tc_kernel<N>, dim3(grid), dim3(TcIssuers<N>::kThreads), smem, st, mw,
                    mb, X, xs,
                    WP, wst, S, ss, B, Y, ys, seq, out, cols, limit, ws, count,
                    wait_flag_device());
}

}  // namespace

size_t ternary_tc_ws_bytes(uint32_t count, uint32_t seq, uint32_t cols) {
  if (seq == 0 || seq > 16u) return 0;
  return tc_xb_bytes(count, seq, cols) + 2 * align256((size_t)count * 16 * 4) +
         align256((size_t)count * 16 * kRowCluster * 8);
}

bool ternary_tc_applies(uint32_t count, uint32_t seq, uint32_t out, uint32_t cols,
                        bool per_block, uint64_t w_stride) {
  static const bool on = [] {
    const char *v = getenv("NELISP_TERNARY_PATH");   // ring / tma: the chunked kernels
    return !(v && (strcmp(v, "ring") == 0 || strcmp(v, "tma") == 0));
  }();
  // tc: this kernel from five rows up.  Up to four rows the other paths
  // carry activations to 30 bits (four limbs); this kernel's format has 22.
  static const bool forced = [] {
    const char *v = getenv("NELISP_TERNARY_PATH");
    return v && strcmp(v, "tc") == 0;
  }();
  if (forced && !per_block && seq >= 5u && seq <= 16u && cols % 128u == 0 && cols >= kTcK &&
      cols <= kTcMaxCols && (count == 1 || w_stride == (uint64_t)out * (cols / 16u)))
    return true;
  // Below six rows the register-fed mma.sync kernels stream faster: the A
  // operand of a tcgen05 MMA is re-read from TMEM for every MMA, and a GEMV
  // (N = 4 limbs per row) reuses it too little (measured crossover, B200).
  return on && !per_block && seq >= kTcMinSeq && seq <= 16u && cols % 128u == 0 && cols >= kTcK &&
         cols <= kTcMaxCols && (count == 1 || w_stride == (uint64_t)out * (cols / 16u));
}

cudaError_t ternary_tc_launch(uint32_t count, const float *X, uint64_t x_stride,
                              const uint32_t *WP, uint64_t w_stride, const float *SCALE,
                              uint64_t s_stride, const float *BIAS, float *Y, uint64_t y_stride,
                              uint32_t seq, uint32_t out, uint32_t cols, uint64_t limit, void *ws,
                              size_t ws_bytes, cudaStream_t st, bool *launched) {
  *launched = false;
  EncodeFn enc = tc_encode_fn();
  if (!enc || !ws || ws_bytes < ternary_tc_ws_bytes(count, seq, cols) || ((uintptr_t)WP & 15u) ||
      ((uintptr_t)X & 15u) || (x_stride % 4u) || ((uintptr_t)ws & 255u))
    return cudaSuccess;
  const uint32_t wng = cols / 16u, rows_b = tc_rows_b(seq);
  CUtensorMap mw, mb;
  {
    const cuuint64_t dims[2] = {wng, (cuuint64_t)count * out};
    const cuuint64_t strides[1] = {(cuuint64_t)wng * 4u};
    const cuuint32_t box[2] = {kTcK / 16, kTcM}, es[2] = {1, 1};
    if (enc(&mw, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<uint32_t *>(WP), dims, strides,
            box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return cudaSuccess;
  }
  {
    const cuuint64_t dims[2] = {cols, (cuuint64_t)count * rows_b}, strides[1] = {cols};
    const cuuint32_t box[2] = {128, rows_b}, es[2] = {1, 1};
    if (enc(&mb, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, ws, dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return cudaSuccess;
  }
  *launched = true;
  // Few rows: a cluster per row splits it over 8 SMs; enough rows to fill
  // the GPU: a CTA per row.
  cudaError_t e;
  if ((uint64_t)seq * count >= 2u * 148u)
    e = launch_k(tc_prep_rows_kernel, dim3(seq, count), dim3(kTcRowThreads), 0, st, false, X,
                 x_stride, seq, cols, count, ws);
  else
    e = launch_k(tc_prep_kernel, dim3(kRowCluster * seq, count), dim3(kTcPrepThreads), 0, st,
                 false, X, x_stride, seq, cols, count, ws);
  if (e != cudaSuccess) return e;
  const uint32_t items = ((out + kTcM - 1) / kTcM) * count;
  switch (tc_mma_n(seq)) {
    case 16: e = launch_tc_n<16>(mw, mb, items, st, X, x_stride, WP, w_stride, SCALE, s_stride, BIAS, Y, y_stride, seq, out, cols, limit, ws, count); break;
    case 32: e = launch_tc_n<32>(mw, mb, items, st, X, x_stride, WP, w_stride, SCALE, s_stride, BIAS, Y, y_stride, seq, out, cols, limit, ws, count); break;
    case 48: e = launch_tc_n<48>(mw, mb, items, st, X, x_stride, WP, w_stride, SCALE, s_stride, BIAS, Y, y_stride, seq, out, cols, limit, ws, count); break;
    default: e = launch_tc_n<64>(mw, mb, items, st, X, x_stride, WP, w_stride, SCALE, s_stride, BIAS, Y, y_stride, seq, out, cols, limit, ws, count); break;
  }
  count_launches(2);
  return e != cudaSuccess ? e : cudaPeekAtLastError();
}

}  // namespace nl

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
//    max|x| lands in [2^21, 2^22), rounded to an integer xq and split into
//    three balanced int8 limbs, xq = l0 + 256 l1 + 65536 l2.  The rounding is
//    the only inexact step (half a unit of 2^-22 of the row maximum, below
//    f32's own accumulation error over a row).  Limbs are written straight
//    into mma B-fragment order, so the main loop loads one uint2 per MMA.
//  * main: each warp owns 16 weight rows.  Lanes load the packed words
//    (8 bytes per row per 128-column block, 4 lanes per row), expand the
//    two-bit codes to int8 with three-instruction PRMT lookups
//    (00->0, 01->+1, 10->-2, 11->-1: the reference's sign-extending decode)
//    and issue mma.m16n8k32.s8 with int32 accumulation: the dot products are
//    exact.  N carries (sequence, limb) pairs: n = 3s + l.
//  * epilogue: the three limb sums of (row, s) are combined in int64,
//    converted once and scaled by 2^-e_s and the row's scale (per-row mode),
//    or flushed per 128-column block against BETA[o,b] (ternary-rows mode).
//
// The K order inside a block is permuted identically in the A (weights) and
// B (activations) fragments, which a dot product does not observe.
// Rows whose activations are non-finite or below 2^-104 cannot be scaled into
// int8 limbs; prep flags them and the epilogue recomputes those outputs on
// the CUDA cores with the generic kernel's arithmetic.

#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include "nl_internal.h"

namespace nl {
namespace {

constexpr int kMaxFastSeq = 16;  // 48 (s, limb) columns = 6 n-tiles of 8
constexpr int kWarps = 4;        // warps per CTA in the MMA kernel
constexpr int kDepth = 8;        // 128-column blocks in flight per warp

__device__ __forceinline__ float trit_of(uint32_t w, uint32_t f) {
  return (float)(((int32_t)(w << (30u - 2u * f))) >> 30);
}

// ---------------------------------------------------------------------------
// Generic CUDA-core path: any shape, the reference's semantics exactly
// (blocks b < nblk, words wi < min(wng, 8*nblk), fields i < cols).  One warp
// per output row; lanes take words, groups of eight lanes form a block.
// ---------------------------------------------------------------------------
template <int SB>
__device__ void ternary_row_generic(const float *__restrict__ X,
                                    const uint32_t *__restrict__ Wrow,
                                    const float *__restrict__ beta_row,
                                    bool per_block, float row_scale,
                                    int s0, int ns, uint32_t cols,
                                    uint32_t nblk, uint32_t wng,
                                    float acc[SB]) {
  const int lane = threadIdx.x & 31;
  for (int s = 0; s < SB; s++) acc[s] = 0.0f;
  const uint32_t nwords = 8u * nblk;
  for (uint32_t base = 0; base < nwords; base += 32) {
    uint32_t wi = base + lane;
    uint32_t w = (wi < wng && wi < nwords) ? __ldg(Wrow + wi) : 0u;
    float part[SB];
#pragma unroll
    for (int s = 0; s < SB; s++) part[s] = 0.0f;
    // Every field is multiplied, zeros included: 0 * inf is NaN in the
    // reference's arithmetic too.
    if (wi < wng && wi < nwords) {
      for (uint32_t f = 0; f < 16; f++) {
        uint32_t i = wi * 16u + f;
        if (i < cols) {
          float t = trit_of(w, f);
#pragma unroll
          for (int s = 0; s < SB; s++)
            if (s < ns) part[s] = fmaf(t, __ldg(X + (size_t)(s0 + s) * cols + i), part[s]);
        }
      }
    }
    // Sum within each group of eight lanes = one 128-column block.
#pragma unroll
    for (int s = 0; s < SB; s++) {
      float v = part[s];
      v += __shfl_xor_sync(0xffffffffu, v, 1);
      v += __shfl_xor_sync(0xffffffffu, v, 2);
      v += __shfl_xor_sync(0xffffffffu, v, 4);
      part[s] = v;
    }
    uint32_t b = wi / 8u;
    if ((lane & 7) == 0 && b < nblk) {
      float sc = per_block ? __ldg(beta_row + b) : 1.0f;
#pragma unroll
      for (int s = 0; s < SB; s++) acc[s] = fmaf(sc, part[s], acc[s]);
    }
  }
#pragma unroll
  for (int s = 0; s < SB; s++) {
    float v = acc[s];
    v += __shfl_xor_sync(0xffffffffu, v, 8);
    v += __shfl_xor_sync(0xffffffffu, v, 16);
    acc[s] = per_block ? v : v * row_scale;
  }
}

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
// Fragment layout for one problem: uint2 frag[nt][blk][j][lane], where n-tile
// nt holds columns n = 8nt .. 8nt+7 (n = 3s + limb), blk is the 128-column
// block, j the k32 step within it and lane = 4*(n%8) + q.  Lane q of MMA j in
// block blk covers word w = 2q + (j>>1) of the block and, within it, codes
// 8*(j&1) + {0,2,4,6} (b0) and 8*(j&1) + {1,3,5,7} (b1).
struct PrepOut {
  uint2 *frag;      // NT * cols * 8 bytes
  float *rowinv;    // [kMaxFastSeq] 2^-e_s
  int *rowflag;     // [kMaxFastSeq] 1: compute (., s) on the CUDA cores
};

__host__ __device__ inline int n_tiles(int seq) { return (3 * seq + 7) / 8; }
__host__ __device__ inline size_t frag_bytes(int seq, uint32_t cols) {
  return (size_t)n_tiles(seq) * cols * 8u;
}
__host__ __device__ inline size_t align256(size_t b) {
  return (b + 255u) & ~(size_t)255u;
}
__host__ __device__ inline size_t prep_bytes(int seq, uint32_t cols) {
  return align256(frag_bytes(seq, cols)) + 256u;
}
__device__ inline PrepOut prep_at(void *ws, int seq, uint32_t cols, uint32_t z) {
  char *base = (char *)ws + (size_t)z * prep_bytes(seq, cols);
  PrepOut p;
  p.frag = (uint2 *)base;
  p.rowinv = (float *)(base + align256(frag_bytes(seq, cols)));
  p.rowflag = (int *)(p.rowinv + kMaxFastSeq);
  return p;
}

__device__ __forceinline__ uint32_t pack4(int a, int b, int c, int d) {
  return (uint32_t)(a & 0xff) | ((uint32_t)(b & 0xff) << 8) |
         ((uint32_t)(c & 0xff) << 16) | ((uint32_t)(d & 0xff) << 24);
}

// grid (ceil(8*NT/3), count), 256 threads.  CTA s handles sequence row s
// (rows s >= seq write the zero padding of the last n-tile).
__global__ void __launch_bounds__(256)
ternary_prep_kernel(const float *__restrict__ X, uint64_t x_stride,
                    uint32_t seq, uint32_t cols, void *ws) {
  const uint32_t s = blockIdx.x, z = blockIdx.y;
  const int NT = n_tiles((int)seq);
  PrepOut P = prep_at(ws, (int)seq, cols, z);
  const uint32_t nblk = cols / 128u;
  const float *xr = X + z * x_stride + (size_t)s * cols;
  __shared__ float red[8];
  __shared__ float s_mul;
  __shared__ int s_ok;
  bool live = s < seq;
  if (live) {
    float m = 0.0f;
    for (uint32_t i = threadIdx.x; i < cols; i += blockDim.x)
      m = fmaxf(m, fabsf(__ldg(xr + i)));
    // NaN is dropped by fmaxf; catch it (and inf) separately.
    int bad = 0;
    for (uint32_t i = threadIdx.x; i < cols; i += blockDim.x)
      bad |= !isfinite(__ldg(xr + i));
    bad = __syncthreads_or(bad);
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
    __syncthreads();
    if (threadIdx.x == 0) {
      float mm = 0.0f;
      for (int w = 0; w < (int)(blockDim.x >> 5); w++) mm = fmaxf(mm, red[w]);
      int ok = !bad;
      float mul = 0.0f, inv = 0.0f;
      if (ok && mm > 0.0f) {
        int E;
        frexpf(mm, &E);              // mm in [2^(E-1), 2^E)
        int e = 22 - E;              // mm * 2^e in [2^21, 2^22)
        if (e > 126 || e < -126) {
          ok = 0;                    // 2^e or 2^-e would leave the normals
        } else {
          mul = ldexpf(1.0f, e);
          inv = ldexpf(1.0f, -e);
        }
      }
      s_mul = mul;
      s_ok = ok;
      P.rowinv[s] = inv;
      P.rowflag[s] = !ok;
    }
    __syncthreads();
  }
  const float mul = live ? s_mul : 0.0f;
  const bool ok = live && s_ok;
  // One thread per 8-column group.
  const uint32_t ngroups = cols / 8u;
  for (uint32_t c8 = threadIdx.x; c8 < ngroups; c8 += blockDim.x) {
    int l[3][8];
    if (ok) {
      float4 v0 = *reinterpret_cast<const float4 *>(xr + 8u * c8);
      float4 v1 = *reinterpret_cast<const float4 *>(xr + 8u * c8 + 4u);
      float v[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
#pragma unroll
      for (int k = 0; k < 8; k++) {
        int q = __float2int_rn(v[k] * mul);   // exact scaling, one rounding
        int l0 = (int)(int8_t)(q & 0xff);
        int r = (q - l0) >> 8;
        int l1 = (int)(int8_t)(r & 0xff);
        int l2 = (r - l1) >> 8;               // |q| <= 2^22 -> |l2| <= 64
        l[0][k] = l0; l[1][k] = l1; l[2][k] = l2;
      }
    } else {
#pragma unroll
      for (int k = 0; k < 8; k++) l[0][k] = l[1][k] = l[2][k] = 0;
    }
    const uint32_t blk = c8 / 16u, wq = (c8 % 16u) / 2u, half = c8 & 1u;
    const uint32_t q = wq >> 1, j = ((wq & 1u) << 1) | half;
#pragma unroll
    for (int li = 0; li < 3; li++) {
      int n = 3 * (int)s + li;
      if (n >= 8 * NT) continue;
      uint2 fr;
      fr.x = pack4(l[li][0], l[li][2], l[li][4], l[li][6]);
      fr.y = pack4(l[li][1], l[li][3], l[li][5], l[li][7]);
      size_t idx = (((size_t)(n / 8) * nblk + blk) * 4u + j) * 32u + (uint32_t)(n % 8) * 4u + q;
      P.frag[idx] = fr;
    }
  }
}

// ---------------------------------------------------------------------------
// Fast path, step 2: the tensor-core GEMV.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mma_s8(int (&d)[4], uint32_t a0, uint32_t a1,
                                       uint32_t a2, uint32_t a3, uint2 b) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b.x), "r"(b.y));
}

// Two-bit code -> int8 lookup: bytes {0, +1, -2, -1} for codes 00,01,10,11.
constexpr uint32_t kTritLut = 0xFFFE0100u;

__device__ __forceinline__ uint32_t expand4(uint32_t sel) {
  return __byte_perm(kTritLut, 0u, sel);
}

template <int NT, bool PER_BLOCK>
__global__ void __launch_bounds__(kWarps * 32)
ternary_mma_kernel(const float *__restrict__ X, uint64_t x_stride,
                   const uint32_t *__restrict__ WP, uint64_t w_stride,
                   const float *__restrict__ SCALE, uint64_t s_stride,
                   const float *__restrict__ BIAS, float *__restrict__ Y,
                   uint64_t y_stride, uint32_t seq, uint32_t out,
                   uint32_t cols, uint64_t limit, void *ws) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, q = lane & 3;
  const uint32_t z = blockIdx.y;
  const uint32_t rg = blockIdx.x * kWarps + warp;          // 16-row group
  const uint32_t nblk = cols / 128u, wng = cols / 16u;
  __shared__ int s_acc[kWarps][16][8 * NT + 1];
  if (rg * 16u >= out) return;
  PrepOut P = prep_at(ws, (int)seq, cols, z);
  const uint32_t rA = min(rg * 16u + (uint32_t)g, out - 1u);
  const uint32_t rB = min(rg * 16u + (uint32_t)g + 8u, out - 1u);
  const uint32_t *Wz = WP + z * w_stride;
  const uint2 *pA = reinterpret_cast<const uint2 *>(Wz + (uint64_t)rA * wng) + q;
  const uint2 *pB = reinterpret_cast<const uint2 *>(Wz + (uint64_t)rB * wng) + q;
  const uint2 *frag = P.frag + lane;
  const float *Sz = SCALE + z * s_stride;

  int acc[NT][4];
  float yf[NT][4];
#pragma unroll
  for (int t = 0; t < NT; t++)
#pragma unroll
    for (int r = 0; r < 4; r++) { acc[t][r] = 0; yf[t][r] = 0.0f; }

  uint2 wa[kDepth], wb[kDepth];
#pragma unroll
  for (int u = 0; u < kDepth; u++) {
    if ((uint32_t)u < nblk) {
      wa[u] = __ldcs(pA + 4u * u);
      wb[u] = __ldcs(pB + 4u * u);
    }
  }
  for (uint32_t b0 = 0; b0 < nblk; b0 += kDepth) {
#pragma unroll
    for (int u = 0; u < kDepth; u++) {
      const uint32_t blk = b0 + u;
      if (blk < nblk) {
        const uint2 a = wa[u], c = wb[u];
        if (blk + kDepth < nblk) {
          wa[u] = __ldcs(pA + 4u * (blk + kDepth));
          wb[u] = __ldcs(pB + 4u * (blk + kDepth));
        }
        const uint32_t loA0 = a.x & 0x33333333u, hiA0 = (a.x >> 2) & 0x33333333u;
        const uint32_t loA1 = a.y & 0x33333333u, hiA1 = (a.y >> 2) & 0x33333333u;
        const uint32_t loB0 = c.x & 0x33333333u, hiB0 = (c.x >> 2) & 0x33333333u;
        const uint32_t loB1 = c.y & 0x33333333u, hiB1 = (c.y >> 2) & 0x33333333u;
        uint32_t A[4][4];
        A[0][0] = expand4(loA0);       A[0][1] = expand4(loB0);
        A[0][2] = expand4(hiA0);       A[0][3] = expand4(hiB0);
        A[1][0] = expand4(loA0 >> 16); A[1][1] = expand4(loB0 >> 16);
        A[1][2] = expand4(hiA0 >> 16); A[1][3] = expand4(hiB0 >> 16);
        A[2][0] = expand4(loA1);       A[2][1] = expand4(loB1);
        A[2][2] = expand4(hiA1);       A[2][3] = expand4(hiB1);
        A[3][0] = expand4(loA1 >> 16); A[3][1] = expand4(loB1 >> 16);
        A[3][2] = expand4(hiA1 >> 16); A[3][3] = expand4(hiB1 >> 16);
#pragma unroll
        for (int t = 0; t < NT; t++) {
          const uint2 *ft = frag + (((size_t)t * nblk + blk) * 4u) * 32u;
#pragma unroll
          for (int j = 0; j < 4; j++) {
            uint2 bf = __ldg(ft + j * 32);
            mma_s8(acc[t], A[j][0], A[j][1], A[j][2], A[j][3], bf);
          }
        }
        if (PER_BLOCK) {
          // BETA is per (row, 128-column block): flush the exact block sums.
          const float bA = __ldg(Sz + (uint64_t)rA * nblk + blk);
          const float bB = __ldg(Sz + (uint64_t)rB * nblk + blk);
#pragma unroll
          for (int t = 0; t < NT; t++) {
            yf[t][0] = fmaf((float)acc[t][0], bA, yf[t][0]);
            yf[t][1] = fmaf((float)acc[t][1], bA, yf[t][1]);
            yf[t][2] = fmaf((float)acc[t][2], bB, yf[t][2]);
            yf[t][3] = fmaf((float)acc[t][3], bB, yf[t][3]);
            acc[t][0] = acc[t][1] = acc[t][2] = acc[t][3] = 0;
          }
        }
      }
    }
  }

  // Epilogue: stage per-(row, n) results in shared memory, then combine the
  // three limbs of each (row, s).
  // Per-block results are float sums; they travel through the int array as
  // bit patterns.
#pragma unroll
  for (int t = 0; t < NT; t++) {
    const int v0 = PER_BLOCK ? __float_as_int(yf[t][0]) : acc[t][0];
    const int v1 = PER_BLOCK ? __float_as_int(yf[t][1]) : acc[t][1];
    const int v2 = PER_BLOCK ? __float_as_int(yf[t][2]) : acc[t][2];
    const int v3 = PER_BLOCK ? __float_as_int(yf[t][3]) : acc[t][3];
    s_acc[warp][g][8 * t + 2 * q] = v0;
    s_acc[warp][g][8 * t + 2 * q + 1] = v1;
    s_acc[warp][g + 8][8 * t + 2 * q] = v2;
    s_acc[warp][g + 8][8 * t + 2 * q + 1] = v3;
  }
  __syncwarp();
  float *Yz = Y + z * y_stride;
  bool any_flag = false;
  for (uint32_t s = 0; s < seq; s++) any_flag |= (P.rowflag[s] != 0);
  for (uint32_t idx = lane; idx < 16u * seq; idx += 32u) {
    const uint32_t r = idx & 15u, s = idx >> 4;
    const uint32_t o = rg * 16u + r;
    if (o >= out) continue;
    float y;
    if (PER_BLOCK) {
      const int *sr = s_acc[warp][r];
      float v = __int_as_float(sr[3 * s]) + __int_as_float(sr[3 * s + 1]) * 256.0f;
      v = v + __int_as_float(sr[3 * s + 2]) * 65536.0f;
      y = v * P.rowinv[s];
    } else {
      long long tot = (long long)s_acc[warp][r][3 * s] +
                      256ll * s_acc[warp][r][3 * s + 1] +
                      65536ll * s_acc[warp][r][3 * s + 2];
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

template <bool PB>
cudaError_t launch_mma(int NT, dim3 grid, cudaStream_t st, const float *X,
                       uint64_t xs, const uint32_t *WP, uint64_t ws_,
                       const float *S, uint64_t ss, const float *B, float *Y,
                       uint64_t ys, uint32_t seq, uint32_t out, uint32_t cols,
                       uint64_t limit, void *ws) {
  dim3 block(kWarps * 32);
#define NL_CASE(N)                                                          \
  case N:                                                                   \
    ternary_mma_kernel<N, PB><<<grid, block, 0, st>>>(                      \
        X, xs, WP, ws_, S, ss, B, Y, ys, seq, out, cols, limit, ws);        \
    break;
  switch (NT) {
    NL_CASE(1) NL_CASE(2) NL_CASE(3) NL_CASE(4) NL_CASE(5) NL_CASE(6)
    default: return cudaErrorInvalidValue;
  }
#undef NL_CASE
  return cudaPeekAtLastError();
}

}  // namespace

bool ternary_fast_shape(uint32_t cols, uint32_t nblk, uint32_t wng,
                        bool per_block) {
  if (cols == 0 || cols % 128u != 0) return false;
  if (wng != cols / 16u) return false;
  if (per_block && nblk != cols / 128u) return false;
  return true;
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
  // Sequences in chunks of 16 (one prep + one main launch per chunk); the
  // workspace is reused chunk to chunk, ordered by the stream.
  for (uint32_t s0 = 0; s0 < seq; s0 += kMaxFastSeq) {
    uint32_t ns = min((uint32_t)kMaxFastSeq, seq - s0);
    int NT = n_tiles((int)ns);
    dim3 pgrid((8 * NT + 2) / 3, count);
    ternary_prep_kernel<<<pgrid, 256, 0, stream>>>(X + (uint64_t)s0 * cols,
                                                    x_stride, ns, cols, ws);
    cudaError_t e = cudaPeekAtLastError();
    if (e != cudaSuccess) return e;
    dim3 grid(ceil_div(ceil_div((int)out, 16), kWarps), count);
    // The short-grid limit is an index into the whole Y; shift it per chunk.
    uint64_t base = (uint64_t)s0 * out;
    uint64_t lim = limit > base ? limit - base : 0;
    if (per_block)
      e = launch_mma<true>(NT, grid, stream, X + (uint64_t)s0 * cols, x_stride,
                           WP, w_stride, SCALE, s_stride, BIAS,
                           Y + (uint64_t)s0 * out, y_stride, ns, out, cols,
                           lim, ws);
    else
      e = launch_mma<false>(NT, grid, stream, X + (uint64_t)s0 * cols,
                            x_stride, WP, w_stride, SCALE, s_stride, BIAS,
                            Y + (uint64_t)s0 * out, y_stride, ns, out, cols,
                            lim, ws);
    count_launches(2);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
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

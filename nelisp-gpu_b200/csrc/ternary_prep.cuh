// ternary_prep.cuh -- activation prep of the tensor-core ternary GEMV:
// the fragment format and a CTA-level routine that converts one activation
// row into exact int8 limbs in mma B-fragment order.  Shared by the GEMV's
// own prep kernel and the decoder's fused normalisation epilogues.
//
// Each row s is scaled by a power of two 2^e_s that puts max|x| in
// [2^21, 2^22), rounded to an integer xq (the only inexact step: half a unit
// of 2^-22 of the row maximum) and split into three balanced int8 limbs,
// xq = l0 + 256 l1 + 65536 l2.  Rows holding a non-finite value, or whose
// maximum is so small that 2^e_s would leave the f32 normals, are flagged
// and computed on the CUDA cores instead.
#pragma once

#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

namespace nl {

constexpr int kMaxFastSeq = 16;  // 48 (s, limb) columns = 6 n-tiles of 8

// Fragment layout for one problem: uint2 frag[blk][nt][j][lane], where blk is
// the 128-column block, n-tile nt holds columns n = 8nt .. 8nt+7
// (n = 3s + limb), j the k32 step within the block and lane = 4*(n%8) + q.
// Lane q of MMA j in block blk covers word w = 2q + (j>>1) of the block and,
// within it, with k = 2*(j&1): codes {k, 4+k, 8+k, 12+k} (b0) and
// {k+1, 5+k, 9+k, 13+k} (b1) -- the order in which the weight operand
// registers carry them (k_ternary.cu, unpack_block).
// Blocks are outermost so that a run of blocks is one contiguous chunk the
// main kernel can stage into shared memory with a single bulk copy.
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

// CTA-level: convert row s (X_ROW, global or shared memory; NULL for the
// padding rows s >= seq of the last n-tile, which are written as zeros) into
// P's fragments, scale and flag.  RED is 34 floats of shared scratch.  Every
// thread of the CTA must call it; it synchronises the CTA.
__device__ __forceinline__ void prep_row(const float *x_row, uint32_t cols,
                                         uint32_t s, uint32_t seq, PrepOut P,
                                         float *red) {
  const int NT = n_tiles((int)seq);
  const float *xr = x_row;
  float &s_mul = red[32];
  int &s_ok = reinterpret_cast<int &>(red[33]);
  const bool live = s < seq && xr != nullptr;
  __syncthreads();
  if (live) {
    float m = 0.0f;
    int bad = 0;
    for (uint32_t i = threadIdx.x; i < cols; i += blockDim.x) {
      float v = xr[i];
      m = fmaxf(m, fabsf(v));
      bad |= !isfinite(v);          // NaN is dropped by fmaxf; catch it here
    }
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
  __syncthreads();
  // One thread per packed word (16 columns).
  const uint32_t nwords = cols / 16u;
  for (uint32_t W = threadIdx.x; W < nwords; W += blockDim.x) {
    int l[3][16];
    if (ok) {
      const float4 *src = reinterpret_cast<const float4 *>(xr + 16u * W);
#pragma unroll
      for (int v4 = 0; v4 < 4; v4++) {
        float4 f = src[v4];
        float v[4] = {f.x, f.y, f.z, f.w};
#pragma unroll
        for (int e = 0; e < 4; e++) {
          int qv = __float2int_rn(v[e] * mul);   // exact scaling, one rounding
          int l0 = (int)(int8_t)(qv & 0xff);
          int r = (qv - l0) >> 8;
          int l1 = (int)(int8_t)(r & 0xff);
          int l2 = (r - l1) >> 8;                // |qv| <= 2^22 -> |l2| <= 64
          l[0][4 * v4 + e] = l0; l[1][4 * v4 + e] = l1; l[2][4 * v4 + e] = l2;
        }
      }
    } else {
#pragma unroll
      for (int k = 0; k < 16; k++) l[0][k] = l[1][k] = l[2][k] = 0;
    }
    const uint32_t blk = W / 8u, wq = W % 8u;
    const uint32_t q = wq >> 1;
#pragma unroll
    for (int li = 0; li < 3; li++) {
      int n = 3 * (int)s + li;
      if (n >= 8 * NT) continue;
#pragma unroll
      for (int jlo = 0; jlo < 2; jlo++) {
        const int k = 2 * jlo;
        const uint32_t j = ((wq & 1u) << 1) | (uint32_t)jlo;
        uint2 fr;
        fr.x = pack4(l[li][k], l[li][4 + k], l[li][8 + k], l[li][12 + k]);
        fr.y = pack4(l[li][k + 1], l[li][5 + k], l[li][9 + k], l[li][13 + k]);
        size_t idx = (((size_t)blk * NT + (uint32_t)(n / 8)) * 4u + j) * 32u +
                     (uint32_t)(n % 8) * 4u + q;
        P.frag[idx] = fr;
      }
    }
  }
}

}  // namespace nl

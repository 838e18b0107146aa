// ternary_prep.cuh -- activation prep of the tensor-core ternary GEMV:
// the fragment format and the cluster-level routines that convert one
// activation row into exact int8 limbs in mma B-fragment order.  Shared by
// the GEMV's own prep kernel and the decoder's fused normalisation epilogues.
//
// Each row s is scaled by a power of two 2^e_s that puts max|x| in
// [2^(8L-3), 2^(8L-2)), rounded to an integer xq (the only inexact step: half
// a unit of 2^-(8L-2) of the row maximum) and split into L balanced int8
// limbs, xq = l0 + 256 l1 + 65536 l2 (+ 2^24 l3).  Problems of up to four
// sequence rows take L = 4 (xq to 30 bits): their limb columns fit the
// n-tiles that three limbs would take anyway, so the fourth costs no MMA.
// More rows take L = 3 (22 bits).  Rows holding a non-finite value, or whose
// maximum is so small that 2^e_s would leave the f32 normals, are flagged
// and computed on the CUDA cores instead.
#pragma once

#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

namespace nl {

constexpr int kMaxFastSeq = 16;  // 48 (s, limb) columns = 6 n-tiles of 8 (L = 3)

// Fragment layout for one problem: uint2 frag[blk][nt][h][lane][e], where
// blk is the 128-column block, n-tile nt holds columns n = 8nt .. 8nt+7
// (n = L s + limb), the k32 step within the block is j = 2h + e and
// lane = 4*(n%8) + q.  A lane's fragments for steps (0,1) and for (2,3) are
// each one 16-byte load, and the 32 lanes of a warp read 512 contiguous
// bytes.  Lane q of MMA j in block blk covers words 2q (b0) and 2q+1 (b1) of
// the block and, within each, codes {j, 4+j, 8+j, 12+j}: two-bit field j of
// every byte, the bits from which the weight operand registers of step j
// are made (k_ternary.cu, unpack_signed / unpack_offset).  Every step thus
// carries one field, so an accumulator per step holds one power-of-four
// scale.  Blocks are outermost so that a run of blocks is one contiguous
// chunk the main kernel can stage into shared memory with a single bulk copy.
//
// XSUM[s][r] is CTA r's share of sum xq_i over the values whose code sits in
// field 0, 1 or 2 of its byte (i % 4 != 3): the exact offset that the
// one-instruction weight operands 4^j (t + 2) of fields 0..2 add.
constexpr int kRowCluster = 8;     // CTAs that share one row in the prep
struct PrepOut {
  uint2 *frag;      // NT * cols * 8 bytes
  float *rowinv;    // [kMaxFastSeq] 2^-e_s
  int *rowflag;     // [kMaxFastSeq] 1: compute (., s) on the CUDA cores
  long long *xsum;  // [kMaxFastSeq][kRowCluster]
};

// Limbs per activation value for a problem of SEQ rows (see above).
__host__ __device__ inline int n_limbs(int seq) { return seq <= 4 ? 4 : 3; }
__host__ __device__ inline int n_tiles(int seq) { return (n_limbs(seq) * seq + 7) / 8; }
// Offset (in uint2) of the fragment pair (j = 2h, 2h+1) of LANE for n-tile T of
// block BLK.
__host__ __device__ inline size_t frag_pair(uint32_t blk, int NT, int t, int h, int lane) {
  return ((((size_t)blk * NT + t) * 2u + h) * 32u + lane) * 2u;
}
__host__ __device__ inline size_t frag_bytes(int seq, uint32_t cols) {
  return (size_t)n_tiles(seq) * cols * 8u;
}
__host__ __device__ inline size_t align256(size_t b) {
  return (b + 255u) & ~(size_t)255u;
}
constexpr size_t kPrepTail = 256u + (size_t)kMaxFastSeq * kRowCluster * 8u;
__host__ __device__ inline size_t prep_bytes(int seq, uint32_t cols) {
  return align256(frag_bytes(seq, cols)) + kPrepTail;
}
__device__ inline PrepOut prep_at(void *ws, int seq, uint32_t cols, uint32_t z) {
  char *base = (char *)ws + (size_t)z * prep_bytes(seq, cols);
  PrepOut p;
  p.frag = (uint2 *)base;
  p.rowinv = (float *)(base + align256(frag_bytes(seq, cols)));
  p.rowflag = (int *)(p.rowinv + kMaxFastSeq);
  p.xsum = (long long *)(base + align256(frag_bytes(seq, cols)) + 256u);
  return p;
}

// Exponent of a row of L-limb values: 2^e puts the row maximum MM in
// [2^(8L-3), 2^(8L-2)).  False when the row cannot be represented
// (non-finite, or 2^e / 2^-e outside the f32 normals); a zero row is
// representable with mul = inv = 0.
__device__ __forceinline__ bool row_scale(float mm, bool bad, float *mul, float *inv, int L) {
  *mul = 0.0f;
  *inv = 0.0f;
  if (bad) return false;
  if (!(mm > 0.0f)) return true;
  int E;
  frexpf(mm, &E);                      // mm in [2^(E-1), 2^E)
  const int e = 8 * L - 2 - E;
  if (e > 126 || e < -126) return false;
  *mul = ldexpf(1.0f, e);
  *inv = ldexpf(1.0f, -e);
  return true;
}

// Quantize the 16 values V of packed word W of sequence row S into the
// fragments of P (zeros when !OK): L balanced int8 limbs per value (MUL from
// row_scale with the same L), written in the column order of the weight
// operands (see the layout note).  Returns the word's share of XSUM: the sum
// of its xq over codes i % 4 != 3.
//
// The balanced base-256 digits d_l in [-128, 127] of xq are the bytes of
// xq + 128 (1 + 256 + ...) less 128: byte l of U = xq + 0x80808080 (L = 4;
// 0x00808080 for L = 3, whose top digit is at most 64 in magnitude) is
// d_l + 128, and d_l as an int8 bit pattern is that byte XOR 0x80.  A
// fragment word gathers digit l of four values with byte permutes.
__device__ __forceinline__ long long quantize_word(const float (&v)[16], float mul, bool ok,
                                                   uint32_t W, uint32_t s, int NT, int L,
                                                   PrepOut P) {
  const uint32_t bias = L == 4 ? 0x80808080u : 0x00808080u;
  uint32_t u[16];
  long long part = 0;
#pragma unroll
  for (int k = 0; k < 16; k++) {
    const int qv = ok ? __float2int_rn(v[k] * mul) : 0;   // exact scaling, one rounding
    if ((k & 3) != 3) part += qv;
    u[k] = (uint32_t)qv + bias;
  }
  const uint32_t blk = W / 8u, wq = W % 8u;
  const uint32_t q = wq >> 1, e = wq & 1u;   // word 2q is b0, word 2q+1 is b1
  uint32_t *fw = reinterpret_cast<uint32_t *>(P.frag);
#pragma unroll
  for (int li = 0; li < 4; li++) {
    if (li >= L) break;
    const int n = L * (int)s + li;
    if (n >= 8 * NT) continue;
    const uint32_t sel = (uint32_t)li | ((4u + (uint32_t)li) << 4);
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const uint32_t lo = __byte_perm(u[j], u[4 + j], sel);
      const uint32_t hi = __byte_perm(u[8 + j], u[12 + j], sel);
      const size_t idx = ((((size_t)blk * NT + (uint32_t)(n / 8)) * 2u + (uint32_t)(j >> 1)) * 32u +
                          (uint32_t)(n % 8) * 4u + q) * 2u + (uint32_t)(j & 1);
      fw[2 * idx + e] = __byte_perm(lo, hi, 0x5410) ^ 0x80808080u;
    }
  }
  return part;
}

// The value of sequence row S from the int32 sums ROW[n] of the limb columns
// n = L s + limb: exact in int64 (limb_total), or, for sums that per-block
// scales made floats (their bits in ROW), in f32 (limb_total_f; the /64 of
// the signed operands folded in).
__device__ __forceinline__ long long limb_total(const int *row, uint32_t s, int L) {
  const int *c = row + L * (int)s;
  long long t = (long long)c[0] + 256ll * c[1] + 65536ll * c[2];
  if (L == 4) t += 16777216ll * c[3];
  return t;
}
__device__ __forceinline__ float limb_total_f(const int *row, uint32_t s, int L) {
  const int *c = row + L * (int)s;
  float v = __int_as_float(c[0]) + __int_as_float(c[1]) * 256.0f;
  v = v + __int_as_float(c[2]) * 65536.0f;
  if (L == 4) v = v + __int_as_float(c[3]) * 16777216.0f;
  return v * 0.015625f;                        // / 64, exact
}

// ---- one row over a thread-block cluster ------------------------------------
// A row of a few thousand columns is too little work to keep a whole GPU busy
// and too much for one CTA to finish quickly, and the prep needs the row's
// maximum before any value can be quantized.  kRowCluster CTAs of a cluster
// share one row: each owns a run of columns starting on a packed-word
// boundary, the row statistics are combined through distributed shared
// memory, and each CTA quantizes its own words.

struct RowSlice {
  uint32_t c0, c1;   // columns [c0, c1) owned by this CTA; c0 % 16 == 0
};
__host__ __device__ inline uint32_t row_slice_cols(uint32_t cols) {
  const uint32_t per = (cols + kRowCluster - 1) / kRowCluster;
  return (per + 15u) & ~15u;
}
__device__ __forceinline__ RowSlice row_slice(uint32_t cols, uint32_t rank) {
  const uint32_t per = row_slice_cols(cols);
  RowSlice r;
  r.c0 = min(cols, rank * per);
  r.c1 = min(cols, r.c0 + per);
  return r;
}

// Quantize this CTA's slice XS (columns [c0, c1) of row s, staged in shared
// memory) into P once the row's maximum MM and non-finite flag BAD are known
// cluster-wide.  LIVE is false for the padding rows s >= seq of the last
// n-tile, whose fragments are written as zeros.  Rank 0 of the cluster
// stores the row's scale and flag; rank RANK stores its share of XSUM.
// Called by every thread of the CTA (it ends in a CTA-wide reduction).
// Needs cols % 16 == 0.
__device__ __forceinline__ void quantize_slice(const float *xs, RowSlice sl, float mm, bool bad,
                                               bool live, uint32_t rank, uint32_t s, uint32_t seq,
                                               PrepOut P) {
  __shared__ long long xred[32];
  const int NT = n_tiles((int)seq), L = n_limbs((int)seq);
  float mul = 0.0f, inv = 0.0f;
  const bool ok = live && row_scale(mm, bad, &mul, &inv, L);
  if (live && rank == 0 && threadIdx.x == 0) {
    P.rowinv[s] = inv;
    P.rowflag[s] = !ok;
  }
  long long part = 0;
  for (uint32_t W = sl.c0 / 16u + threadIdx.x; W < sl.c1 / 16u; W += blockDim.x) {
    float v[16];
    if (ok) {
      const float4 *src = reinterpret_cast<const float4 *>(xs + (16u * W - sl.c0));
#pragma unroll
      for (int v4 = 0; v4 < 4; v4++) {
        float4 f = src[v4];
        v[4 * v4] = f.x; v[4 * v4 + 1] = f.y; v[4 * v4 + 2] = f.z; v[4 * v4 + 3] = f.w;
      }
    }
    part += quantize_word(v, mul, ok, W, s, NT, L, P);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
  if ((threadIdx.x & 31) == 0) xred[threadIdx.x >> 5] = part;
  __syncthreads();
  if (threadIdx.x == 0 && live) {
    long long t = 0;
    for (int w = 0; w < (int)(blockDim.x >> 5); w++) t += xred[w];
    P.xsum[s * kRowCluster + rank] = t;
  }
}

// ---- one row in one CTA --------------------------------------------------------
// Row S of a problem (XR: cols floats, 16-byte aligned, cols % 16 == 0) by
// every thread of one CTA (blockDim.x a multiple of 32): pass 1 reads the row
// for its maximum and non-finite flag, pass 2 reads it again (L2) and
// quantizes one packed word per thread per step.  The CTA's XSUM goes to
// slot 0 of the row and the other slots are zeroed.  Loads bypass L1, so the
// row may have been written by other CTAs of the same kernel (made visible
// by a fence).  RED / XRED: shared scratch of 32 entries each.
__device__ __forceinline__ void prep_row_cta(const float *xr_f, uint32_t cols, uint32_t s,
                                             uint32_t seq, PrepOut P, float *red,
                                             long long *xred) {
  const int NT = n_tiles((int)seq), L = n_limbs((int)seq);
  const uint32_t wng = cols / 16u;
  const float4 *xr = reinterpret_cast<const float4 *>(xr_f);
  const int nwarp = (int)(blockDim.x >> 5);
  float m = 0.0f;
  int bad = 0;
  for (uint32_t W = threadIdx.x; W < wng; W += blockDim.x) {
#pragma unroll
    for (int k = 0; k < 4; k++) {
      const float4 f = __ldcg(xr + 4u * W + k);
      m = fmaxf(fmaxf(m, fabsf(f.x)), fmaxf(fabsf(f.y), fmaxf(fabsf(f.z), fabsf(f.w))));
      bad |= !isfinite(f.x) | !isfinite(f.y) | !isfinite(f.z) | !isfinite(f.w);
    }
  }
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  bad = __syncthreads_or(bad);    // also orders red[]
  float mm = 0.0f;
  for (int w = 0; w < nwarp; w++) mm = fmaxf(mm, red[w]);
  float mul = 0.0f, inv = 0.0f;
  const bool ok = row_scale(mm, bad != 0, &mul, &inv, L);
  if (threadIdx.x == 0) {
    P.rowinv[s] = inv;
    P.rowflag[s] = !ok;
  }
  long long part = 0;
  for (uint32_t W = threadIdx.x; W < wng; W += blockDim.x) {
    float v[16];
#pragma unroll
    for (int k = 0; k < 4; k++) {
      const float4 f = ok ? __ldcg(xr + 4u * W + k) : make_float4(0.f, 0.f, 0.f, 0.f);
      v[4 * k] = f.x; v[4 * k + 1] = f.y; v[4 * k + 2] = f.z; v[4 * k + 3] = f.w;
    }
    part += quantize_word(v, mul, ok, W, s, NT, L, P);
  }
  for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
  if ((threadIdx.x & 31) == 0) xred[threadIdx.x >> 5] = part;
  __syncthreads();
  if (threadIdx.x < (unsigned)kRowCluster) {
    long long t = 0;
    if (threadIdx.x == 0)
      for (int w = 0; w < nwarp; w++) t += xred[w];
    P.xsum[s * kRowCluster + threadIdx.x] = t;
  }
}

// ---- the generic CUDA-core row ------------------------------------------------
__device__ __forceinline__ float trit_of(uint32_t w, uint32_t f) {
  return (float)(((int32_t)(w << (30u - 2u * f))) >> 30);
}

// ---------------------------------------------------------------------------
// Generic CUDA-core path: any shape, the reference's semantics exactly
// (blocks b < nblk, words wi < min(wng, 8*nblk), fields i < cols).  One warp
// per output row; lanes take words, groups of eight lanes form a block.
// ---------------------------------------------------------------------------
template <int SB>
__device__ inline void ternary_row_generic(const float *__restrict__ X,
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

}  // namespace nl

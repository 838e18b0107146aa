// k_attn.cu -- rotary embedding, KV-cache append and single-query decode
// attention for sm_100a.
//
// Reference operators (lisp/nelisp-gpu-kernels.el):
//   rope-half      :857-882  half-split rotation, position = row index
//   decode-rope    :294-306  adjacent pairs, host cos/sin tables at POS[0]
//   decode-rope-b  :342-355  the same for B rows
//   cache-append   :308-315  CACHE[pos*kvdim + t] = SRC[t]
//   cache-append-b :358-365  CACHE[(b*maxseq + pos)*kvdim + t] = SRC[b, t]
//   decode-attn    :317-338  softmax(q.k_j / sqrt(hd)) . V over j <= POS[0]
//   decode-attn-b  :368-390  the same per sequence b of B
//
// The reference's attention runs one invocation per OUTPUT LANE and makes
// two passes over the keys, so every q.k dot product of a head is computed
// 2*hd times.  Here it is split-K flash decoding: CTAs own a (sequence, kv
// head, key range), stream the K and V rows of the range once with 128-bit
// loads (four key rows in flight per warp), compute each dot product once
// per query head of the GQA group with a warp reduction, and keep an online
// softmax (running max, running sum, rescaled context).  A second kernel
// merges the ranges.  The partials live in scratch memory.
//
// POS is device data in the reference's interface, so the key count is read
// on the device; splits past it write empty partials.  Reads past the end of
// a cache buffer return zero (Vulkan's robust buffer access) instead of
// faulting, and positions past the buffer's last row are not attended.

#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>
#include <string.h>

#include "nl_internal.h"

namespace nl {
namespace {

__device__ __forceinline__ float ld_or0(const float *p, uint64_t i, uint64_t n) {
  return i < n ? __ldg(p + i) : 0.0f;
}

// ---- rope ---------------------------------------------------------------------
__global__ void rope_half_kernel(const float *__restrict__ X, float *__restrict__ Y,
                                 uint32_t seq, uint32_t nheads, uint32_t hd,
                                 float rbase, float sgn, uint64_t n) {
  const uint32_t half = hd / 2;
  for (uint64_t idx = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < n;
       idx += (uint64_t)gridDim.x * blockDim.x) {
    uint32_t m = (uint32_t)(idx % half), tmp = (uint32_t)(idx / half);
    uint32_t h = tmp % nheads, p = tmp / nheads;
    uint64_t b0 = (uint64_t)p * nheads * hd + (uint64_t)h * hd;
    float ex = __fdiv_rn(2.0f * (float)m, (float)hd);
    float theta = __fdiv_rn((float)p, powf(rbase, ex));
    float c = cosf(theta), s = __fmul_rn(sgn, sinf(theta));
    float a0 = __ldg(X + b0 + m), a1 = __ldg(X + b0 + m + half);
    Y[b0 + m] = __fsub_rn(__fmul_rn(a0, c), __fmul_rn(a1, s));
    Y[b0 + m + half] = __fadd_rn(__fmul_rn(a1, c), __fmul_rn(a0, s));
  }
}

__global__ void decode_rope_b_kernel(const float *__restrict__ X,
                                     const float *__restrict__ CO,
                                     const float *__restrict__ SI,
                                     const float *__restrict__ SG,
                                     const float *__restrict__ POS,
                                     float *__restrict__ C, uint32_t B,
                                     uint32_t cols, uint32_t heads, uint64_t n,
                                     uint64_t n_co, uint64_t n_si) {
  const uint32_t hd = cols / heads, half = hd / 2, rh = heads * half;
  const uint32_t pos = __float2uint_rz(__ldg(POS));
  const float sg = __ldg(SG);
  for (uint64_t idx = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < n;
       idx += (uint64_t)gridDim.x * blockDim.x) {
    uint32_t bb = (uint32_t)(idx / rh), rem = (uint32_t)(idx % rh);
    uint32_t m = rem % half, h = rem / half;
    uint32_t ci = pos * half + m;
    float cc = ld_or0(CO, ci, n_co), ss = __fmul_rn(ld_or0(SI, ci, n_si), sg);
    uint64_t b0 = (uint64_t)bb * cols + (uint64_t)h * hd;
    uint64_t i0 = b0 + 2 * m, i1 = i0 + 1;
    float a0 = __ldg(X + i0), a1 = __ldg(X + i1);
    C[i0] = __fsub_rn(__fmul_rn(a0, cc), __fmul_rn(a1, ss));
    C[i1] = __fadd_rn(__fmul_rn(a0, ss), __fmul_rn(a1, cc));
  }
}

__global__ void cache_append_b_kernel(const float *__restrict__ SRC,
                                      const float *__restrict__ POS,
                                      float *__restrict__ CACHE, uint32_t kvdim,
                                      uint32_t maxseq, uint64_t n,
                                      uint64_t n_cache) {
  const uint32_t pos = __float2uint_rz(__ldg(POS));
  for (uint64_t idx = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < n;
       idx += (uint64_t)gridDim.x * blockDim.x) {
    uint32_t bb = (uint32_t)(idx / kvdim), t = (uint32_t)(idx % kvdim);
    uint32_t dst = (bb * maxseq + pos) * kvdim + t;   // uint32, as the reference
    if (dst < n_cache) CACHE[dst] = __ldg(SRC + idx);
  }
}

// ---- split-K decode attention -------------------------------------------------
// Partials per (b, query head h, split): m (running max of the scaled
// scores), l (sum of exp(score - m)) and o[hd] (sum of exp(score - m) v).
// The geometry (AttnGeom) is declared in nl_internal.h.

constexpr int kAttnWarps = 4;
constexpr int kMaxGrp = 8;

// One CTA per (split, b*kvheads + kvh).  HD = head dim (multiple of 32*4);
// each lane owns HD/32 consecutive dims (float4 loads when HD = 128).
template <int HD, int GRP>
__global__ void __launch_bounds__(kAttnWarps * 32)
attn_partial_kernel(const float *__restrict__ Q, const float *__restrict__ CK,
                    const float *__restrict__ CV, const float *__restrict__ POS,
                    AttnGeom g, float *__restrict__ part) {
  pdl_trigger();
  pdl_wait();
  constexpr int DPL = HD / 32;  // dims per lane
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint32_t split = blockIdx.x;
  const uint32_t bkv = blockIdx.y, bb = bkv / g.kvheads, kvh = bkv % g.kvheads;
  constexpr uint32_t grp = GRP;
  __shared__ float s_m[kAttnWarps][GRP], s_l[kAttnWarps][GRP];
  __shared__ float s_o[kAttnWarps][GRP][HD];

  uint32_t len = __float2uint_rz(__ldg(POS)) + 1u;
  if (len > g.maxseq) len = g.maxseq;
  const uint32_t p0 = split * g.chunk;
  const uint32_t p1 = min(p0 + g.chunk, len);

  // Query heads of this kv head, this lane's dims.
  float q[GRP][DPL];
#pragma unroll
  for (uint32_t hh = 0; hh < grp; hh++) {
    const float *qh = Q + (uint64_t)bb * g.heads * HD + (uint64_t)(kvh * grp + hh) * HD + lane * DPL;
#pragma unroll
    for (int d = 0; d < DPL; d++) q[hh][d] = __ldg(qh + d);
  }
  float m[GRP], l[GRP], o[GRP][DPL];
#pragma unroll
  for (int hh = 0; hh < GRP; hh++) {
    m[hh] = -INFINITY; l[hh] = 0.0f;
#pragma unroll
    for (int d = 0; d < DPL; d++) o[hh][d] = 0.0f;
  }
  const uint64_t cbase = (uint64_t)bb * g.maxseq * g.kvdim + (uint64_t)kvh * HD + lane * DPL;
  constexpr int U = 4;  // key rows in flight per warp
  for (uint32_t j0 = p0 + warp * U; j0 < p1; j0 += kAttnWarps * U) {
    float kr[U][DPL], vr[U][DPL];
#pragma unroll
    for (int u = 0; u < U; u++) {
      uint32_t j = j0 + u;
      uint64_t off = cbase + (uint64_t)j * g.kvdim;
      bool ok = j < p1 && off + DPL <= g.cache_words;
      if (DPL == 4) {
        float4 k4 = ok ? __ldcs(reinterpret_cast<const float4 *>(CK + off)) : make_float4(0, 0, 0, 0);
        float4 v4 = ok ? __ldcs(reinterpret_cast<const float4 *>(CV + off)) : make_float4(0, 0, 0, 0);
        kr[u][0] = k4.x; kr[u][1] = k4.y; kr[u][2] = k4.z; kr[u][3] = k4.w;
        vr[u][0] = v4.x; vr[u][1] = v4.y; vr[u][2] = v4.z; vr[u][3] = v4.w;
      } else {
#pragma unroll
        for (int d = 0; d < DPL; d++) {
          kr[u][d] = ok ? __ldcs(CK + off + d) : 0.0f;
          vr[u][d] = ok ? __ldcs(CV + off + d) : 0.0f;
        }
      }
    }
#pragma unroll
    for (int u = 0; u < U; u++) {
      if (j0 + u >= p1) break;
#pragma unroll
      for (uint32_t hh = 0; hh < grp; hh++) {
        float dot = 0.0f;
#pragma unroll
        for (int d = 0; d < DPL; d++) dot = fmaf(q[hh][d], kr[u][d], dot);
        for (int off = 16; off > 0; off >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, off);
        const float s = dot * g.coef;
        const float mn = fmaxf(m[hh], s);
        const float corr = expf(m[hh] - mn);   // exp(-inf) = 0 on the first key
        const float p = expf(s - mn);
        l[hh] = l[hh] * corr + p;
#pragma unroll
        for (int d = 0; d < DPL; d++) o[hh][d] = fmaf(p, vr[u][d], o[hh][d] * corr);
        m[hh] = mn;
      }
    }
  }
  // Merge the four warps of the CTA.
#pragma unroll
  for (uint32_t hh = 0; hh < grp; hh++) {
    if (lane == 0) { s_m[warp][hh] = m[hh]; s_l[warp][hh] = l[hh]; }
#pragma unroll
    for (int d = 0; d < DPL; d++) s_o[warp][hh][lane * DPL + d] = o[hh][d];
  }
  __syncthreads();
  const uint32_t nsplit = g.nsplit;
  for (uint32_t e = threadIdx.x; e < grp * HD; e += blockDim.x) {
    uint32_t hh = e / HD, d = e % HD;
    float mm = -INFINITY;
    for (int w = 0; w < kAttnWarps; w++) mm = fmaxf(mm, s_m[w][hh]);
    float ll = 0.0f, oo = 0.0f;
    if (mm > -INFINITY) {
      for (int w = 0; w < kAttnWarps; w++) {
        float c = expf(s_m[w][hh] - mm);
        ll += s_l[w][hh] * c;
        oo += s_o[w][hh][d] * c;
      }
    }
    const uint32_t h = kvh * grp + hh;
    float *pp = part + (((uint64_t)bb * g.heads + h) * nsplit + split) * (HD + 2);
    pp[2 + d] = oo;
    if (d == 0) { pp[0] = mm; pp[1] = ll; }
  }
}

// The decoder's attention step with the RoPE and the cache append fused in
// (the decoder's own composition; the registry ops above keep the reference's
// separate decode-rope / cache-append / decode-attn).  QKV holds, per
// sequence row, the query heads, then the key heads, then the value heads of
// the current position p = POS[0], unrotated.  Each CTA rotates its query
// heads in registers -- the same operation order as a separate half-split
// RoPE pass, hence the same bits -- and the CTA whose split holds p rotates
// the new key, writes key and value to the cache row p and folds them in from
// registers (the cache loop stops before p).
template <int HD, int GRP>
__global__ void __launch_bounds__(kAttnWarps * 32)
attn_rope_partial_kernel(const float *__restrict__ QKV, float *__restrict__ CK,
                         float *__restrict__ CV, const int *__restrict__ POS, AttnGeom g,
                         const float2 *__restrict__ rope, float *__restrict__ part) {
  pdl_wait();
  constexpr int DPL = HD / 32;   // dims per lane; lanes 0-15 hold the first half
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint32_t split = blockIdx.x;
  const uint32_t bkv = blockIdx.y, bb = bkv / g.kvheads, kvh = bkv % g.kvheads;
  __shared__ float s_m[kAttnWarps][GRP], s_l[kAttnWarps][GRP];
  __shared__ float s_o[kAttnWarps][GRP][HD];

  const uint32_t p = (uint32_t)__ldg(POS);
  const uint32_t len = min(p + 1u, g.maxseq);
  const uint32_t p0 = split * g.chunk;
  const uint32_t p1 = min(p0 + g.chunk, len);
  const bool has_p = p < g.maxseq && p >= p0 && p < p1;
  const float *row = QKV + (uint64_t)bb * (g.heads + 2u * g.kvheads) * HD;

  // Rotation of this lane's dims at position p: dim m and m + HD/2 pair up;
  // ROPE[p][m] = (cos, sin) of the angle (rope_table_launch).
  float cs[DPL], sn[DPL];
#pragma unroll
  for (int d = 0; d < DPL; d++) {
    const uint32_t m = (uint32_t)(lane * DPL + d) % (HD / 2);
    const float2 r = __ldg(rope + (uint64_t)min(p, g.maxseq - 1u) * (HD / 2) + m);
    cs[d] = r.x;
    sn[d] = r.y;
  }
  const bool first_half = lane < 16;
  auto rotate = [&](const float *src, float (&out)[DPL]) {
#pragma unroll
    for (int d = 0; d < DPL; d++) {
      const float own = __ldg(src + lane * DPL + d);
      const float other = __shfl_xor_sync(0xffffffffu, own, 16);
      const float a0 = first_half ? own : other, a1 = first_half ? other : own;
      out[d] = first_half ? __fsub_rn(__fmul_rn(a0, cs[d]), __fmul_rn(a1, sn[d]))
                          : __fadd_rn(__fmul_rn(a1, cs[d]), __fmul_rn(a0, sn[d]));
    }
  };
  float q[GRP][DPL];
#pragma unroll
  for (int hh = 0; hh < GRP; hh++) rotate(row + (uint64_t)(kvh * GRP + hh) * HD, q[hh]);
  // The new key (rotated) and value of this kv head, cached by the split holding p.
  float kn[DPL], vn[DPL];
  const uint64_t cbase = (uint64_t)bb * g.maxseq * g.kvdim + (uint64_t)kvh * HD + lane * DPL;
  if (has_p) {
    rotate(row + (uint64_t)(g.heads + kvh) * HD, kn);
    const float *vs = row + (uint64_t)(g.heads + g.kvheads + kvh) * HD + lane * DPL;
#pragma unroll
    for (int d = 0; d < DPL; d++) vn[d] = __ldg(vs + d);
    const uint64_t off = cbase + (uint64_t)p * g.kvdim;
    if (warp == 0 && off + DPL <= g.cache_words) {
#pragma unroll
      for (int d = 0; d < DPL; d++) {
        CK[off + d] = kn[d];
        CV[off + d] = vn[d];
      }
    }
  }

  float m[GRP], l[GRP], o[GRP][DPL];
#pragma unroll
  for (int hh = 0; hh < GRP; hh++) {
    m[hh] = -INFINITY; l[hh] = 0.0f;
#pragma unroll
    for (int d = 0; d < DPL; d++) o[hh][d] = 0.0f;
  }
  auto fold = [&](const float (&kr)[DPL], const float (&vr)[DPL]) {
#pragma unroll
    for (int hh = 0; hh < GRP; hh++) {
      float dot = 0.0f;
#pragma unroll
      for (int d = 0; d < DPL; d++) dot = fmaf(q[hh][d], kr[d], dot);
      for (int off = 16; off > 0; off >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, off);
      const float sc = dot * g.coef;
      const float mn = fmaxf(m[hh], sc);
      const float corr = expf(m[hh] - mn);   // exp(-inf) = 0 on the first key
      const float pr = expf(sc - mn);
      l[hh] = l[hh] * corr + pr;
#pragma unroll
      for (int d = 0; d < DPL; d++) o[hh][d] = fmaf(pr, vr[d], o[hh][d] * corr);
      m[hh] = mn;
    }
  };
  const uint32_t pc = has_p ? p : p1;             // cached keys: [p0, pc)
  constexpr int U = 4;                            // key rows in flight per warp
  for (uint32_t j0 = p0 + warp * U; j0 < pc; j0 += kAttnWarps * U) {
    float kr[U][DPL], vr[U][DPL];
#pragma unroll
    for (int u = 0; u < U; u++) {
      const uint32_t j = j0 + u;
      const uint64_t off = cbase + (uint64_t)j * g.kvdim;
      const bool ok = j < pc && off + DPL <= g.cache_words;
      if (DPL == 4) {
        float4 k4 = ok ? __ldcs(reinterpret_cast<const float4 *>(CK + off)) : make_float4(0, 0, 0, 0);
        float4 v4 = ok ? __ldcs(reinterpret_cast<const float4 *>(CV + off)) : make_float4(0, 0, 0, 0);
        kr[u][0] = k4.x; kr[u][1] = k4.y; kr[u][2] = k4.z; kr[u][3] = k4.w;
        vr[u][0] = v4.x; vr[u][1] = v4.y; vr[u][2] = v4.z; vr[u][3] = v4.w;
      } else {
#pragma unroll
        for (int d = 0; d < DPL; d++) {
          kr[u][d] = ok ? __ldcs(CK + off + d) : 0.0f;
          vr[u][d] = ok ? __ldcs(CV + off + d) : 0.0f;
        }
      }
    }
#pragma unroll
    for (int u = 0; u < U; u++) {
      if (j0 + u >= pc) break;
      fold(kr[u], vr[u]);
    }
  }
  if (has_p && warp == (int)(((pc - p0) / U) % kAttnWarps)) fold(kn, vn);
  // Merge the four warps of the CTA.
#pragma unroll
  for (int hh = 0; hh < GRP; hh++) {
    if (lane == 0) { s_m[warp][hh] = m[hh]; s_l[warp][hh] = l[hh]; }
#pragma unroll
    for (int d = 0; d < DPL; d++) s_o[warp][hh][lane * DPL + d] = o[hh][d];
  }
  __syncthreads();
  for (uint32_t e = threadIdx.x; e < (uint32_t)GRP * HD; e += blockDim.x) {
    const uint32_t hh = e / HD, d = e % HD;
    float mm = -INFINITY;
    for (int w = 0; w < kAttnWarps; w++) mm = fmaxf(mm, s_m[w][hh]);
    float ll = 0.0f, oo = 0.0f;
    if (mm > -INFINITY) {
      for (int w = 0; w < kAttnWarps; w++) {
        const float c = expf(s_m[w][hh] - mm);
        ll += s_l[w][hh] * c;
        oo += s_o[w][hh][d] * c;
      }
    }
    const uint32_t h = kvh * GRP + hh;
    float *pp = part + (((uint64_t)bb * g.heads + h) * g.nsplit + split) * (HD + 2);
    pp[2 + d] = oo;
    if (d == 0) { pp[0] = mm; pp[1] = ll; }
  }
}

// One CTA per (b, h): merge the splits and write C.
template <int HD>
__global__ void attn_combine_kernel(const float *__restrict__ part, AttnGeom g,
                                    float *__restrict__ C, uint64_t limit) {
  pdl_wait();
  const uint32_t bh = blockIdx.x;
  const uint32_t bb = bh / g.heads, h = bh % g.heads;
  const float *pp = part + (uint64_t)bh * g.nsplit * (HD + 2);
  float mm = -INFINITY;
  for (uint32_t s = 0; s < g.nsplit; s++) mm = fmaxf(mm, pp[(uint64_t)s * (HD + 2)]);
  for (uint32_t d = threadIdx.x; d < HD; d += blockDim.x) {
    float ll = 0.0f, oo = 0.0f;
    for (uint32_t s = 0; s < g.nsplit; s++) {
      const float *ps = pp + (uint64_t)s * (HD + 2);
      if (ps[0] > -INFINITY) {
        float c = expf(ps[0] - mm);
        ll += ps[1] * c;
        oo += ps[2 + d] * c;
      }
    }
    uint64_t idx = (uint64_t)bb * g.heads * HD + (uint64_t)h * HD + d;
    if (idx < limit) C[idx] = oo / ll;
  }
}

// Reference arithmetic for head sizes the split kernel does not cover: one
// thread per output lane, two passes, as kernels.el:368-390.
__global__ void attn_simple_kernel(const float *__restrict__ Q,
                                   const float *__restrict__ CK,
                                   const float *__restrict__ CV,
                                   const float *__restrict__ POS, AttnGeom g,
                                   float *__restrict__ C, uint64_t limit) {
  const uint32_t dim = g.heads * g.hd;
  uint64_t idx = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (uint64_t)g.B * dim || idx >= limit) return;
  uint32_t bb = (uint32_t)(idx / dim), c = (uint32_t)(idx % dim);
  uint32_t h = c / g.hd, t = c % g.hd, kvh = h / g.grp;
  uint32_t len = __float2uint_rz(__ldg(POS)) + 1u;
  if (len > g.maxseq) len = g.maxseq;
  uint64_t cbase = (uint64_t)bb * g.maxseq * g.kvdim, c0q = (uint64_t)bb * dim + (uint64_t)h * g.hd;
  float mx = -1.0e30f;
  for (uint32_t j = 0; j < len; j++) {
    uint64_t kb = cbase + (uint64_t)j * g.kvdim + (uint64_t)kvh * g.hd;
    float acc = 0.0f;
    for (uint32_t tt = 0; tt < g.hd; tt++) acc = fmaf(__ldg(Q + c0q + tt), ld_or0(CK, kb + tt, g.cache_words), acc);
    mx = fmaxf(mx, acc * g.coef);
  }
  float z = 0.0f, ctx = 0.0f;
  for (uint32_t j = 0; j < len; j++) {
    uint64_t kb = cbase + (uint64_t)j * g.kvdim + (uint64_t)kvh * g.hd;
    float acc = 0.0f;
    for (uint32_t tt = 0; tt < g.hd; tt++) acc = fmaf(__ldg(Q + c0q + tt), ld_or0(CK, kb + tt, g.cache_words), acc);
    float e = expf(acc * g.coef - mx);
    z += e;
    ctx = fmaf(e, ld_or0(CV, kb + t, g.cache_words), ctx);
  }
  C[idx] = ctx / z;
}

AttnGeom make_geom(uint32_t B, uint32_t dim, uint32_t heads, uint32_t kvheads,
                   uint32_t maxseq, uint64_t cache_words) {
  AttnGeom g;
  g.B = B; g.heads = heads; g.kvheads = kvheads;
  g.hd = heads ? dim / heads : 0;
  g.grp = kvheads ? heads / kvheads : 0;
  g.kvdim = kvheads * g.hd;
  g.maxseq = maxseq;
  g.cache_words = cache_words;
  g.coef = 1.0f / sqrtf((float)g.hd);
  // Enough CTAs for ~4 per SM, at least 32 keys each.
  uint32_t units = B * kvheads;
  uint32_t want = units ? (uint32_t)ceil_div(4 * 148, (int)units) : 1;
  if (want < 1) want = 1;
  uint32_t chunk = maxseq ? (maxseq + want - 1) / want : 1;
  if (chunk < 32) chunk = 32;
  g.chunk = chunk;
  g.nsplit = maxseq ? (maxseq + chunk - 1) / chunk : 1;
  if (g.nsplit == 0) g.nsplit = 1;
  return g;
}

bool split_ok(const AttnGeom &g) {
  return (g.hd == 128 || g.hd == 64) && g.grp >= 1 && g.grp <= (uint32_t)kMaxGrp &&
         g.heads == g.kvheads * g.grp;
}

size_t attn_scratch(const AttnGeom &g) {
  if (!split_ok(g)) return 0;
  return (size_t)g.B * g.heads * g.nsplit * (g.hd + 2) * sizeof(float);
}

cudaError_t attn_launch(const float *Q, const float *CK, const float *CV,
                        const float *POS, float *C, const AttnGeom &g,
                        uint64_t limit, void *scratch, cudaStream_t st, bool pdl = false) {
  if (g.B == 0 || g.heads == 0) return cudaSuccess;
  if (!split_ok(g) || scratch == nullptr || !aligned16(CK) || !aligned16(CV)) {
    uint64_t n = (uint64_t)g.B * g.heads * g.hd;
    attn_simple_kernel<<<(unsigned)ceil_div64(n, 128), 128, 0, st>>>(Q, CK, CV, POS, g, C, limit);
    count_launches(1);
    return cudaPeekAtLastError();
  }
  dim3 grid(g.nsplit, g.B * g.kvheads);
  float *part = (float *)scratch;
  cudaError_t e = cudaSuccess;
#define NL_ATTN(HD, G)                                                       \
  case G:                                                                    \
    e = launch_k(attn_partial_kernel<HD, G>, grid, dim3(kAttnWarps * 32), 0, st, pdl, \
                 Q, CK, CV, POS, g, part);                                       \
    break;
  if (g.hd == 128) {
    switch (g.grp) {
      NL_ATTN(128, 1) NL_ATTN(128, 2) NL_ATTN(128, 3) NL_ATTN(128, 4)
      NL_ATTN(128, 5) NL_ATTN(128, 6) NL_ATTN(128, 7) NL_ATTN(128, 8)
      default: return cudaErrorInvalidValue;
    }
    if (e == cudaSuccess)
      e = launch_k(attn_combine_kernel<128>, dim3(g.B * g.heads), dim3(128), 0, st, pdl, part, g,
                   C, limit);
  } else {
    switch (g.grp) {
      NL_ATTN(64, 1) NL_ATTN(64, 2) NL_ATTN(64, 3) NL_ATTN(64, 4)
      NL_ATTN(64, 5) NL_ATTN(64, 6) NL_ATTN(64, 7) NL_ATTN(64, 8)
      default: return cudaErrorInvalidValue;
    }
    if (e == cudaSuccess)
      e = launch_k(attn_combine_kernel<64>, dim3(g.B * g.heads), dim3(64), 0, st, pdl, part, g, C,
                   limit);
  }
#undef NL_ATTN
  count_launches(2);
  return e != cudaSuccess ? e : cudaPeekAtLastError();
}

// ---- registry glue -------------------------------------------------------------
size_t no_scratch(const OpArgs &) { return 0; }

const char *chk_rope_half(const OpArgs &a) {
  uint64_t n = (uint64_t)a.push[0] * a.push[1] * a.push[2];
  if (a.push[2] % 2) return fmt_msg("rope-half: hd (%u) must be even", a.push[2]);
  const char *m;
  if ((m = need_words(a, 0, n, "X"))) return m;
  return need_words(a, 1, n, "Y");
}
cudaError_t run_rope_half(const OpArgs &a) {
  uint32_t half = a.push[2] / 2;
  uint64_t n = (uint64_t)a.push[0] * a.push[1] * half;
  uint64_t lim = invocations(a.groups, 64);
  if (lim < n) n = lim;
  if (n == 0) return cudaSuccess;
  float rbase, sgn;
  memcpy(&rbase, &a.push[3], 4);
  memcpy(&sgn, &a.push[4], 4);
  rope_half_kernel<<<grid_for(n, 256), 256, 0, a.stream>>>(
      (const float *)a.buf[0], (float *)a.buf[1], a.push[0], a.push[1], a.push[2],
      rbase, sgn, n);
  count_launches(1);
  return cudaPeekAtLastError();
}

// decode-rope(-b): (X CO SI SG POS C) push (B cols heads) / (cols heads)
template <bool BATCHED>
const char *chk_decode_rope(const OpArgs &a) {
  uint64_t B = BATCHED ? a.push[0] : 1, cols = a.push[BATCHED ? 1 : 0], heads = a.push[BATCHED ? 2 : 1];
  if (heads == 0 || cols % heads || (cols / heads) % 2)
    return fmt_msg("decode-rope: cols (%llu) must split into heads (%llu) of even size",
                   (unsigned long long)cols, (unsigned long long)heads);
  const char *m;
  if ((m = need_words(a, 0, B * cols, "X"))) return m;
  if ((m = need_words(a, 3, (B * cols) != 0 ? 1 : 0, "SG"))) return m;
  if ((m = need_words(a, 4, (B * cols) != 0 ? 1 : 0, "POS"))) return m;
  return need_words(a, 5, B * cols, "C");
}
template <bool BATCHED>
cudaError_t run_decode_rope(const OpArgs &a) {
  uint32_t B = BATCHED ? a.push[0] : 1, cols = a.push[BATCHED ? 1 : 0], heads = a.push[BATCHED ? 2 : 1];
  uint64_t n = (uint64_t)B * heads * ((cols / heads) / 2);
  uint64_t lim = invocations(a.groups, 64);
  if (lim < n) n = lim;
  if (n == 0) return cudaSuccess;
  decode_rope_b_kernel<<<grid_for(n, 256), 256, 0, a.stream>>>(
      (const float *)a.buf[0], (const float *)a.buf[1], (const float *)a.buf[2],
      (const float *)a.buf[3], (const float *)a.buf[4], (float *)a.buf[5], B, cols,
      heads, n, a.words[1], a.words[2]);
  count_launches(1);
  return cudaPeekAtLastError();
}

// cache-append(-b): (SRC POS CACHE) push (B kvdim maxseq) / (kvdim)
template <bool BATCHED>
const char *chk_cache_append(const OpArgs &a) {
  uint64_t n = BATCHED ? (uint64_t)a.push[0] * a.push[1] : a.push[0];
  const char *m;
  if ((m = need_words(a, 0, n, "SRC"))) return m;
  return need_words(a, 1, n ? 1 : 0, "POS");
}
template <bool BATCHED>
cudaError_t run_cache_append(const OpArgs &a) {
  uint32_t kvdim = BATCHED ? a.push[1] : a.push[0];
  uint32_t maxseq = BATCHED ? a.push[2] : 0;
  uint64_t n = BATCHED ? (uint64_t)a.push[0] * a.push[1] : a.push[0];
  uint64_t lim = invocations(a.groups, 64);
  if (lim < n) n = lim;
  if (n == 0) return cudaSuccess;
  cache_append_b_kernel<<<grid_for(n, 256), 256, 0, a.stream>>>(
      (const float *)a.buf[0], (const float *)a.buf[1], (float *)a.buf[2], kvdim,
      maxseq, n, a.words[2]);
  count_launches(1);
  return cudaPeekAtLastError();
}

// decode-attn(-b): (Q CK CV POS C) push (B dim heads kvheads maxseq) /
// (dim heads kvheads); for B = 1 the cache holds as many rows as CK has.
template <bool BATCHED>
AttnGeom geom_of(const OpArgs &a) {
  uint32_t B = BATCHED ? a.push[0] : 1;
  uint32_t dim = a.push[BATCHED ? 1 : 0], heads = a.push[BATCHED ? 2 : 1], kvheads = a.push[BATCHED ? 3 : 2];
  uint32_t hd = heads ? dim / heads : 0, kvdim = kvheads * hd;
  uint64_t cw = a.words[1] < a.words[2] ? a.words[1] : a.words[2];
  uint32_t maxseq = BATCHED ? a.push[4] : (kvdim ? (uint32_t)(cw / kvdim) : 0);
  return make_geom(B, dim, heads, kvheads, maxseq, cw);
}
template <bool BATCHED>
const char *chk_attn(const OpArgs &a) {
  uint32_t B = BATCHED ? a.push[0] : 1;
  uint32_t dim = a.push[BATCHED ? 1 : 0], heads = a.push[BATCHED ? 2 : 1], kvheads = a.push[BATCHED ? 3 : 2];
  if (heads == 0 || kvheads == 0 || dim % heads || heads % kvheads)
    return fmt_msg("decode-attn: dim %u, heads %u, kvheads %u do not divide", dim, heads, kvheads);
  const char *m;
  if ((m = need_words(a, 0, (uint64_t)B * dim, "Q"))) return m;
  if ((m = need_words(a, 3, B ? 1 : 0, "POS"))) return m;
  return need_words(a, 4, (uint64_t)B * dim, "C");
}
template <bool BATCHED>
size_t scr_attn(const OpArgs &a) {
  return attn_scratch(geom_of<BATCHED>(a));
}
template <bool BATCHED>
cudaError_t run_attn(const OpArgs &a) {
  AttnGeom g = geom_of<BATCHED>(a);
  return attn_launch((const float *)a.buf[0], (const float *)a.buf[1],
                     (const float *)a.buf[2], (const float *)a.buf[3],
                     (float *)a.buf[4], g, invocations(a.groups, 64), a.scratch,
                     a.stream);
}

}  // namespace

AttnGeom attn_geom(uint32_t B, uint32_t dim, uint32_t heads, uint32_t kvheads,
                   uint32_t maxseq, uint64_t cache_words) {
  return make_geom(B, dim, heads, kvheads, maxseq, cache_words);
}
size_t attn_scratch_bytes(const AttnGeom &g) { return attn_scratch(g); }
cudaError_t attn_decode_launch(const float *Q, const float *CK, const float *CV,
                               const float *POS, float *C, const AttnGeom &g, void *scratch,
                               cudaStream_t st, bool pdl) {
  return attn_launch(Q, CK, CV, POS, C, g, UINT64_MAX, scratch, st, pdl);
}

bool rope_split_ok(const AttnGeom &g) {
  return (g.hd == 32 || g.hd == 64 || g.hd == 128 || g.hd == 256) && g.grp >= 1 &&
         g.grp <= (uint32_t)kMaxGrp && g.heads == g.kvheads * g.grp;
}

// ROPE[p][m] = (cos theta, sin theta), theta = p / base^(2m/hd), for
// p < maxseq and m < hd/2: the half-split rotation's operand order.
__global__ void rope_table_kernel(float2 *rope, uint32_t maxseq, uint32_t hd, float base) {
  const uint32_t half = hd / 2;
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < (uint64_t)maxseq * half;
       i += (uint64_t)gridDim.x * blockDim.x) {
    const uint32_t p = (uint32_t)(i / half), m = (uint32_t)(i % half);
    const float ex = __fdiv_rn(2.0f * (float)m, (float)hd);
    const float theta = __fdiv_rn((float)p, powf(base, ex));
    rope[i] = make_float2(cosf(theta), sinf(theta));
  }
}

cudaError_t rope_table_launch(float2 *rope, uint32_t maxseq, uint32_t hd, float base,
                              cudaStream_t st) {
  rope_table_kernel<<<grid_for((uint64_t)maxseq * (hd / 2), 256), 256, 0, st>>>(rope, maxseq, hd,
                                                                                base);
  count_launches(1);
  return cudaPeekAtLastError();
}

cudaError_t attn_rope_decode_launch(const float *QKV, float *CK, float *CV, const int *POS,
                                    float *C, const AttnGeom &g, const float2 *rope,
                                    void *scratch, cudaStream_t st) {
  if (g.B == 0 || g.heads == 0) return cudaSuccess;
  if (!rope_split_ok(g) || !scratch || !aligned16(CK) || !aligned16(CV))
    return cudaErrorInvalidValue;
  const dim3 grid(g.nsplit, g.B * g.kvheads);
  float *part = (float *)scratch;
  cudaError_t e = cudaErrorInvalidValue;
#define NL_ATTN(HD, G)                                                                    \
  case G:                                                                                 \
    e = launch_pdl(attn_rope_partial_kernel<HD, G>, grid, dim3(kAttnWarps * 32), 0, st, QKV, \
                   CK, CV, POS, g, rope, part);                                           \
    break;
#define NL_HD(HD)                                                                         \
  case HD:                                                                                \
    switch (g.grp) {                                                                      \
      NL_ATTN(HD, 1) NL_ATTN(HD, 2) NL_ATTN(HD, 3) NL_ATTN(HD, 4)                         \
      NL_ATTN(HD, 5) NL_ATTN(HD, 6) NL_ATTN(HD, 7) NL_ATTN(HD, 8)                         \
      default: break;                                                                     \
    }                                                                                     \
    if (e == cudaSuccess)                                                                 \
      e = launch_pdl(attn_combine_kernel<HD>, dim3(g.B * g.heads), dim3(HD < 128 ? HD : 128), \
                     0, st, (const float *)part, g, C, (uint64_t)UINT64_MAX);             \
    break;
  switch (g.hd) {
    NL_HD(32) NL_HD(64) NL_HD(128) NL_HD(256)
    default: break;
  }
#undef NL_HD
#undef NL_ATTN
  count_launches(2);
  return e;
}
size_t attn_rope_scratch_bytes(const AttnGeom &g) {
  if (!rope_split_ok(g)) return 0;
  return (size_t)g.B * g.heads * g.nsplit * (g.hd + 2) * sizeof(float);
}

const OpSpec kAttnOps[] = {
    {"rope-half", 2, 5, chk_rope_half, no_scratch, run_rope_half},
    {"decode-rope", 6, 2, chk_decode_rope<false>, no_scratch, run_decode_rope<false>},
    {"decode-rope-b", 6, 3, chk_decode_rope<true>, no_scratch, run_decode_rope<true>},
    {"cache-append", 3, 1, chk_cache_append<false>, no_scratch, run_cache_append<false>},
    {"cache-append-b", 3, 3, chk_cache_append<true>, no_scratch, run_cache_append<true>},
    {"decode-attn", 5, 3, chk_attn<false>, scr_attn<false>, run_attn<false>},
    {"decode-attn-b", 5, 5, chk_attn<true>, scr_attn<true>, run_attn<true>},
};
const int kAttnOpsCount = sizeof(kAttnOps) / sizeof(kAttnOps[0]);

}  // namespace nl

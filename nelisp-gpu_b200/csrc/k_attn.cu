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
#include "ternary_prep.cuh"

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
  // Warp w takes the groups of U rows starting at p0 + w U, p0 + (w + 4) U,
  // ...  The next group's rows are requested before the current group is
  // folded (two groups in registers).  U = 2 keeps the kernel within the
  // 72 registers a thread that let 7 CTAs share an SM (one wave of splits);
  // more query heads per KV head take U = 1 for the same reason.
  constexpr int U = GRP <= 2 ? 2 : 1;
  auto load_rows = [&](uint32_t j0, float (&kr)[U][DPL], float (&vr)[U][DPL]) {
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
  };
  {
    float kr[U][DPL], vr[U][DPL];
    uint32_t j0 = p0 + warp * U;
    if (j0 < pc) load_rows(j0, kr, vr);
    for (; j0 < pc; j0 += kAttnWarps * U) {
      float kq[U][DPL], vq[U][DPL];
      const uint32_t jn = j0 + kAttnWarps * U;
      if (jn < pc) load_rows(jn, kq, vq);
#pragma unroll
      for (int u = 0; u < U; u++) {
        if (j0 + u >= pc) break;
        fold(kr[u], vr[u]);
      }
#pragma unroll
      for (int u = 0; u < U; u++)
#pragma unroll
        for (int d = 0; d < DPL; d++) {
          kr[u][d] = kq[u][d];
          vr[u][d] = vq[u][d];
        }
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

// ---- causal attention over a whole sequence (attn-causal-gqa, prefill) --------
// Reference: lisp/nelisp-gpu-kernels.el:949-990 -- for every (head h, row i),
// softmax over keys j <= i of (q_i . k_j) / sqrt(hd), context = sum p_j v_j,
// kv head h / (heads / kvheads).  Here, flash-style in f32 on the CUDA cores
// (TF32 products would miss the 1e-4 bar): one CTA per (sequence, head,
// 32-row query block) walks 64-key tiles up to the diagonal with an online
// softmax.  Threads ty*16 .. ty*16+15 own query rows 4ty .. 4ty+3: their
// scores (4 rows x 4 keys each) and their context columns (4 rows x HD/16),
// so the running max / sum stay in registers.  Q, K and the probabilities
// are kept transposed in shared memory ([dim][row], [dim][key], [key][row]),
// so each operand group of four is one 128-bit load: two loads per 16 FMAs
// for the scores, three per 32 for the context.  Query blocks are issued
// from the last (the longest causal walk) to the first.
constexpr int kCausalBK = 64;

struct CausalGeom {
  uint32_t seq, heads, kvheads;
  uint64_t q_row, kv_row;           // row strides (floats) of Q / CTX and of K / V
  uint64_t q_batch, kv_batch;       // sequence strides (floats), grid z
  uint64_t limit;                   // invocations (h * seq + i) to compute
};

// Shared-memory strides (floats) of the transposed arrays: four past the
// row length keeps rows 16-byte aligned and staggers the transposing stores
// over the banks.
template <int BQ>
struct CausalTile {
  static constexpr int kThreads = 4 * BQ;          // 16 threads per 4 query rows
  static constexpr int QS = BQ + 4, KS = kCausalBK + 4, PS = BQ + 4;
};

// Stage ROWS rows x HD columns of SRC (row stride LD, rows past NROWS read
// as 0) transposed into DST[col * STRIDE + row].  A warp takes 8 rows x 4
// float4 columns: 64-byte runs from global memory, stores spread over the
// banks by the padded stride.
template <int HD, int ROWS, int STRIDE, int NT>
__device__ __forceinline__ void stage_transposed(float *dst, const float *src, uint64_t ld,
                                                 uint32_t nrows, int tid) {
  constexpr int kLogRows = ROWS == 32 ? 5 : 6;
  static_assert(ROWS == 32 || ROWS == 64, "tile rows");
  for (int e = tid; e < ROWS * HD / 4; e += NT) {
    const int r = (e >> 2) & (ROWS - 1), c4 = ((e >> (2 + kLogRows)) << 2) | (e & 3);
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if ((uint32_t)r < nrows) v = *reinterpret_cast<const float4 *>(src + (uint64_t)r * ld + 4 * c4);
    dst[(4 * c4 + 0) * STRIDE + r] = v.x;
    dst[(4 * c4 + 1) * STRIDE + r] = v.y;
    dst[(4 * c4 + 2) * STRIDE + r] = v.z;
    dst[(4 * c4 + 3) * STRIDE + r] = v.w;
  }
}

template <int HD, int BQ>
__global__ void __launch_bounds__(4 * BQ)
attn_causal_kernel(const float *__restrict__ Q, const float *__restrict__ K,
                   const float *__restrict__ V, float *__restrict__ CTX, CausalGeom g) {
  using T = CausalTile<BQ>;
  constexpr int NT = T::kThreads;
  constexpr int DPT = HD / 16;                     // context columns per thread
  extern __shared__ __align__(16) float smc[];
  float *Qt = smc;                                 // [HD][QS]
  float *Kt = Qt + HD * T::QS;                     // [HD][KS]
  float *Vs = Kt + HD * T::KS;                     // [BK][HD]
  float *Pt = Vs + kCausalBK * HD;                 // [BK][PS]
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const uint32_t q0 = (gridDim.x - 1u - blockIdx.x) * BQ, h = blockIdx.y, bz = blockIdx.z;
  const uint32_t kvh = h / (g.heads / g.kvheads);
  const float *Qb = Q + bz * g.q_batch + (uint64_t)h * HD;
  const float *Kb = K + bz * g.kv_batch + (uint64_t)kvh * HD;
  const float *Vb = V + bz * g.kv_batch + (uint64_t)kvh * HD;
  const float scale = 1.0f / sqrtf((float)HD);
  stage_transposed<HD, BQ, T::QS, NT>(Qt, Qb + (uint64_t)q0 * g.q_row, g.q_row,
                                      g.seq > q0 ? g.seq - q0 : 0u, tid);
  float m[4], l[4], o[4][DPT];
#pragma unroll
  for (int a = 0; a < 4; a++) {
    m[a] = -INFINITY;
    l[a] = 0.0f;
#pragma unroll
    for (int c = 0; c < DPT; c++) o[a][c] = 0.0f;
  }
  const uint32_t kend = min(g.seq, q0 + BQ);       // keys past the block's last row
  for (uint32_t k0 = 0; k0 < kend; k0 += kCausalBK) {
    __syncthreads();
    stage_transposed<HD, kCausalBK, T::KS, NT>(Kt, Kb + (uint64_t)k0 * g.kv_row, g.kv_row,
                                               g.seq - k0, tid);
    for (int e = tid; e < kCausalBK * HD / 4; e += NT) {
      const int r = e / (HD / 4), c4 = e % (HD / 4);
      const uint32_t j = k0 + r;
      float4 vv = make_float4(0.f, 0.f, 0.f, 0.f);
      if (j < g.seq) vv = *reinterpret_cast<const float4 *>(Vb + j * g.kv_row + 4 * c4);
      reinterpret_cast<float4 *>(Vs + r * HD)[c4] = vv;
    }
    __syncthreads();
    // scores: rows 4ty + a, keys 4tx + b, summed over d in order
    float sc[4][4];
#pragma unroll
    for (int a = 0; a < 4; a++)
#pragma unroll
      for (int b = 0; b < 4; b++) sc[a][b] = 0.0f;
#pragma unroll 8
    for (int d = 0; d < HD; d++) {
      const float4 kk = *reinterpret_cast<const float4 *>(Kt + d * T::KS + 4 * tx);
      const float4 qq = *reinterpret_cast<const float4 *>(Qt + d * T::QS + 4 * ty);
      const float qa[4] = {qq.x, qq.y, qq.z, qq.w};
#pragma unroll
      for (int a = 0; a < 4; a++) {
        sc[a][0] = fmaf(qa[a], kk.x, sc[a][0]);
        sc[a][1] = fmaf(qa[a], kk.y, sc[a][1]);
        sc[a][2] = fmaf(qa[a], kk.z, sc[a][2]);
        sc[a][3] = fmaf(qa[a], kk.w, sc[a][3]);
      }
    }
    // causal mask, online softmax per row (reductions over the 16 threads of a row)
    float pr[4][4];
#pragma unroll
    for (int a = 0; a < 4; a++) {
      const uint32_t i = q0 + 4 * ty + a;
      float rmax = -INFINITY;
#pragma unroll
      for (int b = 0; b < 4; b++) {
        const uint32_t j = k0 + 4 * tx + b;
        sc[a][b] = (j <= i && j < g.seq) ? sc[a][b] * scale : -INFINITY;
        rmax = fmaxf(rmax, sc[a][b]);
      }
      for (int off = 8; off > 0; off >>= 1)
        rmax = fmaxf(rmax, __shfl_xor_sync(0xffffffffu, rmax, off));
      const float mn = fmaxf(m[a], rmax);
      const float corr = mn == -INFINITY ? 1.0f : expf(m[a] - mn);   // exp(-inf) = 0
      float rsum = 0.0f;
#pragma unroll
      for (int b = 0; b < 4; b++) {
        const float p = mn == -INFINITY ? 0.0f : expf(sc[a][b] - mn);
        pr[a][b] = p;
        rsum += p;
      }
      for (int off = 8; off > 0; off >>= 1) rsum += __shfl_xor_sync(0xffffffffu, rsum, off);
      l[a] = l[a] * corr + rsum;
      m[a] = mn;
#pragma unroll
      for (int c = 0; c < DPT; c++) o[a][c] *= corr;
    }
    // The probabilities of rows 4ty .. 4ty+3 are written and read by the 16
    // threads that own those rows, all in one warp.
#pragma unroll
    for (int b = 0; b < 4; b++)
      *reinterpret_cast<float4 *>(Pt + (4 * tx + b) * T::PS + 4 * ty) =
          make_float4(pr[0][b], pr[1][b], pr[2][b], pr[3][b]);
    __syncwarp();
    // context: rows 4ty + a, columns tx*DPT .. tx*DPT + DPT-1
    const int jn = (int)min((uint32_t)kCausalBK, kend - k0);
    for (int j = 0; j < jn; j++) {
      const float4 pp = *reinterpret_cast<const float4 *>(Pt + j * T::PS + 4 * ty);
      const float pa[4] = {pp.x, pp.y, pp.z, pp.w};
      float vv[DPT];
#pragma unroll
      for (int c4 = 0; c4 < DPT / 4; c4++) {
        const float4 v4 = *reinterpret_cast<const float4 *>(Vs + j * HD + tx * DPT + 4 * c4);
        vv[4 * c4] = v4.x; vv[4 * c4 + 1] = v4.y; vv[4 * c4 + 2] = v4.z; vv[4 * c4 + 3] = v4.w;
      }
#pragma unroll
      for (int a = 0; a < 4; a++)
#pragma unroll
        for (int c = 0; c < DPT; c++) o[a][c] = fmaf(pa[a], vv[c], o[a][c]);
    }
  }
#pragma unroll
  for (int a = 0; a < 4; a++) {
    const uint32_t i = q0 + 4 * ty + a;
    if (i >= g.seq || (uint64_t)h * g.seq + i >= g.limit) continue;
    float *cr = CTX + bz * g.q_batch + i * g.q_row + (uint64_t)h * HD + tx * DPT;
#pragma unroll
    for (int c = 0; c < DPT; c++) cr[c] = o[a][c] / l[a];
  }
}

// ---- causal attention on the tensor cores (3xTF32) ----------------------------
// The same operation as attn_causal_kernel with both products, Q K^T and
// P V, on mma.sync.m16n8k8 tf32: every f32 operand x is split into a tf32
// x_big and the rest x_small (tf32_split), and each product is summed as
// a_small b_big + a_big b_small + a_big b_big (the small x small term, about
// 2^-20 of the product, is dropped), accumulating in f32.
//
// One CTA of 4 warps per (sequence, head, 16-row query block): the CTA
// stages 32-key tiles of K and V up to the diagonal into shared memory, and
// warp w takes keys 8w .. 8w+7 of every tile for all 16 rows, with its own
// online softmax; the four warps' (max, sum, context) are merged at the end
// in warp order.  Splitting the keys over the warps gives a 512-row prefill
// of 20 heads 2560 warps instead of 640.  Q is kept split (tf32 big, small)
// in shared memory; K and V as f32 rows padded by 4 floats, which makes
// every fragment load conflict-free.  The probabilities are taken from the
// score accumulators as the A operand of P V as they are: the MMA's K index
// t stands for key 2t and t + 4 for key 2t + 1 of the warp's 8 keys, and the
// V fragments are read in that order.  Query blocks are issued from the last
// (the longest causal walk) to the first.
constexpr int kTcBQ = 16, kTcBK = 32;
// x = big + small: big keeps the sign, exponent and top 10 mantissa bits of
// x (the low 13 bits cleared: a truncation, one instruction), small = x - big
// is exact in f32, and the tensor core reads it as tf32 (its low 13 bits
// ignored).  The products keep about 20 bits.
__device__ __forceinline__ void tf32_split(float x, uint32_t &big, uint32_t &small) {
  big = __float_as_uint(x) & 0xFFFFE000u;
  small = __float_as_uint(x - __uint_as_float(big));
}
__device__ __forceinline__ void mma_tf32(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
// d += a b with both split: a_small b_big + a_big b_small + a_big b_big.
__device__ __forceinline__ void mma_3xtf32(float (&d)[4], const uint32_t (&ab)[4],
                                           const uint32_t (&as)[4], uint32_t bb0, uint32_t bb1,
                                           uint32_t bs0, uint32_t bs1) {
  mma_tf32(d, as, bb0, bb1);
  mma_tf32(d, ab, bs0, bs1);
  mma_tf32(d, ab, bb0, bb1);
}
__host__ __device__ constexpr size_t causal_tc_smem(int hd) {
  // Q split [BQ][HD + 4] uint2, then K and V [BK][HD + 4] floats each (the
  // merge reuses K and V for the warps' contexts: 4 x 16 x HD floats)
  return (size_t)kTcBQ * (hd + 4) * 8u + (size_t)2 * kTcBK * (hd + 4) * 4u + 2u * 4u * kTcBQ * 4u;
}

template <int HD>
__global__ void __launch_bounds__(128)
attn_causal_tc_kernel(const float *__restrict__ Q, const float *__restrict__ K,
                      const float *__restrict__ V, float *__restrict__ CTX, CausalGeom g) {
  constexpr int LD = HD + 4, NO = HD / 8;
  static_assert(4 * kTcBQ * HD <= 2 * kTcBK * LD, "the merge fits the K and V tiles");
  extern __shared__ __align__(16) float smt[];
  uint2 *Qs = reinterpret_cast<uint2 *>(smt);                 // [BQ][LD] (big, small)
  float *Ks = smt + 2 * kTcBQ * LD;                           // [BK][LD]
  float *Vs = Ks + kTcBK * LD;                                // [BK][LD]
  float *Ms = Vs + kTcBK * LD;                                // [4 warps][BQ]
  float *Ls = Ms + 4 * kTcBQ;                                 // [4 warps][BQ]
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, gq = lane >> 2, t4 = lane & 3;
  const uint32_t q0 = (gridDim.x - 1u - blockIdx.x) * kTcBQ, h = blockIdx.y, bz = blockIdx.z;
  const uint32_t kvh = h / (g.heads / g.kvheads);
  const float *Qb = Q + bz * g.q_batch + (uint64_t)h * HD;
  const float *Kb = K + bz * g.kv_batch + (uint64_t)kvh * HD;
  const float *Vb = V + bz * g.kv_batch + (uint64_t)kvh * HD;
  const float scale = 1.0f / sqrtf((float)HD);
  // Q rows, split once (rows past seq as 0)
  for (int e = tid; e < kTcBQ * HD / 4; e += 128) {
    const int r = e / (HD / 4), c4 = e % (HD / 4);
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (q0 + (uint32_t)r < g.seq)
      v = *reinterpret_cast<const float4 *>(Qb + (uint64_t)(q0 + r) * g.q_row + 4 * c4);
    const float f[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; i++) {
      uint32_t b, sm;
      tf32_split(f[i], b, sm);
      Qs[r * LD + 4 * c4 + i] = make_uint2(b, sm);
    }
  }
  float o[NO][4], m[2], l[2];
#pragma unroll
  for (int dt = 0; dt < NO; dt++) o[dt][0] = o[dt][1] = o[dt][2] = o[dt][3] = 0.0f;
  m[0] = m[1] = -INFINITY;
  l[0] = l[1] = 0.0f;
  const uint32_t kend = min(g.seq, q0 + kTcBQ);
  for (uint32_t k0 = 0; k0 < kend; k0 += kTcBK) {
    __syncthreads();                               // the previous tile is consumed
    // the K and V tiles by cp.async (no register round trip; rows past seq
    // are zero-filled without a read)
    for (int e = tid; e < kTcBK * HD / 4; e += 128) {
      const int r = e / (HD / 4), c4 = e % (HD / 4);
      const bool in = k0 + (uint32_t)r < g.seq;
      const uint64_t go = in ? (uint64_t)(k0 + r) * g.kv_row + 4 * c4 : 0;
      const unsigned n = in ? 16u : 0u;            // 0: zero fill
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n"
                   ::"r"((unsigned)__cvta_generic_to_shared(Ks + r * LD + 4 * c4)),
                   "l"(Kb + go), "r"(n) : "memory");
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n"
                   ::"r"((unsigned)__cvta_generic_to_shared(Vs + r * LD + 4 * c4)),
                   "l"(Vb + go), "r"(n) : "memory");
    }
    asm volatile("cp.async.commit_group;\ncp.async.wait_all;\n" ::: "memory");
    __syncthreads();
    const uint32_t kw = k0 + 8u * (uint32_t)warp;  // this warp's 8 keys
    if (kw > q0 + kTcBQ - 1u || kw >= g.seq) continue;   // all past every row of the block
    // scores of rows gq, gq + 8 and keys kw + 2 t4 (+1)
    float sc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    const uint2 *qa = Qs + gq * LD + t4;
    const float *kb = Ks + (8 * warp + gq) * LD + t4;
#pragma unroll 8
    for (int kk = 0; kk < HD / 8; kk++) {
      const uint2 x0 = qa[8 * kk], x1 = qa[8 * LD + 8 * kk];
      const uint2 x2 = qa[8 * kk + 4], x3 = qa[8 * LD + 8 * kk + 4];
      const uint32_t ab[4] = {x0.x, x1.x, x2.x, x3.x}, as[4] = {x0.y, x1.y, x2.y, x3.y};
      uint32_t bb0, bs0, bb1, bs1;
      tf32_split(kb[8 * kk], bb0, bs0);
      tf32_split(kb[8 * kk + 4], bb1, bs1);
      mma_3xtf32(sc, ab, as, bb0, bb1, bs0, bs1);
    }
    // causal mask and online softmax over this warp's keys; a row's 8 keys
    // sit in the 4 lanes of its quad
#pragma unroll
    for (int hf = 0; hf < 2; hf++) {
      const uint32_t i = q0 + (uint32_t)gq + 8u * hf;
      float mx = -INFINITY;
#pragma unroll
      for (int e = 0; e < 2; e++) {
        const uint32_t j = kw + 2u * t4 + e;
        const float v = (j <= i && j < g.seq) ? sc[2 * hf + e] * scale : -INFINITY;
        sc[2 * hf + e] = v;
        mx = fmaxf(mx, v);
      }
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      const float mn = fmaxf(m[hf], mx);
      const float corr = mn == -INFINITY ? 1.0f : expf(m[hf] - mn);   // exp(-inf) = 0
      float sum = 0.0f;
#pragma unroll
      for (int e = 0; e < 2; e++) {
        const float p = mn == -INFINITY ? 0.0f : expf(sc[2 * hf + e] - mn);
        sc[2 * hf + e] = p;
        sum += p;
      }
      sum += __shfl_xor_sync(0xffffffffu, sum, 1);
      sum += __shfl_xor_sync(0xffffffffu, sum, 2);
      l[hf] = l[hf] * corr + sum;
      m[hf] = mn;
#pragma unroll
      for (int dt = 0; dt < NO; dt++) {
        o[dt][2 * hf] *= corr;
        o[dt][2 * hf + 1] *= corr;
      }
    }
    // context += P V over the warp's 8 keys
    uint32_t pb[4], ps[4];
    tf32_split(sc[0], pb[0], ps[0]);               // P[gq][2 t4]
    tf32_split(sc[2], pb[1], ps[1]);               // P[gq + 8][2 t4]
    tf32_split(sc[1], pb[2], ps[2]);               // P[gq][2 t4 + 1]
    tf32_split(sc[3], pb[3], ps[3]);               // P[gq + 8][2 t4 + 1]
    const float *vb = Vs + (8 * warp + 2 * t4) * LD + gq;
#pragma unroll
    for (int dt = 0; dt < NO; dt++) {
      uint32_t bb0, bs0, bb1, bs1;
      tf32_split(vb[8 * dt], bb0, bs0);            // V[key 2 t4][dim 8 dt + gq]
      tf32_split(vb[LD + 8 * dt], bb1, bs1);       // V[key 2 t4 + 1][dim 8 dt + gq]
      mma_3xtf32(o[dt], pb, ps, bb0, bb1, bs0, bs1);
    }
  }
  // merge the warps: max, then the rescaled sums in warp order
  __syncthreads();                                 // K and V are free
  float *Os = Ks;                                  // [4 warps][BQ][HD]
#pragma unroll
  for (int hf = 0; hf < 2; hf++) {
    const int r = gq + 8 * hf;
    if (t4 == 0) {
      Ms[warp * kTcBQ + r] = m[hf];
      Ls[warp * kTcBQ + r] = l[hf];
    }
#pragma unroll
    for (int dt = 0; dt < NO; dt++)
      *reinterpret_cast<float2 *>(Os + ((size_t)warp * kTcBQ + r) * HD + 8 * dt + 2 * t4) =
          make_float2(o[dt][2 * hf], o[dt][2 * hf + 1]);
  }
  __syncthreads();
  for (int e = tid; e < kTcBQ * HD; e += 128) {
    const int r = e / HD, d = e % HD;
    const uint32_t i = q0 + (uint32_t)r;
    if (i >= g.seq || (uint64_t)h * g.seq + i >= g.limit) continue;
    float mm = -INFINITY;
#pragma unroll
    for (int w = 0; w < 4; w++) mm = fmaxf(mm, Ms[w * kTcBQ + r]);
    float ll = 0.0f, oo = 0.0f;
#pragma unroll
    for (int w = 0; w < 4; w++) {
      const float mw = Ms[w * kTcBQ + r];
      if (mw > -INFINITY) {
        const float c = expf(mw - mm);
        ll += Ls[w * kTcBQ + r] * c;
        oo += Os[((size_t)w * kTcBQ + r) * HD + d] * c;
      }
    }
    CTX[bz * g.q_batch + i * g.q_row + (uint64_t)h * HD + d] = oo / ll;
  }
}

// Any head size: the reference's three passes, one thread per (head, row).
__global__ void attn_causal_simple_kernel(const float *__restrict__ Q, const float *__restrict__ K,
                                          const float *__restrict__ V, float *__restrict__ CTX,
                                          CausalGeom g, uint32_t hd) {
  const uint64_t idx = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (uint64_t)g.heads * g.seq || idx >= g.limit) return;
  const uint32_t h = (uint32_t)(idx / g.seq), i = (uint32_t)(idx % g.seq);
  const uint32_t kvh = h / (g.heads / g.kvheads);
  const float *q = Q + i * g.q_row + (uint64_t)h * hd;
  const float scale = 1.0f / sqrtf((float)hd);
  auto score = [&](uint32_t j) {
    const float *k = K + j * g.kv_row + (uint64_t)kvh * hd;
    float acc = 0.0f;
    for (uint32_t t = 0; t < hd; t++) acc = fmaf(q[t], k[t], acc);
    return acc * scale;
  };
  float mx = -1.0e30f;
  for (uint32_t j = 0; j <= i; j++) mx = fmaxf(mx, score(j));
  float sm = 0.0f;
  for (uint32_t j = 0; j <= i; j++) sm += expf(score(j) - mx);
  float *c = CTX + i * g.q_row + (uint64_t)h * hd;
  for (uint32_t t = 0; t < hd; t++) c[t] = 0.0f;
  for (uint32_t j = 0; j <= i; j++) {
    const float p = expf(score(j) - mx) / sm;
    const float *v = V + j * g.kv_row + (uint64_t)kvh * hd;
    for (uint32_t t = 0; t < hd; t++) c[t] = fmaf(p, v[t], c[t]);
  }
}

template <int BQ>
size_t causal_smem(int hd) {
  using T = CausalTile<BQ>;
  return ((size_t)hd * T::QS + (size_t)hd * T::KS + (size_t)kCausalBK * hd +
          (size_t)kCausalBK * T::PS) * sizeof(float);
}

// Query block: 32 rows by default (a shorter causal critical path and twice
// the CTAs; measured faster than 64 rows at 512 and 2048 rows on B200:
// 126 vs 150 us and 1137 vs 1270 us for 20 heads x 128).
// NELISP_CAUSAL_BQ=64 selects 64-row blocks.
template <int HD, int BQ>
cudaError_t causal_fast(const float *Q, const float *K, const float *V, float *CTX,
                        const CausalGeom &g, uint32_t batch, cudaStream_t st) {
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(attn_causal_kernel<HD, BQ>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)causal_smem<BQ>(HD));
    if (e != cudaSuccess) return e;
    configured = true;
  }
  const dim3 grid((g.seq + BQ - 1) / BQ, g.heads, batch);
  attn_causal_kernel<HD, BQ><<<grid, CausalTile<BQ>::kThreads, causal_smem<BQ>(HD), st>>>(
      Q, K, V, CTX, g);
  count_launches(1);
  return cudaPeekAtLastError();
}

template <int HD>
cudaError_t causal_tc(const float *Q, const float *K, const float *V, float *CTX,
                      const CausalGeom &g, uint32_t batch, cudaStream_t st) {
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(attn_causal_tc_kernel<HD>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)causal_tc_smem(HD));
    if (e != cudaSuccess) return e;
    configured = true;
  }
  const dim3 grid((g.seq + kTcBQ - 1) / kTcBQ, g.heads, batch);
  attn_causal_tc_kernel<HD><<<grid, 128, causal_tc_smem(HD), st>>>(Q, K, V, CTX, g);
  count_launches(1);
  return cudaPeekAtLastError();
}

cudaError_t causal_launch(const float *Q, const float *K, const float *V, float *CTX,
                          const CausalGeom &g, uint32_t hd, uint32_t batch, cudaStream_t st) {
  if (g.seq == 0 || g.heads == 0 || batch == 0) return cudaSuccess;
  const bool fast = (hd == 64 || hd == 128) && aligned16(Q) && aligned16(K) && aligned16(V) &&
                    aligned16(CTX) && g.q_row % 4 == 0 && g.kv_row % 4 == 0 &&
                    g.q_batch % 4 == 0 && g.kv_batch % 4 == 0;
  if (fast) {
    // NELISP_CAUSAL_PATH=ffma: the CUDA-core kernel instead of the tensor cores
    static const bool ffma = [] {
      const char *v = getenv("NELISP_CAUSAL_PATH");
      return v && strcmp(v, "ffma") == 0;
    }();
    if (!ffma) return hd == 128 ? causal_tc<128>(Q, K, V, CTX, g, batch, st)
                                : causal_tc<64>(Q, K, V, CTX, g, batch, st);
    static const int forced = [] {
      const char *v = getenv("NELISP_CAUSAL_BQ");
      return v ? atoi(v) : 0;
    }();
    const bool small = forced != 64;
    if (hd == 128)
      return small ? causal_fast<128, 32>(Q, K, V, CTX, g, batch, st)
                   : causal_fast<128, 64>(Q, K, V, CTX, g, batch, st);
    return small ? causal_fast<64, 32>(Q, K, V, CTX, g, batch, st)
                 : causal_fast<64, 64>(Q, K, V, CTX, g, batch, st);
  }
  for (uint32_t b = 0; b < batch; b++) {
    attn_causal_simple_kernel<<<(unsigned)ceil_div64((uint64_t)g.heads * g.seq, 128), 128, 0, st>>>(
        Q + b * g.q_batch, K + b * g.kv_batch, V + b * g.kv_batch, CTX + b * g.q_batch, g, hd);
    count_launches(1);
  }
  return cudaPeekAtLastError();
}

// One CTA per (b, h): merge the splits and write C.
// One head's merge at output lane d: the NSPLIT partials (max, sum, HD
// outputs each) are combined with the global maximum first, then the scaled
// sums in split order.  Up to kMergeBatch splits -- a decode step's usual
// count -- are loaded in one round trip; more take two passes in batches.
constexpr int kMergeBatch = 32;
template <int HD>
__device__ __forceinline__ float merge_splits(const float *__restrict__ pp, uint32_t nsplit,
                                              uint32_t d) {
  if (nsplit <= (uint32_t)kMergeBatch) {
    float mv[kMergeBatch], lv[kMergeBatch], ov[kMergeBatch];
#pragma unroll
    for (int u = 0; u < kMergeBatch; u++) {
      const bool in = (uint32_t)u < nsplit;
      const float *ps = pp + (uint64_t)u * (HD + 2);
      mv[u] = in ? ps[0] : -INFINITY;
      lv[u] = in ? ps[1] : 0.0f;
      ov[u] = in ? ps[2 + d] : 0.0f;
    }
    float mm = -INFINITY;
#pragma unroll
    for (int u = 0; u < kMergeBatch; u++) mm = fmaxf(mm, mv[u]);
    float ll = 0.0f, oo = 0.0f;
#pragma unroll
    for (int u = 0; u < kMergeBatch; u++) {
      if (mv[u] > -INFINITY) {
        const float c = expf(mv[u] - mm);
        ll += lv[u] * c;
        oo += ov[u] * c;
      }
    }
    return oo / ll;
  }
  constexpr int SB = 8;
  float mm = -INFINITY;
  for (uint32_t s0 = 0; s0 < nsplit; s0 += SB) {
    float mv[SB];
#pragma unroll
    for (int u = 0; u < SB; u++)
      mv[u] = s0 + u < nsplit ? pp[(uint64_t)(s0 + u) * (HD + 2)] : -INFINITY;
#pragma unroll
    for (int u = 0; u < SB; u++) mm = fmaxf(mm, mv[u]);
  }
  float ll = 0.0f, oo = 0.0f;
  for (uint32_t s0 = 0; s0 < nsplit; s0 += SB) {
    float mv[SB], lv[SB], ov[SB];
#pragma unroll
    for (int u = 0; u < SB; u++) {
      const bool in = s0 + u < nsplit;
      const float *ps = pp + (uint64_t)(s0 + u) * (HD + 2);
      mv[u] = in ? ps[0] : -INFINITY;
      lv[u] = in ? ps[1] : 0.0f;
      ov[u] = in ? ps[2 + d] : 0.0f;
    }
#pragma unroll
    for (int u = 0; u < SB; u++) {
      if (mv[u] > -INFINITY) {
        const float c = expf(mv[u] - mm);
        ll += lv[u] * c;
        oo += ov[u] * c;
      }
    }
  }
  return oo / ll;
}

template <int HD>
__global__ void attn_combine_kernel(const float *__restrict__ part, AttnGeom g,
                                    float *__restrict__ C, uint64_t limit) {
  pdl_wait();
  const uint32_t bh = blockIdx.x;
  const uint32_t bb = bh / g.heads, h = bh % g.heads;
  const float *pp = part + (uint64_t)bh * g.nsplit * (HD + 2);
  for (uint32_t d = threadIdx.x; d < HD; d += blockDim.x) {
    const uint64_t idx = (uint64_t)bb * g.heads * HD + (uint64_t)h * HD + d;
    const float v = merge_splits<HD>(pp, g.nsplit, d);
    if (idx < limit) C[idx] = v;
  }
}

// The decoder's combine: attn_combine_kernel's merge, then the last CTA of
// sequence row b to finish (ROW_CTR[b] counts the row's heads; that CTA
// resets it for the next launch) quantizes the row's context C[b] (heads *
// HD columns) into WS, the O-projection GEMV's activation workspace for
// g.B rows -- the work of a separate prep launch.  Other CTAs' C values are
// read through L2 after a fence on both sides of the counter.
template <int HD>
__global__ void attn_combine_prep_kernel(const float *__restrict__ part, AttnGeom g,
                                         float *__restrict__ C, void *ws, int *row_ctr) {
  pdl_trigger();                 // the O-projection may start streaming its weights
  pdl_wait();
  extern __shared__ __align__(16) float xrow[];   // the finished row, for the last CTA
  __shared__ float red[32];
  __shared__ long long xred[32];
  __shared__ int s_last;
  const uint32_t bh = blockIdx.x;
  const uint32_t bb = bh / g.heads, h = bh % g.heads;
  const float *pp = part + (uint64_t)bh * g.nsplit * (HD + 2);
  for (uint32_t d = threadIdx.x; d < HD; d += blockDim.x)
    C[(uint64_t)bb * g.heads * HD + (uint64_t)h * HD + d] = merge_splits<HD>(pp, g.nsplit, d);
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    s_last = atomicAdd(row_ctr + bb, 1) == (int)g.heads - 1;
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  // The last CTA of the row: the whole row into shared memory in one round
  // trip (every float4 load issued before any is used), its maximum, then
  // the prep's quantisation from shared memory (prep_row_cta's format: the
  // CTA's offset sum in slot 0, the other slots zeroed).
  const uint32_t cols = g.heads * (uint32_t)HD, n4 = cols / 4u;
  const float4 *c4 = reinterpret_cast<const float4 *>(C + (uint64_t)bb * cols);
  float4 *x4 = reinterpret_cast<float4 *>(xrow);
  constexpr int LB = 8;
  float mx = 0.0f;
  int bad = 0;
  for (uint32_t i0 = threadIdx.x; i0 < n4; i0 += LB * blockDim.x) {
    float4 v[LB];
#pragma unroll
    for (int u = 0; u < LB; u++) {
      const uint32_t i = i0 + (uint32_t)u * blockDim.x;
      v[u] = i < n4 ? __ldcg(c4 + i) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int u = 0; u < LB; u++) {
      const uint32_t i = i0 + (uint32_t)u * blockDim.x;
      if (i < n4) {
        x4[i] = v[u];
        mx = fmaxf(fmaxf(mx, fmaxf(fabsf(v[u].x), fabsf(v[u].y))),
                   fmaxf(fabsf(v[u].z), fabsf(v[u].w)));
        bad |= !isfinite(v[u].x) | !isfinite(v[u].y) | !isfinite(v[u].z) | !isfinite(v[u].w);
      }
    }
  }
  const int nw = (int)(blockDim.x >> 5), w = (int)(threadIdx.x >> 5), lane = (int)(threadIdx.x & 31);
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if (lane == 0) red[w] = mx;
  bad = __syncthreads_or(bad);
  float rm = 0.0f;
  for (int i = 0; i < nw; i++) rm = fmaxf(rm, red[i]);
  PrepOut P = prep_at(ws, (int)g.B, cols, 0);
  const int NT = n_tiles((int)g.B), L = n_limbs((int)g.B);
  float mul = 0.0f, inv = 0.0f;
  const bool ok = row_scale(rm, bad != 0, &mul, &inv, L);
  if (threadIdx.x == 0) {
    P.rowinv[bb] = inv;
    P.rowflag[bb] = !ok;
  }
  long long partx = 0;
  for (uint32_t W = threadIdx.x; W < cols / 16u; W += blockDim.x) {
    float q[16];
#pragma unroll
    for (int e = 0; e < 4; e++) {
      const float4 f = x4[4u * W + e];
      q[4 * e] = f.x; q[4 * e + 1] = f.y; q[4 * e + 2] = f.z; q[4 * e + 3] = f.w;
    }
    partx += quantize_word(q, mul, ok, W, bb, NT, L, P);
  }
  for (int o = 16; o > 0; o >>= 1) partx += __shfl_xor_sync(0xffffffffu, partx, o);
  if (lane == 0) xred[w] = partx;
  __syncthreads();
  if (threadIdx.x < (unsigned)kRowCluster) {
    long long t = 0;
    if (threadIdx.x == 0)
      for (int i = 0; i < nw; i++) t += xred[i];
    P.xsum[bb * kRowCluster + threadIdx.x] = t;
  }
  if (threadIdx.x == 0) row_ctr[bb] = 0;
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
  // About one full wave of the split kernel (7 CTAs of 128 threads fit an SM
  // at its register count), at least 32 keys each.
  uint32_t units = B * kvheads;
  uint32_t want = units ? (7u * 148u) / units : 1;
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

// attn-causal-gqa: buffers Q K V CTX, push (seq heads kvheads hd).
const char *chk_causal(const OpArgs &a) {
  const uint64_t seq = a.push[0], heads = a.push[1], kvheads = a.push[2], hd = a.push[3];
  if (heads == 0 || kvheads == 0 || heads % kvheads || hd == 0)
    return fmt_msg("attn-causal-gqa: heads %u, kvheads %u, hd %u do not divide", a.push[1],
                   a.push[2], a.push[3]);
  const char *m;
  if ((m = need_words(a, 0, seq * heads * hd, "Q"))) return m;
  if ((m = need_words(a, 1, seq * kvheads * hd, "K"))) return m;
  if ((m = need_words(a, 2, seq * kvheads * hd, "V"))) return m;
  return need_words(a, 3, seq * heads * hd, "CTX");
}
cudaError_t run_causal(const OpArgs &a) {
  CausalGeom g;
  g.seq = a.push[0];
  g.heads = a.push[1];
  g.kvheads = a.push[2];
  const uint32_t hd = a.push[3];
  g.q_row = (uint64_t)g.heads * hd;
  g.kv_row = (uint64_t)g.kvheads * hd;
  g.q_batch = g.kv_batch = 0;
  g.limit = invocations(a.groups, 64);
  return causal_launch((const float *)a.buf[0], (const float *)a.buf[1], (const float *)a.buf[2],
                       (float *)a.buf[3], g, hd, 1, a.stream);
}

}  // namespace

cudaError_t attn_causal_prefill_launch(const float *Q, const float *CK, const float *CV,
                                       float *CTX, uint32_t B, uint32_t seq, uint32_t heads,
                                       uint32_t kvheads, uint32_t hd, uint64_t q_batch,
                                       uint64_t kv_batch, cudaStream_t st) {
  CausalGeom g;
  g.seq = seq;
  g.heads = heads;
  g.kvheads = kvheads;
  g.q_row = (uint64_t)heads * hd;
  g.kv_row = (uint64_t)kvheads * hd;
  g.q_batch = q_batch;
  g.kv_batch = kv_batch;
  g.limit = UINT64_MAX;
  return causal_launch(Q, CK, CV, CTX, g, hd, B, st);
}

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
                                    void *scratch, cudaStream_t st, void *prep_ws,
                                    int *row_ctr) {
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
    if (e == cudaSuccess && prep_ws && row_ctr && (size_t)g.heads * HD * 4 > (48u << 10)) \
      e = cudaFuncSetAttribute(attn_combine_prep_kernel<HD>,                               \
                               cudaFuncAttributeMaxDynamicSharedMemorySize,                \
                               (int)((size_t)g.heads * HD * 4));                           \
    if (e == cudaSuccess && prep_ws && row_ctr)                                           \
      e = launch_pdl(attn_combine_prep_kernel<HD>, dim3(g.B * g.heads),                   \
                     dim3(HD < 128 ? HD : 128), (size_t)g.heads * HD * 4, st,               \
                     (const float *)part, g, C, prep_ws, row_ctr);                         \
    else if (e == cudaSuccess)                                                            \
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
    {"attn-causal-gqa", 4, 4, chk_causal, no_scratch, run_causal},
};
const int kAttnOpsCount = sizeof(kAttnOps) / sizeof(kAttnOps[0]);

}  // namespace nl

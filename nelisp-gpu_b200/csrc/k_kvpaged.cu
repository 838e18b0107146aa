// k_kvpaged.cu -- paged, ring (attention sink + rolling window) and
// entry-list KV caches for sm_100a.
//
// Reference operators (lisp/nelisp-gpu-kernels.el):
//   cache-append-ring       :396-404   SRC at the ring slot of POS[0]
//   decode-attn-stream      :409-451   single query over sink + window, RoPE
//                                      (adjacent pairs) of q and keys in-kernel
//   qkv-append              :1044-1050 K / V of a fused QKV row into the pools
//   attn-stream-entries     :1057-1092 single query over an entry list
//                                      [physical base, cache-relative pos]
//   cache-append-paged      :1099-1108 B rows into a block-paged pool at POS[0]
//   decode-attn-paged       :1111-1137 per-sequence attention through the table
//   block-copy              :1184-1190 one pool block to another (copy-on-write)
//   decode-rope-b-v         :1195-1207 RoPE of row b at its own length LENS[b]
//   cache-append-paged-v    :1210-1218 B rows, each at LENS[b]
//   decode-attn-paged-v     :1221-1246 sequence s attends 0..LENS[s]
//
// The four attention operators share one split-K kernel (as the contiguous
// decode attention): a CTA takes (split, sequence x kv head); each warp walks
// keys, its lanes holding hd/32 consecutive dims of every query head of the
// group, with an online softmax; a second kernel merges the splits.  What
// differs is only where key j of a sequence lives (and, for the streaming
// operators, the cache-relative position it is rotated by), a compile-time
// mode.  Table and entry values are range-checked: a key whose row would fall
// outside the pool is skipped rather than read.  Head sizes other than 64 and
// 128 take a per-output kernel with the reference's two passes.

#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include "nl_internal.h"

namespace nl {
namespace {

__device__ __forceinline__ uint32_t f2u(float v) {
  return v > 0.0f ? __float2uint_rz(v) : 0u;   // the reference's uint() of a float
}

enum { kModePaged = 0, kModePagedV = 1, kModeRing = 2, kModeEnt = 3 };

struct GatherGeom {
  uint32_t B, dim, heads, kvheads, hd, grp, kvdim;
  uint32_t nsplit, chunk;        // key range per split
  float coef;
  const float *pos;              // POS[0] (paged, ring) or LENS[s] (paged-v)
  const float *table;            // paged: [B x mbps] physical block ids
  uint32_t bs, mbps;
  uint32_t nsink, win;           // ring
  const float *ent;              // entries: [ne x 2] (base, crel)
  uint32_t ne, qcrel;
  const float *co, *si;          // RoPE tables [rows x hd/2] (ring, entries)
  uint64_t kv_words, table_words, rope_words;
};

// Keys of sequence s (count), and for key j: the float offset of its K/V row
// (UINT64_MAX: skip) and its cache-relative position (rotated modes).
template <int MODE>
__device__ __forceinline__ uint32_t key_count(const GatherGeom &g, uint32_t s) {
  if (MODE == kModePaged) return f2u(__ldg(g.pos)) + 1u;
  if (MODE == kModePagedV) return f2u(__ldg(g.pos + s)) + 1u;
  if (MODE == kModeRing) {
    const uint32_t cap = g.nsink + g.win;
    return min(f2u(__ldg(g.pos)) + 1u, cap);
  }
  return g.ne;
}
template <int MODE>
__device__ __forceinline__ uint64_t key_row(const GatherGeom &g, uint32_t s, uint32_t j,
                                            uint32_t kvh, uint32_t *crel) {
  uint64_t row;
  if (MODE == kModePaged || MODE == kModePagedV) {
    const uint64_t ti = (uint64_t)s * g.mbps + j / g.bs;
    if (j / g.bs >= g.mbps || ti >= g.table_words) return UINT64_MAX;
    const uint32_t phys = f2u(__ldg(g.table + ti));
    row = ((uint64_t)phys * g.bs + j % g.bs) * g.kvdim;
  } else if (MODE == kModeRing) {
    const uint32_t pos = f2u(__ldg(g.pos)), cap = g.nsink + g.win;
    const uint32_t start = pos >= cap ? pos - g.win + 1u : g.nsink;
    const uint32_t woff = (start - g.nsink) % g.win;
    const uint32_t slot = j < g.nsink ? j : g.nsink + (woff + (j - g.nsink)) % g.win;
    row = (uint64_t)slot * g.kvdim;
    *crel = j;
  } else {
    if (2ull * j + 1 >= 2ull * g.ne) return UINT64_MAX;
    row = f2u(__ldg(g.ent + 2 * j));
    *crel = f2u(__ldg(g.ent + 2 * j + 1));
  }
  row += (uint64_t)kvh * g.hd;
  if (row + g.hd > g.kv_words) return UINT64_MAX;
  if ((MODE == kModeRing || MODE == kModeEnt) &&
      ((uint64_t)*crel + 1) * (g.hd / 2) > g.rope_words)
    return UINT64_MAX;
  return row;
}

// Rotate adjacent pairs (2m, 2m+1) of this lane's DPL dims by table row CREL.
template <int DPL>
__device__ __forceinline__ void rot_pairs(float (&v)[DPL], const GatherGeom &g, uint32_t crel,
                                          int lane) {
  const uint32_t half = g.hd / 2;
#pragma unroll
  for (int d = 0; d < DPL; d += 2) {
    const uint32_t m = (uint32_t)(lane * DPL + d) / 2u;
    const float cc = __ldg(g.co + (uint64_t)crel * half + m);
    const float ss = __ldg(g.si + (uint64_t)crel * half + m);
    const float a0 = v[d], a1 = v[d + 1];
    v[d] = a0 * cc - a1 * ss;
    v[d + 1] = a0 * ss + a1 * cc;
  }
}

constexpr int kGWarps = 4, kGMaxGrp = 8;

template <int HD, int MODE>
__global__ void __launch_bounds__(kGWarps * 32)
gather_attn_partial(const float *__restrict__ Q, const float *__restrict__ CK,
                    const float *__restrict__ CV, GatherGeom g, float *__restrict__ part) {
  constexpr int DPL = HD / 32;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint32_t split = blockIdx.x, skv = blockIdx.y;
  const uint32_t s = skv / g.kvheads, kvh = skv % g.kvheads, grp = g.grp;
  __shared__ float s_m[kGWarps][kGMaxGrp], s_l[kGWarps][kGMaxGrp];
  __shared__ float s_o[kGWarps][kGMaxGrp][HD];
  const uint32_t len = key_count<MODE>(g, s);
  const uint32_t p0 = split * g.chunk, p1 = min(p0 + g.chunk, len);
  const bool rope = MODE == kModeRing || MODE == kModeEnt;
  uint32_t qcrel = 0;
  if (MODE == kModeRing) qcrel = min(f2u(__ldg(g.pos)), g.nsink + g.win - 1u);
  if (MODE == kModeEnt) qcrel = g.qcrel;
  float q[kGMaxGrp][DPL], m[kGMaxGrp], l[kGMaxGrp], o[kGMaxGrp][DPL];
#pragma unroll
  for (int hh = 0; hh < kGMaxGrp; hh++) {
    m[hh] = -INFINITY;
    l[hh] = 0.0f;
#pragma unroll
    for (int d = 0; d < DPL; d++) {
      o[hh][d] = 0.0f;
      q[hh][d] = (uint32_t)hh < grp
                     ? __ldg(Q + (uint64_t)s * g.dim + (uint64_t)(kvh * grp + hh) * HD +
                             lane * DPL + d)
                     : 0.0f;
    }
    if (rope && (uint32_t)hh < grp) rot_pairs<DPL>(q[hh], g, qcrel, lane);
  }
  for (uint32_t j = p0 + warp; j < p1; j += kGWarps) {
    uint32_t crel = 0;
    const uint64_t row = key_row<MODE>(g, s, j, kvh, &crel);
    if (row == UINT64_MAX) continue;                 // warp-uniform
    float kr[DPL], vr[DPL];
#pragma unroll
    for (int d = 0; d < DPL; d++) {
      kr[d] = __ldg(CK + row + lane * DPL + d);
      vr[d] = __ldg(CV + row + lane * DPL + d);
    }
    if (rope) rot_pairs<DPL>(kr, g, crel, lane);
#pragma unroll
    for (int hh = 0; hh < kGMaxGrp; hh++) {
      if ((uint32_t)hh >= grp) break;
      float dot = 0.0f;
#pragma unroll
      for (int d = 0; d < DPL; d++) dot = fmaf(q[hh][d], kr[d], dot);
      for (int off = 16; off > 0; off >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, off);
      const float sc = dot * g.coef;
      const float mn = fmaxf(m[hh], sc);
      const float corr = expf(m[hh] - mn);
      const float p = expf(sc - mn);
      l[hh] = l[hh] * corr + p;
#pragma unroll
      for (int d = 0; d < DPL; d++) o[hh][d] = fmaf(p, vr[d], o[hh][d] * corr);
      m[hh] = mn;
    }
  }
#pragma unroll
  for (int hh = 0; hh < kGMaxGrp; hh++) {
    if ((uint32_t)hh >= grp) break;
    if (lane == 0) { s_m[warp][hh] = m[hh]; s_l[warp][hh] = l[hh]; }
#pragma unroll
    for (int d = 0; d < DPL; d++) s_o[warp][hh][lane * DPL + d] = o[hh][d];
  }
  __syncthreads();
  for (uint32_t e = threadIdx.x; e < grp * HD; e += blockDim.x) {
    const uint32_t hh = e / HD, d = e % HD;
    float mm = -INFINITY;
    for (int w = 0; w < kGWarps; w++) mm = fmaxf(mm, s_m[w][hh]);
    float ll = 0.0f, oo = 0.0f;
    if (mm > -INFINITY) {
      for (int w = 0; w < kGWarps; w++) {
        const float c = expf(s_m[w][hh] - mm);
        ll += s_l[w][hh] * c;
        oo += s_o[w][hh][d] * c;
      }
    }
    const uint32_t h = kvh * grp + hh;
    float *pp = part + (((uint64_t)s * g.heads + h) * g.nsplit + split) * (HD + 2);
    pp[2 + d] = oo;
    if (d == 0) { pp[0] = mm; pp[1] = ll; }
  }
}

// Merge the splits of (sequence, head) into C (outputs past LIMIT untouched).
template <int HD>
__global__ void gather_attn_combine(const float *__restrict__ part, GatherGeom g,
                                    float *__restrict__ C, uint64_t limit) {
  const uint32_t sh = blockIdx.x, s = sh / g.heads, h = sh % g.heads;
  const float *pp = part + (uint64_t)sh * g.nsplit * (HD + 2);
  float mm = -INFINITY;
  for (uint32_t k = 0; k < g.nsplit; k++) mm = fmaxf(mm, pp[(uint64_t)k * (HD + 2)]);
  for (uint32_t d = threadIdx.x; d < HD; d += blockDim.x) {
    float ll = 0.0f, oo = 0.0f;
    for (uint32_t k = 0; k < g.nsplit; k++) {
      const float *ps = pp + (uint64_t)k * (HD + 2);
      if (ps[0] > -INFINITY) {
        const float c = expf(ps[0] - mm);
        ll += ps[1] * c;
        oo += ps[2 + d] * c;
      }
    }
    const uint64_t idx = (uint64_t)s * g.dim + (uint64_t)h * HD + d;
    if (idx < limit) C[idx] = ll > 0.0f ? oo / ll : 0.0f;
  }
}

// Head sizes the split kernel does not cover: one thread per output, the
// reference's two passes (max, then normaliser and context).
template <int MODE>
__global__ void gather_attn_simple(const float *__restrict__ Q, const float *__restrict__ CK,
                                   const float *__restrict__ CV, GatherGeom g,
                                   float *__restrict__ C, uint64_t limit) {
  const uint64_t idx = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (uint64_t)g.B * g.dim || idx >= limit) return;
  const uint32_t s = (uint32_t)(idx / g.dim), c = (uint32_t)(idx % g.dim);
  const uint32_t h = c / g.hd, t = c % g.hd, kvh = h / g.grp, half = g.hd / 2;
  const bool rope = MODE == kModeRing || MODE == kModeEnt;
  uint32_t qcrel = MODE == kModeEnt ? g.qcrel : 0;
  if (MODE == kModeRing) qcrel = min(f2u(__ldg(g.pos)), g.nsink + g.win - 1u);
  const float *q = Q + (uint64_t)s * g.dim + (uint64_t)h * g.hd;
  const uint32_t len = key_count<MODE>(g, s);
  auto score = [&](uint64_t row, uint32_t crel) {
    float acc = 0.0f;
    if (rope) {
      for (uint32_t mm = 0; mm < half; mm++) {
        const float cc = g.co[(uint64_t)crel * half + mm], ss = g.si[(uint64_t)crel * half + mm];
        const float k0 = CK[row + 2 * mm], k1 = CK[row + 2 * mm + 1];
        const float qc = g.co[(uint64_t)qcrel * half + mm], qs = g.si[(uint64_t)qcrel * half + mm];
        const float q0 = q[2 * mm], q1 = q[2 * mm + 1];
        acc += (q0 * qc - q1 * qs) * (k0 * cc - k1 * ss) + (q0 * qs + q1 * qc) * (k0 * ss + k1 * cc);
      }
    } else {
      for (uint32_t tt = 0; tt < g.hd; tt++) acc = fmaf(q[tt], CK[row + tt], acc);
    }
    return acc * g.coef;
  };
  float mx = -1.0e30f;
  for (uint32_t j = 0; j < len; j++) {
    uint32_t crel = 0;
    const uint64_t row = key_row<MODE>(g, s, j, kvh, &crel);
    if (row != UINT64_MAX) mx = fmaxf(mx, score(row, crel));
  }
  float z = 0.0f, ctx = 0.0f;
  for (uint32_t j = 0; j < len; j++) {
    uint32_t crel = 0;
    const uint64_t row = key_row<MODE>(g, s, j, kvh, &crel);
    if (row == UINT64_MAX) continue;
    const float e = expf(score(row, crel) - mx);
    z += e;
    ctx = fmaf(e, CV[row + t], ctx);
  }
  C[idx] = z > 0.0f ? ctx / z : 0.0f;
}

// ---- the simple operators -------------------------------------------------------
__global__ void k_append_ring(const float *SRC, const float *POS, float *CACHE, uint32_t kvdim,
                              uint32_t nsink, uint32_t win, uint64_t limit, uint64_t cache_words) {
  const uint32_t idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= kvdim || idx >= limit) return;
  const uint32_t pos = f2u(__ldg(POS));
  const uint32_t slot = pos < nsink ? pos : nsink + (pos - nsink) % win;
  const uint64_t o = (uint64_t)slot * kvdim + idx;
  if (o < cache_words) CACHE[o] = SRC[idx];
}
__global__ void k_qkv_append(const float *QKV, float *CK, float *CV, uint32_t dim, uint32_t kvdim,
                             uint32_t wbase, uint64_t limit) {
  const uint32_t idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= kvdim || idx >= limit) return;
  CK[(uint64_t)wbase + idx] = QKV[(uint64_t)dim + idx];
  CV[(uint64_t)wbase + idx] = QKV[(uint64_t)dim + kvdim + idx];
}
// LENS == nullptr: every row at POS[0].
__global__ void k_append_paged(const float *SRC, const float *POS, const float *LENS,
                               const float *TABLE, float *POOL, uint32_t B, uint32_t kvdim,
                               uint32_t bs, uint32_t mbps, uint64_t limit, uint64_t table_words,
                               uint64_t pool_words) {
  const uint64_t idx = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (uint64_t)B * kvdim || idx >= limit) return;
  const uint32_t s = (uint32_t)(idx / kvdim), t = (uint32_t)(idx % kvdim);
  const uint32_t pos = f2u(__ldg(LENS ? LENS + s : POS));
  const uint64_t ti = (uint64_t)s * mbps + pos / bs;
  if (pos / bs >= mbps || ti >= table_words) return;
  const uint32_t phys = f2u(__ldg(TABLE + ti));
  const uint64_t o = ((uint64_t)phys * bs + pos % bs) * kvdim + t;
  if (o < pool_words) POOL[o] = SRC[idx];
}
__global__ void k_block_copy(float *POOL, uint64_t bn, uint32_t src, uint32_t dst, uint64_t limit) {
  const uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= bn || i >= limit) return;
  POOL[(uint64_t)dst * bn + i] = POOL[(uint64_t)src * bn + i];
}
// Adjacent-pair RoPE of row b at its own length LENS[b]; SI scaled by SG[0].
__global__ void k_rope_b_v(const float *X, const float *CO, const float *SI, const float *SG,
                           const float *LENS, float *C, uint32_t B, uint32_t cols,
                           uint32_t heads, uint64_t limit, uint64_t rope_words) {
  const uint32_t hd = cols / heads, half = hd / 2, rh = heads * half;
  const uint64_t idx = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (uint64_t)B * rh || idx >= limit) return;
  const uint32_t bb = (uint32_t)(idx / rh), rem = (uint32_t)(idx % rh);
  const uint32_t m = rem % half, h = rem / half;
  const uint64_t ci = (uint64_t)f2u(__ldg(LENS + bb)) * half + m;
  if (ci >= rope_words) return;
  const float cc = CO[ci], ss = SI[ci] * SG[0];
  const uint64_t i0 = (uint64_t)bb * cols + (uint64_t)h * hd + 2 * m;
  const float a0 = X[i0], a1 = X[i0 + 1];
  C[i0] = a0 * cc - a1 * ss;
  C[i0 + 1] = a0 * ss + a1 * cc;
}

// ---- geometry, checks and launches ----------------------------------------------
uint32_t max_keys(int mode, const OpArgs &a, uint32_t B) {
  switch (mode) {
    case kModePaged:
    case kModePagedV: return a.push[5] * a.push[4];   // mbps * bs
    case kModeRing: return a.push[3] + a.push[4];      // nsink + win
    default: return a.push[3];                         // ne
  }
  (void)B;
}

template <int MODE>
GatherGeom gather_geom(const OpArgs &a) {
  GatherGeom g = {};
  const bool paged = MODE == kModePaged || MODE == kModePagedV;
  g.B = paged ? a.push[0] : 1;
  g.dim = a.push[paged ? 1 : 0];
  g.heads = a.push[paged ? 2 : 1];
  g.kvheads = a.push[paged ? 3 : 2];
  g.hd = g.heads ? g.dim / g.heads : 0;
  g.grp = g.kvheads ? g.heads / g.kvheads : 0;
  g.kvdim = g.kvheads * g.hd;
  g.coef = g.hd ? 1.0f / sqrtf((float)g.hd) : 0.0f;
  g.kv_words = a.words[1] < a.words[2] ? a.words[1] : a.words[2];
  if (paged) {
    g.bs = a.push[4];
    g.mbps = a.push[5];
    g.pos = (const float *)a.buf[3];
    g.table = (const float *)a.buf[4];
    g.table_words = a.words[4];
  } else if (MODE == kModeRing) {
    g.nsink = a.push[3];
    g.win = a.push[4];
    g.pos = (const float *)a.buf[3];
    g.co = (const float *)a.buf[4];
    g.si = (const float *)a.buf[5];
  } else {
    g.ne = a.push[3];
    g.qcrel = a.push[4];
    g.ent = (const float *)a.buf[3];
    g.co = (const float *)a.buf[4];
    g.si = (const float *)a.buf[5];
  }
  if (!paged) g.rope_words = a.words[4] < a.words[5] ? a.words[4] : a.words[5];
  const uint32_t units = g.B * g.kvheads;
  const uint32_t keys = max_keys(MODE, a, g.B);
  uint32_t want = units ? (uint32_t)ceil_div(4 * 148, (int)units) : 1;
  if (want < 1) want = 1;
  uint32_t chunk = keys ? (keys + want - 1) / want : 1;
  if (chunk < 32) chunk = 32;
  g.chunk = chunk;
  g.nsplit = keys ? (keys + chunk - 1) / chunk : 1;
  if (g.nsplit == 0) g.nsplit = 1;
  return g;
}

bool split_ok(const GatherGeom &g) {
  return (g.hd == 64 || g.hd == 128) && g.grp >= 1 && g.grp <= (uint32_t)kGMaxGrp &&
         g.heads == g.kvheads * g.grp;
}

template <int MODE>
const char *chk_gather(const OpArgs &a) {
  const GatherGeom g = gather_geom<MODE>(a);
  const bool paged = MODE == kModePaged || MODE == kModePagedV;
  if (g.heads == 0 || g.kvheads == 0 || g.dim % g.heads || g.heads % g.kvheads)
    return fmt_msg("attention: dim %u, heads %u, kvheads %u do not divide", g.dim, g.heads,
                   g.kvheads);
  if (!paged && g.hd % 2) return fmt_msg("attention: head size %u is odd (RoPE pairs)", g.hd);
  if (paged && g.bs == 0) return "attention: block size 0";
  if (MODE == kModeRing && g.win == 0) return "decode-attn-stream: window 0";
  const char *m;
  if ((m = need_words(a, 0, (uint64_t)g.B * g.dim, "Q"))) return m;
  const uint32_t out = paged ? 5 : 6;
  if ((m = need_words(a, out, (uint64_t)g.B * g.dim, "C"))) return m;
  if (MODE == kModePaged || MODE == kModeRing)
    if ((m = need_words(a, 3, 1, "POS"))) return m;
  if (MODE == kModePagedV && (m = need_words(a, 3, g.B, "LENS"))) return m;
  if (MODE == kModeEnt && (m = need_words(a, 3, 2ull * g.ne, "ENT"))) return m;
  if (MODE == kModeEnt &&
      ((m = need_words(a, 4, ((uint64_t)g.qcrel + 1) * (g.hd / 2), "CO")) ||
       (m = need_words(a, 5, ((uint64_t)g.qcrel + 1) * (g.hd / 2), "SI"))))
    return m;
  if (MODE == kModeRing &&
      ((m = need_words(a, 4, (uint64_t)(g.nsink + g.win) * (g.hd / 2), "CO")) ||
       (m = need_words(a, 5, (uint64_t)(g.nsink + g.win) * (g.hd / 2), "SI"))))
    return m;
  return nullptr;
}

template <int MODE>
size_t scr_gather(const OpArgs &a) {
  const GatherGeom g = gather_geom<MODE>(a);
  if (!split_ok(g)) return 0;
  return (size_t)g.B * g.heads * g.nsplit * (g.hd + 2) * sizeof(float);
}

template <int MODE>
cudaError_t run_gather(const OpArgs &a) {
  const GatherGeom g = gather_geom<MODE>(a);
  const bool paged = MODE == kModePaged || MODE == kModePagedV;
  const float *Q = (const float *)a.buf[0], *CK = (const float *)a.buf[1],
              *CV = (const float *)a.buf[2];
  float *C = (float *)a.buf[paged ? 5 : 6];
  const uint64_t limit = invocations(a.groups, 64);
  if (g.B == 0 || g.dim == 0) return cudaSuccess;
  if (!split_ok(g) || !a.scratch) {
    const uint64_t n = (uint64_t)g.B * g.dim;
    gather_attn_simple<MODE><<<(unsigned)ceil_div64(n, 128), 128, 0, a.stream>>>(Q, CK, CV, g, C,
                                                                                  limit);
    count_launches(1);
    return cudaPeekAtLastError();
  }
  float *part = (float *)a.scratch;
  const dim3 grid(g.nsplit, g.B * g.kvheads);
  if (g.hd == 128) {
    gather_attn_partial<128, MODE><<<grid, kGWarps * 32, 0, a.stream>>>(Q, CK, CV, g, part);
    gather_attn_combine<128><<<g.B * g.heads, 128, 0, a.stream>>>(part, g, C, limit);
  } else {
    gather_attn_partial<64, MODE><<<grid, kGWarps * 32, 0, a.stream>>>(Q, CK, CV, g, part);
    gather_attn_combine<64><<<g.B * g.heads, 64, 0, a.stream>>>(part, g, C, limit);
  }
  count_launches(2);
  return cudaPeekAtLastError();
}

size_t no_scr(const OpArgs &) { return 0; }

// cache-append-ring: SRC POS CACHE; kvdim nsink win
const char *chk_ring(const OpArgs &a) {
  if (a.push[2] == 0) return "cache-append-ring: window 0";
  const char *m;
  if ((m = need_words(a, 0, a.push[0], "SRC"))) return m;
  if ((m = need_words(a, 1, 1, "POS"))) return m;
  return need_words(a, 2, (uint64_t)(a.push[1] + a.push[2]) * a.push[0], "CACHE");
}
cudaError_t run_ring(const OpArgs &a) {
  const uint32_t kvdim = a.push[0];
  if (!kvdim) return cudaSuccess;
  k_append_ring<<<ceil_div((int)kvdim, 128), 128, 0, a.stream>>>(
      (const float *)a.buf[0], (const float *)a.buf[1], (float *)a.buf[2], kvdim, a.push[1],
      a.push[2], invocations(a.groups, 64), a.words[2]);
  count_launches(1);
  return cudaPeekAtLastError();
}
// qkv-append: QKV CK CV; dim kvdim wbase
const char *chk_qkv_append(const OpArgs &a) {
  const uint64_t dim = a.push[0], kvdim = a.push[1], wbase = a.push[2];
  const char *m;
  if ((m = need_words(a, 0, dim + 2 * kvdim, "QKV"))) return m;
  if ((m = need_words(a, 1, wbase + kvdim, "CK"))) return m;
  return need_words(a, 2, wbase + kvdim, "CV");
}
cudaError_t run_qkv_append(const OpArgs &a) {
  if (!a.push[1]) return cudaSuccess;
  k_qkv_append<<<ceil_div((int)a.push[1], 128), 128, 0, a.stream>>>(
      (const float *)a.buf[0], (float *)a.buf[1], (float *)a.buf[2], a.push[0], a.push[1],
      a.push[2], invocations(a.groups, 64));
  count_launches(1);
  return cudaPeekAtLastError();
}
// cache-append-paged(-v): SRC POS|LENS TABLE POOL; B kvdim bs mbps
template <bool VAR>
const char *chk_append_paged(const OpArgs &a) {
  const uint64_t B = a.push[0], kvdim = a.push[1];
  if (a.push[2] == 0) return "cache-append-paged: block size 0";
  const char *m;
  if ((m = need_words(a, 0, B * kvdim, "SRC"))) return m;
  if ((m = need_words(a, 1, VAR ? B : 1, VAR ? "LENS" : "POS"))) return m;
  return need_words(a, 2, B * a.push[3], "TABLE");
}
template <bool VAR>
cudaError_t run_append_paged(const OpArgs &a) {
  const uint64_t n = (uint64_t)a.push[0] * a.push[1];
  if (!n) return cudaSuccess;
  k_append_paged<<<(unsigned)ceil_div64(n, 128), 128, 0, a.stream>>>(
      (const float *)a.buf[0], VAR ? nullptr : (const float *)a.buf[1],
      VAR ? (const float *)a.buf[1] : nullptr, (const float *)a.buf[2], (float *)a.buf[3],
      a.push[0], a.push[1], a.push[2], a.push[3], invocations(a.groups, 64), a.words[2],
      a.words[3]);
  count_launches(1);
  return cudaPeekAtLastError();
}
// block-copy: POOL; bs kvdim src dst
const char *chk_block_copy(const OpArgs &a) {
  const uint64_t bn = (uint64_t)a.push[0] * a.push[1];
  const uint64_t top = (uint64_t)(a.push[2] > a.push[3] ? a.push[2] : a.push[3]) + 1;
  return need_words(a, 0, bn * top, "POOL");
}
cudaError_t run_block_copy(const OpArgs &a) {
  const uint64_t bn = (uint64_t)a.push[0] * a.push[1];
  if (!bn || a.push[2] == a.push[3]) return cudaSuccess;
  k_block_copy<<<(unsigned)ceil_div64(bn, 256), 256, 0, a.stream>>>(
      (float *)a.buf[0], bn, a.push[2], a.push[3], invocations(a.groups, 64));
  count_launches(1);
  return cudaPeekAtLastError();
}
// decode-rope-b-v: X CO SI SG LENS C; B cols heads
const char *chk_rope_b_v(const OpArgs &a) {
  const uint64_t B = a.push[0], cols = a.push[1], heads = a.push[2];
  if (heads == 0 || cols % heads || (cols / heads) % 2)
    return fmt_msg("decode-rope-b-v: cols %u, heads %u (even head size)", a.push[1], a.push[2]);
  const char *m;
  if ((m = need_words(a, 0, B * cols, "X"))) return m;
  if ((m = need_words(a, 3, 1, "SG"))) return m;
  if ((m = need_words(a, 4, B, "LENS"))) return m;
  return need_words(a, 5, B * cols, "C");
}
cudaError_t run_rope_b_v(const OpArgs &a) {
  const uint32_t B = a.push[0], cols = a.push[1], heads = a.push[2];
  const uint64_t n = (uint64_t)B * heads * (cols / heads / 2);
  if (!n) return cudaSuccess;
  const uint64_t rw = a.words[1] < a.words[2] ? a.words[1] : a.words[2];
  k_rope_b_v<<<(unsigned)ceil_div64(n, 128), 128, 0, a.stream>>>(
      (const float *)a.buf[0], (const float *)a.buf[1], (const float *)a.buf[2],
      (const float *)a.buf[3], (const float *)a.buf[4], (float *)a.buf[5], B, cols, heads,
      invocations(a.groups, 64), rw);
  count_launches(1);
  return cudaPeekAtLastError();
}

}  // namespace

const OpSpec kKvOps[] = {
    {"cache-append-ring", 3, 3, chk_ring, no_scr, run_ring},
    {"decode-attn-stream", 7, 5, chk_gather<kModeRing>, scr_gather<kModeRing>,
     run_gather<kModeRing>},
    {"qkv-append", 3, 3, chk_qkv_append, no_scr, run_qkv_append},
    {"attn-stream-entries", 7, 5, chk_gather<kModeEnt>, scr_gather<kModeEnt>,
     run_gather<kModeEnt>},
    {"cache-append-paged", 4, 4, chk_append_paged<false>, no_scr, run_append_paged<false>},
    {"decode-attn-paged", 6, 6, chk_gather<kModePaged>, scr_gather<kModePaged>,
     run_gather<kModePaged>},
    {"block-copy", 1, 4, chk_block_copy, no_scr, run_block_copy},
    {"decode-rope-b-v", 6, 3, chk_rope_b_v, no_scr, run_rope_b_v},
    {"cache-append-paged-v", 4, 4, chk_append_paged<true>, no_scr, run_append_paged<true>},
    {"decode-attn-paged-v", 6, 6, chk_gather<kModePagedV>, scr_gather<kModePagedV>,
     run_gather<kModePagedV>},
};
const int kKvOpsCount = sizeof(kKvOps) / sizeof(kKvOps[0]);

}  // namespace nl

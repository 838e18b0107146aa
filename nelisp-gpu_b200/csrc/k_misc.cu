// k_misc.cu -- the remaining operators of the decode / prefill path and its
// backward, for sm_100a.
//
// Reference operators (lisp/nelisp-gpu-kernels.el):
//   causal-mask     :148-155    S[i, j] = -1e30 for j > i (in place)
//   attn-scores     :208-221    S[h, i, j] = <q_i^h, k_j^kvh> / sqrt(hd), -1e30 past i
//   attn-context    :224-235    C[i, h*hd+t] = sum_j P[h, i, j] V[j, kvh*hd+t]
//   attn-sc-dq/-dk, attn-ctx-dp/-dv :237-290  their gradients
//   dp4a-dot        :592-602    OUT[i] = sdot4x8(A, B), the words rebuilt from two
//                               f32 halves (lo + hi * 65536)
//   bitlinear-dp4a  :606-620    Y = BIAS[o] + (BETA[0] GAMMA[s]) float(sum sdot)
//   dp4a-rows-t     :792-810    X[p, i] = sum_o sv(o, i) (BETA[o] G[p, o]),
//                               sv the sign-extended int8 lane of a bitcast word
//   rmsnorm-heads   :828-845    per (position, head): x * rsqrt(mean x^2 + 1e-6) * G
//   rope-apply      :1290-1303  adjacent-pair RoPE at the row's position, SG sign
//   silu            :1306-1312  x * sigmoid(x)
//   scale-rows      :1365-1372  C[r, j] = Y[r, j] S[r]
// Integer sums are exact (int32) like the reference's; f32 sums keep the
// reference's order where one thread owns an output.  attn-scores and
// attn-context stage tiles in shared memory (a head's scores are a small
// GEMM); the others are bandwidth-bound streams.

#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include "nl_internal.h"

namespace nl {
namespace {

__device__ __forceinline__ uint32_t f2u(float v) { return v > 0.0f ? __float2uint_rz(v) : 0u; }

size_t no_scr(const OpArgs &) { return 0; }
unsigned blocks_for(uint64_t n, unsigned t = 256) { return grid_for(n, t, 148u * 64u); }

// ---- causal-mask ------------------------------------------------------------------
__global__ void k_causal_mask(float *S, uint32_t n, uint64_t limit) {
  const uint64_t total = (uint64_t)n * n;
  for (uint64_t idx = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total && idx < limit;
       idx += (uint64_t)gridDim.x * blockDim.x)
    if (idx % n > idx / n) S[idx] = -1.0e30f;
}
const char *chk_causal_mask(const OpArgs &a) {
  return need_words(a, 0, (uint64_t)a.push[0] * a.push[0], "S");
}
cudaError_t run_causal_mask(const OpArgs &a) {
  const uint64_t n2 = (uint64_t)a.push[0] * a.push[0];
  if (!n2) return cudaSuccess;
  k_causal_mask<<<blocks_for(n2), 256, 0, a.stream>>>((float *)a.buf[0], a.push[0],
                                                      invocations(a.groups, 64));
  count_launches(1);
  return cudaPeekAtLastError();
}

// ---- attn-scores: per head a [seq x seq] tile product, 32 x 32 per CTA --------------
constexpr int kSc = 32, kScK = 32;
// CAUSAL: attn-scores (scaled by 1/sqrt(hd), -1e30 above the diagonal);
// otherwise attn-ctx-dp (DP[h,i,j] = sum_t DC[i,h,t] V[j,kvh,t], every (i, j)).
template <bool CAUSAL = true>
__global__ void __launch_bounds__(256)
k_attn_scores(const float *__restrict__ Q, const float *__restrict__ K, float *__restrict__ S,
              uint32_t seq, uint32_t dim, uint32_t heads, uint32_t kvheads, uint64_t limit) {
  __shared__ float Qs[kSc][kScK + 1], Ks[kSc][kScK + 1];
  const uint32_t hd = dim / heads, kvh = blockIdx.z / (heads / kvheads), kvdim = kvheads * hd;
  const uint32_t h = blockIdx.z, i0 = blockIdx.y * kSc, j0 = blockIdx.x * kSc;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;   // 8 row groups of 4
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  const bool live = !CAUSAL || j0 <= i0 + kSc - 1;          // a tile above the diagonal is all masked
  if (live) {
    for (uint32_t t0 = 0; t0 < hd; t0 += kScK) {
      for (int e = threadIdx.x; e < kSc * kScK; e += 256) {
        const int r = e / kScK, c = e % kScK;
        const uint32_t i = i0 + r, j = j0 + r, t = t0 + c;
        Qs[r][c] = (i < seq && t < hd) ? Q[(uint64_t)i * dim + (uint64_t)h * hd + t] : 0.0f;
        Ks[r][c] = (j < seq && t < hd) ? K[(uint64_t)j * kvdim + (uint64_t)kvh * hd + t] : 0.0f;
      }
      __syncthreads();
#pragma unroll 8
      for (int c = 0; c < kScK; c++) {
        const float kv = Ks[tx][c];
#pragma unroll
        for (int a = 0; a < 4; a++) acc[a] = fmaf(Qs[ty * 4 + a][c], kv, acc[a]);
      }
      __syncthreads();
    }
  }
  const float scale = 1.0f / sqrtf((float)hd);
#pragma unroll
  for (int a = 0; a < 4; a++) {
    const uint32_t i = i0 + ty * 4 + a, j = j0 + tx;
    if (i >= seq || j >= seq) continue;
    const uint64_t idx = (uint64_t)h * seq * seq + (uint64_t)i * seq + j;
    if (idx >= limit) continue;
    S[idx] = CAUSAL ? (j > i ? -1.0e30f : acc[a] * scale) : acc[a];
  }
}
const char *chk_scores(const OpArgs &a) {
  const uint64_t seq = a.push[0], dim = a.push[1], heads = a.push[2], kvheads = a.push[3];
  if (!heads || !kvheads || dim % heads || heads % kvheads)
    return fmt_msg("attention: dim %u, heads %u, kvheads %u do not divide", a.push[1], a.push[2],
                   a.push[3]);
  const char *m;
  if ((m = need_words(a, 0, seq * dim, "Q"))) return m;
  if ((m = need_words(a, 1, seq * kvheads * (dim / heads), "K"))) return m;
  return need_words(a, 2, heads * seq * seq, "S");
}
cudaError_t run_scores(const OpArgs &a) {
  const uint32_t seq = a.push[0];
  if (!seq) return cudaSuccess;
  const dim3 grid((seq + kSc - 1) / kSc, (seq + kSc - 1) / kSc, a.push[2]);
  k_attn_scores<true><<<grid, 256, 0, a.stream>>>((const float *)a.buf[0], (const float *)a.buf[1],
                                           (float *)a.buf[2], seq, a.push[1], a.push[2],
                                           a.push[3], invocations(a.groups, 64));
  count_launches(1);
  return cudaPeekAtLastError();
}

// ---- attn-context: per head C_h = P_h [seq x seq] V_kvh [seq x hd] --------------------
// SCALED: attn-sc-dq (DQ = (sum_j DS[h,i,j] K[j,kvh,t]) / sqrt(hd)); else
// attn-context.
template <bool SCALED = false>
__global__ void __launch_bounds__(256)
k_attn_context(const float *__restrict__ P, const float *__restrict__ V, float *__restrict__ C,
               uint32_t seq, uint32_t dim, uint32_t heads, uint32_t kvheads, uint64_t limit) {
  __shared__ float Ps[kSc][kScK + 1], Vs[kScK][kSc + 1];
  const uint32_t hd = dim / heads, h = blockIdx.z, kvh = h / (heads / kvheads);
  const uint32_t kvdim = kvheads * hd, i0 = blockIdx.y * kSc, t0 = blockIdx.x * kSc;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  const float *Ph = P + (uint64_t)h * seq * seq;
  for (uint32_t j0 = 0; j0 < seq; j0 += kScK) {
    for (int e = threadIdx.x; e < kSc * kScK; e += 256) {
      const int r = e / kScK, c = e % kScK;
      const uint32_t i = i0 + r, j = j0 + c;
      Ps[r][c] = (i < seq && j < seq) ? Ph[(uint64_t)i * seq + j] : 0.0f;
      const uint32_t jv = j0 + r, t = t0 + c;
      Vs[r][c] = (jv < seq && t < hd) ? V[(uint64_t)jv * kvdim + (uint64_t)kvh * hd + t] : 0.0f;
    }
    __syncthreads();
#pragma unroll 8
    for (int c = 0; c < kScK; c++) {
      const float vv = Vs[c][tx];
#pragma unroll
      for (int a = 0; a < 4; a++) acc[a] = fmaf(Ps[ty * 4 + a][c], vv, acc[a]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int a = 0; a < 4; a++) {
    const uint32_t i = i0 + ty * 4 + a, t = t0 + tx;
    if (i >= seq || t >= hd) continue;
    const uint64_t idx = (uint64_t)i * dim + (uint64_t)h * hd + t;
    if (idx < limit) C[idx] = SCALED ? acc[a] * (1.0f / sqrtf((float)hd)) : acc[a];
  }
}
const char *chk_context(const OpArgs &a) {
  const uint64_t seq = a.push[0], dim = a.push[1], heads = a.push[2], kvheads = a.push[3];
  if (!heads || !kvheads || dim % heads || heads % kvheads)
    return fmt_msg("attention: dim %u, heads %u, kvheads %u do not divide", a.push[1], a.push[2],
                   a.push[3]);
  const char *m;
  if ((m = need_words(a, 0, heads * seq * seq, "P"))) return m;
  if ((m = need_words(a, 1, seq * kvheads * (dim / heads), "V"))) return m;
  return need_words(a, 2, seq * dim, "C");
}
cudaError_t run_context(const OpArgs &a) {
  const uint32_t seq = a.push[0], hd = a.push[2] ? a.push[1] / a.push[2] : 0;
  if (!seq || !hd) return cudaSuccess;
  const dim3 grid((hd + kSc - 1) / kSc, (seq + kSc - 1) / kSc, a.push[2]);
  k_attn_context<false><<<grid, 256, 0, a.stream>>>((const float *)a.buf[0], (const float *)a.buf[1],
                                            (float *)a.buf[2], seq, a.push[1], a.push[2],
                                            a.push[3], invocations(a.groups, 64));
  count_launches(1);
  return cudaPeekAtLastError();
}

// ---- attention backward (kernels.el:237-290) ------------------------------------
// attn-sc-dq (DS K DQ) and attn-ctx-dp (DC V DP) are the tiled products above;
// attn-sc-dk (DS Q DK) and attn-ctx-dv (DC P DV) sum over the query rows i and
// the heads of a kv group, one thread per output as the reference does.
const char *chk_dq(const OpArgs &a) {
  const uint64_t seq = a.push[0], dim = a.push[1], heads = a.push[2], kvheads = a.push[3];
  if (!heads || !kvheads || dim % heads || heads % kvheads)
    return fmt_msg("attention: dim %u, heads %u, kvheads %u do not divide", a.push[1], a.push[2],
                   a.push[3]);
  const char *m;
  if ((m = need_words(a, 0, heads * seq * seq, "DS"))) return m;
  if ((m = need_words(a, 1, seq * kvheads * (dim / heads), "K"))) return m;
  return need_words(a, 2, seq * dim, "DQ");
}
cudaError_t run_dq(const OpArgs &a) {
  const uint32_t seq = a.push[0], hd = a.push[2] ? a.push[1] / a.push[2] : 0;
  if (!seq || !hd) return cudaSuccess;
  const dim3 grid((hd + kSc - 1) / kSc, (seq + kSc - 1) / kSc, a.push[2]);
  k_attn_context<true><<<grid, 256, 0, a.stream>>>((const float *)a.buf[0], (const float *)a.buf[1],
                                                  (float *)a.buf[2], seq, a.push[1], a.push[2],
                                                  a.push[3], invocations(a.groups, 64));
  count_launches(1);
  return cudaPeekAtLastError();
}
const char *chk_dp(const OpArgs &a) {
  const uint64_t seq = a.push[0], dim = a.push[1], heads = a.push[2], kvheads = a.push[3];
  if (!heads || !kvheads || dim % heads || heads % kvheads)
    return fmt_msg("attention: dim %u, heads %u, kvheads %u do not divide", a.push[1], a.push[2],
                   a.push[3]);
  const char *m;
  if ((m = need_words(a, 0, seq * dim, "DC"))) return m;
  if ((m = need_words(a, 1, seq * kvheads * (dim / heads), "V"))) return m;
  return need_words(a, 2, heads * seq * seq, "DP");
}
cudaError_t run_dp(const OpArgs &a) {
  const uint32_t seq = a.push[0];
  if (!seq) return cudaSuccess;
  const dim3 grid((seq + kSc - 1) / kSc, (seq + kSc - 1) / kSc, a.push[2]);
  k_attn_scores<false><<<grid, 256, 0, a.stream>>>((const float *)a.buf[0], (const float *)a.buf[1],
                                                  (float *)a.buf[2], seq, a.push[1], a.push[2],
                                                  a.push[3], invocations(a.groups, 64));
  count_launches(1);
  return cudaPeekAtLastError();
}
// DK[j,kvh,t] = scale * sum_{h in group} sum_i DS[h,i,j] Q[i,h,t] (DV: P, DC, no scale)
template <bool SCALED>
__global__ void k_attn_kv_grad(const float *__restrict__ D, const float *__restrict__ X,
                               float *__restrict__ OUT, uint32_t seq, uint32_t dim, uint32_t heads,
                               uint32_t kvheads, uint64_t limit) {
  const uint32_t hd = dim / heads, grp = heads / kvheads, kvdim = kvheads * hd;
  const uint64_t total = (uint64_t)seq * kvdim;
  for (uint64_t idx = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total && idx < limit;
       idx += (uint64_t)gridDim.x * blockDim.x) {
    const uint32_t j = (uint32_t)(idx / kvdim), rem = (uint32_t)(idx % kvdim);
    const uint32_t kvh = rem / hd, t = rem % hd;
    float acc = 0.0f;
    for (uint32_t hh = 0; hh < grp; hh++) {
      const uint32_t h = kvh * grp + hh;
      const float *dcol = D + (uint64_t)h * seq * seq + j;
      const float *xcol = X + (uint64_t)h * hd + t;
      for (uint32_t i = 0; i < seq; i++)
        acc = __fadd_rn(acc, __fmul_rn(__ldg(dcol + (uint64_t)i * seq), __ldg(xcol + (uint64_t)i * dim)));
    }
    OUT[idx] = SCALED ? acc * (1.0f / sqrtf((float)hd)) : acc;
  }
}
template <bool SCALED>
const char *chk_kv_grad(const OpArgs &a) {
  const uint64_t seq = a.push[0], dim = a.push[1], heads = a.push[2], kvheads = a.push[3];
  if (!heads || !kvheads || dim % heads || heads % kvheads)
    return fmt_msg("attention: dim %u, heads %u, kvheads %u do not divide", a.push[1], a.push[2],
                   a.push[3]);
  const char *m;
  // buffer 0 is DS (attn-sc-dk) or DC (attn-ctx-dv); buffer 1 is Q or P
  if ((m = need_words(a, SCALED ? 0 : 1, heads * seq * seq, SCALED ? "DS" : "P"))) return m;
  if ((m = need_words(a, SCALED ? 1 : 0, seq * dim, SCALED ? "Q" : "DC"))) return m;
  return need_words(a, 2, seq * kvheads * (dim / heads), SCALED ? "DK" : "DV");
}
template <bool SCALED>
cudaError_t run_kv_grad(const OpArgs &a) {
  const uint64_t n = (uint64_t)a.push[0] * (a.push[2] ? a.push[3] * (a.push[1] / a.push[2]) : 0);
  if (!n) return cudaSuccess;
  // attn-sc-dk: (DS Q DK); attn-ctx-dv: (DC P DV) -- the score-shaped operand first
  const float *Dm = (const float *)a.buf[SCALED ? 0 : 1];
  const float *Xm = (const float *)a.buf[SCALED ? 1 : 0];
  k_attn_kv_grad<SCALED><<<blocks_for(n), 256, 0, a.stream>>>(Dm, Xm, (float *)a.buf[2], a.push[0],
                                                              a.push[1], a.push[2], a.push[3],
                                                              invocations(a.groups, 64));
  count_launches(1);
  return cudaPeekAtLastError();
}

// ---- dp4a family ------------------------------------------------------------------
__device__ __forceinline__ uint32_t word_of(const float *lo, const float *hi, uint64_t i) {
  return f2u(__ldg(lo + i)) + f2u(__ldg(hi + i)) * 65536u;
}
__global__ void k_dp4a_dot(const float *ALO, const float *AHI, const float *BLO, const float *BHI,
                           float *OUT, uint32_t n, uint64_t limit) {
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n && i < limit;
       i += (uint64_t)gridDim.x * blockDim.x)
    OUT[i] = (float)__dp4a((int)word_of(ALO, AHI, i), (int)word_of(BLO, BHI, i), 0);
}
// one warp per output, lanes over the groups, exact int32 sum
__global__ void k_bitlinear_dp4a(const float *ALO, const float *AHI, const float *WLO,
                                 const float *WHI, const float *BIAS, const float *BETA,
                                 const float *GAMMA, float *Y, uint32_t seq, uint32_t out,
                                 uint32_t ng, uint64_t limit) {
  const uint64_t idx = (uint64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (idx >= (uint64_t)seq * out) return;
  const uint32_t s = (uint32_t)(idx / out), o = (uint32_t)(idx % out);
  int acc = 0;
  for (uint32_t g = lane; g < ng; g += 32)
    acc = __dp4a((int)word_of(ALO, AHI, (uint64_t)s * ng + g),
                 (int)word_of(WLO, WHI, (uint64_t)o * ng + g), acc);
  for (int d = 16; d > 0; d >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, d);
  if (lane == 0 && idx < limit)
    Y[idx] = __fadd_rn(__ldg(BIAS + o), __fmul_rn(__fmul_rn(__ldg(BETA), __ldg(GAMMA + s)),
                                                  (float)acc));
}
// X[p, i]: one thread per (p, i), the reference's order over o
__global__ void k_dp4a_rows_t(const float *WP, const float *BETA, const float *G, float *X,
                              uint32_t out, uint32_t cols, uint32_t ng, uint32_t seq,
                              uint64_t limit) {
  const uint64_t idx = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (uint64_t)seq * cols || idx >= limit) return;
  const uint32_t p = (uint32_t)(idx / cols), i = (uint32_t)(idx % cols);
  const uint32_t word = i / 4, lane = i % 4;
  const float *gp = G + (uint64_t)p * out;
  float acc = 0.0f;
  for (uint32_t o = 0; o < out; o++) {
    const uint32_t w = __float_as_uint(__ldg(WP + (uint64_t)o * ng + word));
    const float sv = (float)(int)(int8_t)(w >> (8 * lane));
    acc = __fadd_rn(acc, __fmul_rn(sv, __fmul_rn(__ldg(BETA + o), __ldg(gp + o))));
  }
  X[idx] = acc;
}
const char *chk_dp4a_dot(const OpArgs &a) {
  const char *m;
  for (uint32_t b = 0; b < 5; b++)
    if ((m = need_words(a, b, a.push[0], b < 4 ? "A/B halves" : "OUT"))) return m;
  return nullptr;
}
cudaError_t run_dp4a_dot(const OpArgs &a) {
  if (!a.push[0]) return cudaSuccess;
  k_dp4a_dot<<<blocks_for(a.push[0]), 256, 0, a.stream>>>(
      (const float *)a.buf[0], (const float *)a.buf[1], (const float *)a.buf[2],
      (const float *)a.buf[3], (float *)a.buf[4], a.push[0], invocations(a.groups, 64));
  count_launches(1);
  return cudaPeekAtLastError();
}
const char *chk_bitlinear_dp4a(const OpArgs &a) {
  const uint64_t seq = a.push[0], out = a.push[1], ng = a.push[2];
  const char *m;
  if ((m = need_words(a, 0, seq * ng, "ALO")) || (m = need_words(a, 1, seq * ng, "AHI")) ||
      (m = need_words(a, 2, out * ng, "WLO")) || (m = need_words(a, 3, out * ng, "WHI")) ||
      (m = need_words(a, 4, out, "BIAS")) || (m = need_words(a, 5, 1, "BETA")) ||
      (m = need_words(a, 6, seq, "GAMMA")))
    return m;
  return need_words(a, 7, seq * out, "Y");
}
cudaError_t run_bitlinear_dp4a(const OpArgs &a) {
  const uint64_t n = (uint64_t)a.push[0] * a.push[1];
  if (!n) return cudaSuccess;
  k_bitlinear_dp4a<<<(unsigned)ceil_div64(n, 8), 256, 0, a.stream>>>(
      (const float *)a.buf[0], (const float *)a.buf[1], (const float *)a.buf[2],
      (const float *)a.buf[3], (const float *)a.buf[4], (const float *)a.buf[5],
      (const float *)a.buf[6], (float *)a.buf[7], a.push[0], a.push[1], a.push[2],
      invocations(a.groups, 64));
  count_launches(1);
  return cudaPeekAtLastError();
}
const char *chk_dp4a_rows_t(const OpArgs &a) {
  const uint64_t out = a.push[0], cols = a.push[1], ng = a.push[2], seq = a.push[3];
  if (cols > 4 * ng) return fmt_msg("dp4a-rows-t: cols %u exceed 4 x ng %u", a.push[1], a.push[2]);
  const char *m;
  if ((m = need_words(a, 0, out * ng, "WP")) || (m = need_words(a, 1, out, "BETA")) ||
      (m = need_words(a, 2, seq * out, "G")))
    return m;
  return need_words(a, 3, seq * cols, "X");
}
cudaError_t run_dp4a_rows_t(const OpArgs &a) {
  const uint64_t n = (uint64_t)a.push[3] * a.push[1];
  if (!n) return cudaSuccess;
  k_dp4a_rows_t<<<(unsigned)ceil_div64(n, 128), 128, 0, a.stream>>>(
      (const float *)a.buf[0], (const float *)a.buf[1], (const float *)a.buf[2], (float *)a.buf[3],
      a.push[0], a.push[1], a.push[2], a.push[3], invocations(a.groups, 64));
  count_launches(1);
  return cudaPeekAtLastError();
}

// ---- rmsnorm-heads: one warp per (position, head) ------------------------------------
__global__ void k_rmsnorm_heads(const float *X, const float *G, float *Y, uint32_t rows,
                                uint32_t hd, uint64_t limit) {
  const uint64_t r = (uint64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (r >= rows || r >= limit) return;
  const float *x = X + r * hd;
  float ss = 0.0f;
  for (uint32_t i = lane; i < hd; i += 32) ss = fmaf(x[i], x[i], ss);
  for (int d = 16; d > 0; d >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, d);
  const float inv = 1.0f / sqrtf(ss / (float)hd + 0.000001f);
  for (uint32_t j = lane; j < hd; j += 32) Y[r * hd + j] = __fmul_rn(__fmul_rn(x[j], inv), G[j]);
}
const char *chk_rmsnorm_heads(const OpArgs &a) {
  const uint64_t n = (uint64_t)a.push[0] * a.push[1] * a.push[2];
  const char *m;
  if ((m = need_words(a, 0, n, "X")) || (m = need_words(a, 1, a.push[2], "G"))) return m;
  return need_words(a, 2, n, "Y");
}
cudaError_t run_rmsnorm_heads(const OpArgs &a) {
  const uint64_t rows = (uint64_t)a.push[0] * a.push[1];
  if (!rows || !a.push[2]) return cudaSuccess;
  k_rmsnorm_heads<<<(unsigned)ceil_div64(rows, 8), 256, 0, a.stream>>>(
      (const float *)a.buf[0], (const float *)a.buf[1], (float *)a.buf[2], (uint32_t)rows,
      a.push[2], invocations(a.groups, 64));
  count_launches(1);
  return cudaPeekAtLastError();
}

// ---- rope-apply: adjacent pairs at the row's position p (tables [seq x half]) ------
__global__ void k_rope_apply(const float *X, const float *CO, const float *SI, const float *SG,
                             float *C, uint32_t seq, uint32_t dim, uint32_t heads,
                             uint64_t limit) {
  const uint32_t hd = dim / heads, half = hd / 2;
  const uint64_t total = (uint64_t)seq * heads * half;
  for (uint64_t idx = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total && idx < limit;
       idx += (uint64_t)gridDim.x * blockDim.x) {
    const uint32_t m = (uint32_t)(idx % half);
    const uint64_t tmp = idx / half;
    const uint32_t h = (uint32_t)(tmp % heads), p = (uint32_t)(tmp / heads);
    const uint64_t ci = (uint64_t)p * half + m;
    const float cc = CO[ci], ss = SI[ci] * SG[0];
    const uint64_t i0 = (uint64_t)p * dim + (uint64_t)h * hd + 2 * m;
    const float a0 = X[i0], a1 = X[i0 + 1];
    C[i0] = a0 * cc - a1 * ss;
    C[i0 + 1] = a0 * ss + a1 * cc;
  }
}
const char *chk_rope_apply(const OpArgs &a) {
  const uint64_t seq = a.push[0], dim = a.push[1], heads = a.push[2];
  if (!heads || dim % heads || (dim / heads) % 2)
    return fmt_msg("rope-apply: dim %u, heads %u (even head size)", a.push[1], a.push[2]);
  const uint64_t half = dim / heads / 2;
  const char *m;
  if ((m = need_words(a, 0, seq * dim, "X")) || (m = need_words(a, 1, seq * half, "CO")) ||
      (m = need_words(a, 2, seq * half, "SI")) || (m = need_words(a, 3, 1, "SG")))
    return m;
  return need_words(a, 4, seq * dim, "C");
}
cudaError_t run_rope_apply(const OpArgs &a) {
  const uint64_t n = (uint64_t)a.push[0] * a.push[1] / 2;
  if (!n) return cudaSuccess;
  k_rope_apply<<<blocks_for(n), 256, 0, a.stream>>>(
      (const float *)a.buf[0], (const float *)a.buf[1], (const float *)a.buf[2],
      (const float *)a.buf[3], (float *)a.buf[4], a.push[0], a.push[1], a.push[2],
      invocations(a.groups, 64));
  count_launches(1);
  return cudaPeekAtLastError();
}

// ---- silu, scale-rows (float4 streams where aligned) ---------------------------------
__global__ void k_silu(const float *X, float *C, uint64_t n) {
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (uint64_t)gridDim.x * blockDim.x) {
    const float x = X[i];
    C[i] = __fmul_rn(x, 1.0f / (1.0f + expf(-x)));
  }
}
__global__ void k_scale_rows(const float *Y, const float *S, float *C, uint32_t N, uint64_t n) {
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (uint64_t)gridDim.x * blockDim.x)
    C[i] = __fmul_rn(Y[i], S[i / N]);
}
const char *chk_silu(const OpArgs &a) {
  const char *m;
  if ((m = need_words(a, 0, a.push[0], "X"))) return m;
  return need_words(a, 1, a.push[0], "C");
}
cudaError_t run_silu(const OpArgs &a) {
  uint64_t n = a.push[0], lim = invocations(a.groups, 64);
  if (lim < n) n = lim;
  if (!n) return cudaSuccess;
  k_silu<<<blocks_for(n), 256, 0, a.stream>>>((const float *)a.buf[0], (float *)a.buf[1], n);
  count_launches(1);
  return cudaPeekAtLastError();
}
const char *chk_scale_rows(const OpArgs &a) {
  const uint64_t n = (uint64_t)a.push[0] * a.push[1];
  const char *m;
  if ((m = need_words(a, 0, n, "Y")) || (m = need_words(a, 1, a.push[0], "S"))) return m;
  return need_words(a, 2, n, "C");
}
cudaError_t run_scale_rows(const OpArgs &a) {
  uint64_t n = (uint64_t)a.push[0] * a.push[1], lim = invocations(a.groups, 64);
  if (lim < n) n = lim;
  if (!n) return cudaSuccess;
  k_scale_rows<<<blocks_for(n), 256, 0, a.stream>>>((const float *)a.buf[0],
                                                    (const float *)a.buf[1], (float *)a.buf[2],
                                                    a.push[1], n);
  count_launches(1);
  return cudaPeekAtLastError();
}

}  // namespace

const OpSpec kMiscOps[] = {
    {"causal-mask", 1, 1, chk_causal_mask, no_scr, run_causal_mask},
    {"attn-scores", 3, 4, chk_scores, no_scr, run_scores},
    {"attn-context", 3, 4, chk_context, no_scr, run_context},
    {"attn-sc-dq", 3, 4, chk_dq, no_scr, run_dq},
    {"attn-sc-dk", 3, 4, chk_kv_grad<true>, no_scr, run_kv_grad<true>},
    {"attn-ctx-dp", 3, 4, chk_dp, no_scr, run_dp},
    {"attn-ctx-dv", 3, 4, chk_kv_grad<false>, no_scr, run_kv_grad<false>},
    {"dp4a-dot", 5, 1, chk_dp4a_dot, no_scr, run_dp4a_dot},
    {"bitlinear-dp4a", 8, 3, chk_bitlinear_dp4a, no_scr, run_bitlinear_dp4a},
    {"dp4a-rows-t", 4, 4, chk_dp4a_rows_t, no_scr, run_dp4a_rows_t},
    {"rmsnorm-heads", 3, 3, chk_rmsnorm_heads, no_scr, run_rmsnorm_heads},
    {"rope-apply", 5, 3, chk_rope_apply, no_scr, run_rope_apply},
    {"silu", 2, 1, chk_silu, no_scr, run_silu},
    {"scale-rows", 3, 2, chk_scale_rows, no_scr, run_scale_rows},
};
const int kMiscOpsCount = sizeof(kMiscOps) / sizeof(kMiscOps[0]);

}  // namespace nl

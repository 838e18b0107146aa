// k_quant.cu -- BitNet b1.58 quantization: the reference's weight / activation
// quantization operators and the on-device repacking of an f32 weight matrix
// into the two-bit GEMV format.
//
// Reference operators (lisp/nelisp-gpu-kernels.el):
//   sumsq-acc   :496-503   GSQ[0] += sum G^2
//   clip-scale  :505-512   SCALE[0] = min(1, CFG[0] / sqrt(GSQ[0] + 1e-12))
//   absmean-acc :516-526   ACC[0] += sum |G|
//   quant-act   :529-548   per row: gamma = max|x| / 127, XQ = gamma * clip(round(x / gamma))
//   quant-w     :550-561   beta = S[0] / n, WQ = beta * (W/beta >= 0.5 ? 1 : W/beta <= -0.5 ? -1 : 0)
// The reference's two accumulators sum serially in one thread in f32; here
// the sum is a parallel f64 reduction (fixed order, so the result is
// reproducible) added to the accumulator once in f32 -- within f32 rounding
// of the reference's, not bit-identical.  quant-act, quant-w and clip-scale
// are elementwise and bit-identical.
//
// quant_w_pack_launch: the importer's dense f32 weights -> quant-w's ternary
// values, written directly as packed two-bit codes (field i of word i/16 at
// bits 2(i%16): 00 -> 0, 01 -> +1, 11 -> -1) plus the scale per row, the
// operands of the ternary GEMV; beta is mean |W| per tensor (quant-w) or per
// row.  diag(S) (T x) then equals quant-w's fake-quantized weights times x.

#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include "nl_internal.h"

namespace nl {
namespace {

size_t no_scr(const OpArgs &) { return 0; }

// Block-wide f64 sum (blockDim.x a multiple of 32, <= 1024), fixed order.
__device__ double block_sum(double v) {
  __shared__ double red[32];
  for (int o = 16; o > 0; o >>= 1) v += __shfl_down_sync(0xffffffffu, v, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  double t = 0.0;
  if (threadIdx.x == 0)
    for (int w = 0; w < (int)(blockDim.x >> 5); w++) t += red[w];
  __syncthreads();
  return t;                                   // valid in thread 0
}

// ---- absmean-acc / sumsq-acc: one CTA, grid-stride over G ---------------------
template <bool SQ>
__global__ void k_acc(const float *__restrict__ G, float *ACC, uint32_t n) {
  double s = 0.0;
  for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) {
    const double g = (double)G[i];
    s += SQ ? g * g : fabs(g);
  }
  s = block_sum(s);
  if (threadIdx.x == 0) ACC[0] = __fadd_rn(ACC[0], (float)s);
}
const char *chk_acc(const OpArgs &a) {
  const char *m;
  if ((m = need_words(a, 0, a.push[0], "G"))) return m;
  return need_words(a, 1, 1, "ACC");
}
template <bool SQ>
cudaError_t run_acc(const OpArgs &a) {
  if (!a.groups) return cudaSuccess;         // invocation 0 does the work
  k_acc<SQ><<<1, 1024, 0, a.stream>>>((const float *)a.buf[0], (float *)a.buf[1], a.push[0]);
  count_launches(1);
  return cudaPeekAtLastError();
}

// ---- clip-scale ---------------------------------------------------------------
__global__ void k_clip_scale(const float *GSQ, const float *CFG, float *SCALE) {
  const float s = __fdiv_rn(CFG[0], sqrtf(__fadd_rn(GSQ[0], 1.0e-12f)));
  SCALE[0] = s < 1.0f ? s : 1.0f;
}
const char *chk_clip(const OpArgs &a) {
  const char *m;
  if ((m = need_words(a, 0, 1, "GSQ")) || (m = need_words(a, 1, 1, "CFG"))) return m;
  return need_words(a, 2, 1, "SCALE");
}
cudaError_t run_clip(const OpArgs &a) {
  if (!a.groups) return cudaSuccess;
  k_clip_scale<<<1, 1, 0, a.stream>>>((const float *)a.buf[0], (const float *)a.buf[1],
                                      (float *)a.buf[2]);
  count_launches(1);
  return cudaPeekAtLastError();
}

// ---- quant-act: one CTA per row -----------------------------------------------
__global__ void k_quant_act(const float *__restrict__ X, float *__restrict__ XQ, uint32_t seq,
                            uint32_t cols, uint64_t limit) {
  __shared__ float red[32];
  const uint32_t row = blockIdx.x;
  if (row >= seq || row >= limit) return;
  const float *x = X + (size_t)row * cols;
  float m = 0.0f;
  for (uint32_t c = threadIdx.x; c < cols; c += blockDim.x) m = fmaxf(m, fabsf(x[c]));
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  float amax = 0.0f;
  for (int w = 0; w < (int)(blockDim.x >> 5); w++) amax = fmaxf(amax, red[w]);
  const float gamma = __fdiv_rn(amax, 127.0f);
  for (uint32_t c = threadIdx.x; c < cols; c += blockDim.x) {
    const float v = x[c];
    float xq = 0.0f;
    if (gamma > 0.0f) {
      const float q = __fdiv_rn(v, gamma);
      const float sgn = q < 0.0f ? -1.0f : 1.0f, aq = q < 0.0f ? -q : q;
      float rf = (float)__float2uint_rz(__fadd_rn(aq, 0.5f));
      if (rf > 127.0f) rf = 127.0f;
      xq = __fmul_rn(gamma, __fmul_rn(sgn, rf));
    }
    XQ[(size_t)row * cols + c] = xq;
  }
}
const char *chk_quant_act(const OpArgs &a) {
  const uint64_t n = (uint64_t)a.push[0] * a.push[1];
  const char *m;
  if ((m = need_words(a, 0, n, "X"))) return m;
  return need_words(a, 1, n, "XQ");
}
cudaError_t run_quant_act(const OpArgs &a) {
  if (!a.push[0] || !a.push[1]) return cudaSuccess;
  k_quant_act<<<a.push[0], 256, 0, a.stream>>>((const float *)a.buf[0], (float *)a.buf[1],
                                               a.push[0], a.push[1], invocations(a.groups, 64));
  count_launches(1);
  return cudaPeekAtLastError();
}

// ---- quant-w ------------------------------------------------------------------
__device__ __forceinline__ int trit_of_q(float w, float beta) {
  if (!(beta > 0.0f)) return 0;
  const float q = __fdiv_rn(w, beta);
  return q >= 0.5f ? 1 : (q <= -0.5f ? -1 : 0);
}
__global__ void k_quant_w(const float *__restrict__ W, const float *__restrict__ S,
                          float *__restrict__ WQ, uint32_t n, uint64_t limit) {
  const float beta = __fdiv_rn(S[0], (float)n);
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n && i < limit;
       i += (uint64_t)gridDim.x * blockDim.x)
    WQ[i] = __fmul_rn(beta, (float)trit_of_q(W[i], beta));
}
const char *chk_quant_w(const OpArgs &a) {
  const char *m;
  if ((m = need_words(a, 0, a.push[0], "W")) || (m = need_words(a, 1, 1, "S"))) return m;
  return need_words(a, 2, a.push[0], "WQ");
}
cudaError_t run_quant_w(const OpArgs &a) {
  if (!a.push[0]) return cudaSuccess;
  k_quant_w<<<grid_for(a.push[0], 256, 148u * 64u), 256, 0, a.stream>>>(
      (const float *)a.buf[0], (const float *)a.buf[1], (float *)a.buf[2], a.push[0],
      invocations(a.groups, 64));
  count_launches(1);
  return cudaPeekAtLastError();
}

// ---- f32 matrix -> packed ternary + scales ---------------------------------------
__global__ void k_row_abssum(const float *__restrict__ W, uint32_t cols, double *rowsum) {
  const float *w = W + (size_t)blockIdx.x * cols;
  double s = 0.0;
  for (uint32_t c = threadIdx.x; c < cols; c += blockDim.x) s += fabs((double)w[c]);
  s = block_sum(s);
  if (threadIdx.x == 0) rowsum[blockIdx.x] = s;
}
__global__ void k_tensor_beta(const double *rowsum, uint32_t rows, uint64_t n, float *beta) {
  double s = 0.0;
  for (uint32_t r = threadIdx.x; r < rows; r += blockDim.x) s += rowsum[r];
  s = block_sum(s);
  if (threadIdx.x == 0) *beta = (float)(s / (double)n);
}
// One thread per packed word: sixteen thresholded fields.
__global__ void k_pack_trits(const float *__restrict__ W, uint32_t rows, uint32_t cols,
                             const double *rowsum, const float *tensor_beta, uint32_t *WP,
                             float *S) {
  const uint32_t wng = (cols + 15) / 16;
  const uint64_t total = (uint64_t)rows * wng;
  for (uint64_t idx = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (uint64_t)gridDim.x * blockDim.x) {
    const uint32_t o = (uint32_t)(idx / wng), wi = (uint32_t)(idx % wng);
    const float beta = tensor_beta ? *tensor_beta : (float)(rowsum[o] / (double)cols);
    const float *w = W + (size_t)o * cols + 16u * wi;
    uint32_t word = 0;
#pragma unroll
    for (int f = 0; f < 16; f++) {
      const uint32_t c = 16u * wi + f;
      const int t = c < cols ? trit_of_q(w[f], beta) : 0;
      word |= (t == 1 ? 1u : (t == -1 ? 3u : 0u)) << (2 * f);
    }
    WP[idx] = word;
    if (wi == 0) S[o] = beta;
  }
}

}  // namespace

size_t quant_w_scratch_bytes(uint32_t rows) { return ((size_t)rows + 2) * sizeof(double); }

cudaError_t quant_w_pack_launch(const float *W, uint32_t rows, uint32_t cols, bool per_row,
                                uint32_t *WP, float *S, void *scratch, cudaStream_t st) {
  if (!rows || !cols) return cudaSuccess;
  double *rowsum = (double *)scratch;
  float *tbeta = per_row ? nullptr : (float *)(rowsum + rows);
  k_row_abssum<<<rows, 256, 0, st>>>(W, cols, rowsum);
  if (!per_row) k_tensor_beta<<<1, 1024, 0, st>>>(rowsum, rows, (uint64_t)rows * cols, tbeta);
  const uint64_t words = (uint64_t)rows * ((cols + 15) / 16);
  k_pack_trits<<<grid_for(words, 256, 148u * 32u), 256, 0, st>>>(W, rows, cols, rowsum, tbeta,
                                                                  WP, S);
  count_launches(per_row ? 2 : 3);
  return cudaPeekAtLastError();
}

const OpSpec kQuantOps[] = {
    {"sumsq-acc", 2, 1, chk_acc, no_scr, run_acc<true>},
    {"clip-scale", 3, 1, chk_clip, no_scr, run_clip},
    {"absmean-acc", 2, 1, chk_acc, no_scr, run_acc<false>},
    {"quant-act", 2, 2, chk_quant_act, no_scr, run_quant_act},
    {"quant-w", 3, 1, chk_quant_w, no_scr, run_quant_w},
};
const int kQuantOpsCount = sizeof(kQuantOps) / sizeof(kQuantOps[0]);

}  // namespace nl

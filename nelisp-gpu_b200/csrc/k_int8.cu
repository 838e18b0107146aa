// k_int8.cu -- int8 activation quantizer and the DP4A linear for sm_100a.
//
// Reference operators (lisp/nelisp-gpu-kernels.el):
//   pack-act-rows       :898-932  per row: gamma = amax/127, lanes
//                                 r = min(uint(|v/gamma| + 0.5), 127), two's
//                                 complement for negatives, 4 lanes per word
//   bitlinear-dp4a-rows :642-653  Y = BIAS[o] + (BETA[o]*GAMMA[s]) * float(acc)
//   bitlinear-dp4a-1f   :623-634  the same with BETA[0]
//
// Both are bit-exact against the CPU restatement: the quantizer uses IEEE
// division and rounding-mode-explicit adds, the accumulator is an exact
// int32 sum (wrapping like the reference's 32-bit OpIAdd, so the order of
// the warp reduction does not change it), and the epilogue's multiplies and
// add are not contracted into an FMA.

#include <cuda_runtime.h>
#include <stdint.h>

#include "nl_internal.h"

namespace nl {
namespace {

__global__ void __launch_bounds__(256)
pack_act_rows_kernel(const float *__restrict__ X, uint32_t *__restrict__ XQ,
                     float *__restrict__ GAMMA, uint32_t seq, uint32_t cols,
                     uint32_t ng, uint64_t limit) {
  __shared__ float red[8];
  __shared__ float s_gamma;
  const uint32_t row = blockIdx.x;
  if (row >= seq || row >= limit) return;
  const float *x = X + (uint64_t)row * cols;
  float amax = 0.0f;
  for (uint32_t c = threadIdx.x; c < cols; c += blockDim.x)
    amax = fmaxf(amax, fabsf(__ldg(x + c)));   // NaN never wins, as in `>`
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
  __syncthreads();
  if (threadIdx.x == 0) {
    float m = 0.0f;
    for (int w = 0; w < (int)(blockDim.x >> 5); w++) m = fmaxf(m, red[w]);
    float gamma = __fdiv_rn(m, 127.0f);
    s_gamma = gamma;
    GAMMA[row] = gamma;
  }
  __syncthreads();
  const float gamma = s_gamma;
  for (uint32_t w = threadIdx.x; w < ng; w += blockDim.x) {
    uint32_t word = 0;
#pragma unroll
    for (uint32_t l = 0; l < 4; l++) {
      uint32_t c = w * 4 + l, lane = 0;
      if (c < cols) {
        float v = __ldg(x + c);
        float q = 0.0f;
        if (gamma > 0.0f) q = __fdiv_rn(v, gamma);
        bool neg = q < 0.0f;
        float aq = neg ? __fsub_rn(0.0f, q) : q;
        uint32_t ri = __float2uint_rz(__fadd_rn(aq, 0.5f));
        if (ri > 127u) ri = 127u;
        lane = neg ? (256u - ri) % 256u : ri;
      }
      word += lane << (8 * l);
    }
    XQ[(uint64_t)row * ng + w] = word;
  }
}

// One warp per output row o; lanes take words; sequence rows in chunks of 8.
__global__ void __launch_bounds__(256)
dp4a_rows_kernel(const uint32_t *__restrict__ AP, const uint32_t *__restrict__ WP,
                 const float *__restrict__ BIAS, const float *__restrict__ BETA,
                 const float *__restrict__ GAMMA, float *__restrict__ Y,
                 uint32_t seq, uint32_t out, uint32_t ng, int per_row,
                 uint64_t limit) {
  const uint32_t o = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (o >= out) return;
  const uint32_t *w = WP + (uint64_t)o * ng;
  const float beta = per_row ? __ldg(BETA + o) : __ldg(BETA);
  const float bias = __ldg(BIAS + o);
  for (uint32_t s0 = 0; s0 < seq; s0 += 8) {
    const uint32_t ns = min(8u, seq - s0);
    int acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (uint32_t g = lane; g < ng; g += 32) {
      int wv = (int)__ldg(w + g);
#pragma unroll
      for (uint32_t s = 0; s < 8; s++)
        if (s < ns) acc[s] = __dp4a((int)__ldg(AP + (uint64_t)(s0 + s) * ng + g), wv, acc[s]);
    }
#pragma unroll
    for (uint32_t s = 0; s < 8; s++) {
      int v = acc[s];
      for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
      acc[s] = v;
    }
    if (lane == 0) {
      for (uint32_t s = 0; s < ns; s++) {
        uint64_t idx = (uint64_t)(s0 + s) * out + o;
        if (idx >= limit) continue;
        float bg = __fmul_rn(beta, __ldg(GAMMA + s0 + s));
        Y[idx] = __fadd_rn(bias, __fmul_rn(bg, __int2float_rn(acc[s])));
      }
    }
  }
}

size_t no_scratch(const OpArgs &) { return 0; }

const char *chk_pack(const OpArgs &a) {
  // (X XQ GAMMA) push (seq cols ng)
  uint64_t seq = a.push[0], cols = a.push[1], ng = a.push[2];
  const char *m;
  if ((m = need_words(a, 0, seq * cols, "X"))) return m;
  if ((m = need_words(a, 1, seq * ng, "XQ"))) return m;
  return need_words(a, 2, seq, "GAMMA");
}
cudaError_t run_pack(const OpArgs &a) {
  if (a.push[0] == 0) return cudaSuccess;
  pack_act_rows_kernel<<<a.push[0], 256, 0, a.stream>>>(
      (const float *)a.buf[0], (uint32_t *)a.buf[1], (float *)a.buf[2],
      a.push[0], a.push[1], a.push[2], invocations(a.groups, 64));
  count_launches(1);
  return cudaPeekAtLastError();
}

template <int PER_ROW>
const char *chk_dp4a(const OpArgs &a) {
  // (AP WP BIAS BETA GAMMA Y) push (seq out ng)
  uint64_t seq = a.push[0], out = a.push[1], ng = a.push[2];
  bool any = seq && out;
  const char *m;
  if ((m = need_words(a, 0, any ? seq * ng : 0, "AP"))) return m;
  if ((m = need_words(a, 1, any ? out * ng : 0, "WP"))) return m;
  if ((m = need_words(a, 2, any ? out : 0, "BIAS"))) return m;
  if ((m = need_words(a, 3, any ? (PER_ROW ? out : 1) : 0, "BETA"))) return m;
  if ((m = need_words(a, 4, any ? seq : 0, "GAMMA"))) return m;
  return need_words(a, 5, seq * out, "Y");
}
template <int PER_ROW>
cudaError_t run_dp4a(const OpArgs &a) {
  if (a.push[0] == 0 || a.push[1] == 0) return cudaSuccess;
  dp4a_rows_kernel<<<(a.push[1] + 7) / 8, 256, 0, a.stream>>>(
      (const uint32_t *)a.buf[0], (const uint32_t *)a.buf[1],
      (const float *)a.buf[2], (const float *)a.buf[3], (const float *)a.buf[4],
      (float *)a.buf[5], a.push[0], a.push[1], a.push[2], PER_ROW,
      invocations(a.groups, 64));
  count_launches(1);
  return cudaPeekAtLastError();
}

}  // namespace

const OpSpec kInt8Ops[] = {
    {"pack-act-rows", 3, 3, chk_pack, no_scratch, run_pack},
    {"bitlinear-dp4a-rows", 6, 3, chk_dp4a<1>, no_scratch, run_dp4a<1>},
    {"bitlinear-dp4a-1f", 6, 3, chk_dp4a<0>, no_scratch, run_dp4a<0>},
};
const int kInt8OpsCount = sizeof(kInt8Ops) / sizeof(kInt8Ops[0]);

}  // namespace nl

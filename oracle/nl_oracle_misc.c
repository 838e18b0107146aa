/* nl_oracle_misc.c -- CPU restatements (test infrastructure only: the parity
 * checker for libnelisp_cuda, never a product path) of the reference
 * operators for the unfused prefill attention pieces, QK-norm, adjacent-pair
 * RoPE, SiLU, row scaling, the DP4A spikes, the backward GEMMs and the BitNet
 * quantization family (with the on-device repacking of upload-file).  One loop
 * iteration per reference invocation (gid-x), the reference's f32 operation
 * order, no contraction (built with -ffp-contract=off). */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include "nl_oracle.h"

static uint32_t u_of(float v) { return v > 0.0f ? (uint32_t)v : 0u; }

/* lisp/nelisp-gpu-kernels.el:177-186 (matmul-at): C[m,n] = sum_k A[k,m] B[k,n] */
void nlo_matmul_at(const float *A, const float *B, float *C, uint32_t M, uint32_t K,
                   uint32_t N) {
  long long total = (long long)M * N;
#pragma omp parallel for schedule(static)
  for (long long idx = 0; idx < total; idx++) {
    uint32_t m = (uint32_t)(idx / N), n = (uint32_t)(idx % N);
    float acc = 0.0f;
    for (uint32_t k = 0; k < K; k++) acc = acc + A[(size_t)k * M + m] * B[(size_t)k * N + n];
    C[idx] = acc;
  }
}

/* :148-155 (causal-mask) */
void nlo_causal_mask(float *S, uint32_t n) {
  for (uint64_t i = 0; i < n; i++)
    for (uint64_t j = i + 1; j < n; j++) S[i * n + j] = -1.0e30f;
}

/* :208-221 (attn-scores) */
void nlo_attn_scores(const float *Q, const float *K, float *S, uint32_t seq, uint32_t dim,
                     uint32_t heads, uint32_t kvheads) {
  uint32_t hd = dim / heads, grp = heads / kvheads, kvdim = kvheads * hd;
  float scale = 1.0f / sqrtf((float)hd);
  long long total = (long long)heads * seq * seq;
#pragma omp parallel for schedule(static)
  for (long long idx = 0; idx < total; idx++) {
    uint32_t h = (uint32_t)(idx / ((long long)seq * seq));
    uint64_t rem = (uint64_t)(idx % ((long long)seq * seq));
    uint32_t i = (uint32_t)(rem / seq), j = (uint32_t)(rem % seq);
    if (j > i) { S[idx] = -1.0e30f; continue; }
    const float *q = Q + (size_t)i * dim + (size_t)h * hd;
    const float *k = K + (size_t)j * kvdim + (size_t)(h / grp) * hd;
    float acc = 0.0f;
    for (uint32_t t = 0; t < hd; t++) acc = acc + q[t] * k[t];
    S[idx] = acc * scale;
  }
}

/* :224-235 (attn-context) */
void nlo_attn_context(const float *P, const float *V, float *C, uint32_t seq, uint32_t dim,
                      uint32_t heads, uint32_t kvheads) {
  uint32_t hd = dim / heads, grp = heads / kvheads, kvdim = kvheads * hd;
  long long total = (long long)seq * dim;
#pragma omp parallel for schedule(static)
  for (long long idx = 0; idx < total; idx++) {
    uint32_t i = (uint32_t)(idx / dim), c = (uint32_t)(idx % dim);
    uint32_t h = c / hd, t = c % hd;
    const float *p = P + (size_t)h * seq * seq + (size_t)i * seq;
    const float *v = V + (size_t)(h / grp) * hd + t;
    float acc = 0.0f;
    for (uint32_t j = 0; j < seq; j++) acc = acc + p[j] * v[(size_t)j * kvdim];
    C[idx] = acc;
  }
}

/* The reference's OpSDot: four signed int8 lanes, products summed in int32. */
static int32_t sdot4(uint32_t a, uint32_t b) {
  int32_t s = 0;
  for (int l = 0; l < 4; l++) s += (int32_t)(int8_t)(a >> (8 * l)) * (int32_t)(int8_t)(b >> (8 * l));
  return s;
}

/* :592-602 (dp4a-dot) */
void nlo_dp4a_dot(const float *ALO, const float *AHI, const float *BLO, const float *BHI,
                  float *OUT, uint32_t n) {
  for (uint32_t i = 0; i < n; i++) {
    uint32_t a = u_of(ALO[i]) + u_of(AHI[i]) * 65536u, b = u_of(BLO[i]) + u_of(BHI[i]) * 65536u;
    OUT[i] = (float)sdot4(a, b);
  }
}

/* :606-620 (bitlinear-dp4a) */
void nlo_bitlinear_dp4a(const float *ALO, const float *AHI, const float *WLO, const float *WHI,
                        const float *BIAS, const float *BETA, const float *GAMMA, float *Y,
                        uint32_t seq, uint32_t out, uint32_t ng) {
  long long total = (long long)seq * out;
#pragma omp parallel for schedule(static)
  for (long long idx = 0; idx < total; idx++) {
    uint32_t s = (uint32_t)(idx / out), o = (uint32_t)(idx % out);
    size_t ab = (size_t)s * ng, wb = (size_t)o * ng;
    int32_t acc = 0;
    for (uint32_t g = 0; g < ng; g++) {
      uint32_t a = u_of(ALO[ab + g]) + u_of(AHI[ab + g]) * 65536u;
      uint32_t w = u_of(WLO[wb + g]) + u_of(WHI[wb + g]) * 65536u;
      acc += sdot4(a, w);
    }
    Y[idx] = BIAS[o] + (BETA[0] * GAMMA[s]) * (float)acc;
  }
}

/* :792-810 (dp4a-rows-t): the WP words are carried bit-cast in f32 */
void nlo_dp4a_rows_t(const float *WP, const float *BETA, const float *G, float *X, uint32_t out,
                     uint32_t cols, uint32_t ng, uint32_t seq) {
  long long total = (long long)seq * cols;
#pragma omp parallel for schedule(static)
  for (long long idx = 0; idx < total; idx++) {
    uint32_t p = (uint32_t)(idx / cols), i = (uint32_t)(idx % cols);
    uint32_t word = i / 4, lane = i % 4;
    const float *g = G + (size_t)p * out;
    float acc = 0.0f;
    for (uint32_t o = 0; o < out; o++) {
      uint32_t w;
      memcpy(&w, WP + (size_t)o * ng + word, 4);
      uint32_t b = (w >> (8 * lane)) & 255u;
      float sv = (float)((b + 128u) % 256u) - 128.0f;
      acc = acc + sv * (BETA[o] * g[o]);
    }
    X[idx] = acc;
  }
}

/* :828-845 (rmsnorm-heads), eps 1e-6 */
void nlo_rmsnorm_heads(const float *X, const float *G, float *Y, uint32_t seq, uint32_t nheads,
                       uint32_t hd) {
  long long rows = (long long)seq * nheads;
#pragma omp parallel for schedule(static)
  for (long long r = 0; r < rows; r++) {
    const float *x = X + (size_t)r * hd;
    float ss = 0.0f;
    for (uint32_t i = 0; i < hd; i++) ss = ss + x[i] * x[i];
    float inv = 1.0f / sqrtf(ss / (float)hd + 0.000001f);
    for (uint32_t j = 0; j < hd; j++) Y[(size_t)r * hd + j] = (x[j] * inv) * G[j];
  }
}

/* :1290-1303 (rope-apply) */
void nlo_rope_apply(const float *X, const float *CO, const float *SI, const float *SG, float *C,
                    uint32_t seq, uint32_t dim, uint32_t heads) {
  uint32_t hd = dim / heads, half = hd / 2;
  for (uint32_t p = 0; p < seq; p++)
    for (uint32_t h = 0; h < heads; h++)
      for (uint32_t m = 0; m < half; m++) {
        size_t ci = (size_t)p * half + m;
        float cc = CO[ci], ss = SI[ci] * SG[0];
        size_t i0 = (size_t)p * dim + (size_t)h * hd + 2 * m;
        float a0 = X[i0], a1 = X[i0 + 1];
        C[i0] = a0 * cc - a1 * ss;
        C[i0 + 1] = a0 * ss + a1 * cc;
      }
}

/* :1306-1312 (silu) */
void nlo_silu(const float *X, float *C, uint32_t n) {
  for (uint32_t i = 0; i < n; i++) {
    float x = X[i];
    float sg = 1.0f / (1.0f + expf(0.0f - x));
    C[i] = x * sg;
  }
}

/* :1365-1372 (scale-rows) */
void nlo_scale_rows(const float *Y, const float *S, float *C, uint32_t M, uint32_t N) {
  for (uint64_t idx = 0; idx < (uint64_t)M * N; idx++) C[idx] = Y[idx] * S[idx / N];
}

/* :496-503 (sumsq-acc) and :516-526 (absmean-acc): serial f32 sums, as the
 * reference's single thread does them. */
void nlo_sumsq_acc(const float *G, float *ACC, uint32_t n) {
  float acc = 0.0f;
  for (uint32_t i = 0; i < n; i++) acc = acc + G[i] * G[i];
  ACC[0] = ACC[0] + acc;
}
void nlo_absmean_acc(const float *G, float *ACC, uint32_t n) {
  float acc = 0.0f;
  for (uint32_t i = 0; i < n; i++) acc = acc + (G[i] < 0.0f ? 0.0f - G[i] : G[i]);
  ACC[0] = ACC[0] + acc;
}

/* :505-512 (clip-scale) */
void nlo_clip_scale(const float *GSQ, const float *CFG, float *SCALE) {
  float s = CFG[0] / sqrtf(GSQ[0] + 1.0e-12f);
  SCALE[0] = 1.0f;
  if (s < 1.0f) SCALE[0] = s;
}

/* :529-548 (quant-act) */
void nlo_quant_act(const float *X, float *XQ, uint32_t seq, uint32_t cols) {
  for (uint32_t row = 0; row < seq; row++) {
    const float *x = X + (size_t)row * cols;
    float amax = 0.0f;
    for (uint32_t c = 0; c < cols; c++) {
      float av = x[c] < 0.0f ? 0.0f - x[c] : x[c];
      if (av > amax) amax = av;
    }
    float gamma = amax / 127.0f;
    for (uint32_t c = 0; c < cols; c++) {
      float xq = 0.0f;
      if (gamma > 0.0f) {
        float q = x[c] / gamma, sgn = 1.0f, aq = q;
        if (q < 0.0f) { sgn = -1.0f; aq = 0.0f - q; }
        uint32_t ri = (uint32_t)(aq + 0.5f);
        float rf = (float)ri;
        if (rf > 127.0f) rf = 127.0f;
        xq = gamma * (sgn * rf);
      }
      XQ[(size_t)row * cols + c] = xq;
    }
  }
}

static int trit_q(float w, float beta) {
  if (!(beta > 0.0f)) return 0;
  float q = w / beta;
  return q >= 0.5f ? 1 : (q <= -0.5f ? -1 : 0);
}

/* :550-561 (quant-w) */
void nlo_quant_w(const float *W, const float *S, float *WQ, uint32_t n) {
  float beta = S[0] / (float)n;
  for (uint32_t i = 0; i < n; i++) WQ[i] = beta * (float)trit_q(W[i], beta);
}

/* The on-device repacking of nl_upload_file_ternary: quant-w's rule with
 * beta = mean |W| per tensor or per row, the sum of |W| taken in f64 (as the
 * device does; the reference's absmean-acc sums serially in f32), written as
 * packed two-bit codes (01 -> +1, 11 -> -1, 00 -> 0) and per-row scales. */
void nlo_quant_w_pack(const float *W, uint32_t rows, uint32_t cols, int per_row, uint32_t *WP,
                      float *S) {
  uint32_t wng = (cols + 15) / 16;
  double total = 0.0;
  double *rs = (double *)malloc(sizeof(double) * (rows ? rows : 1));
  for (uint32_t o = 0; o < rows; o++) {
    double s = 0.0;
    for (uint32_t c = 0; c < cols; c++) s += fabs((double)W[(size_t)o * cols + c]);
    rs[o] = s;
    total += s;
  }
  float tbeta = (float)(total / ((double)rows * cols));
  for (uint32_t o = 0; o < rows; o++) {
    float beta = per_row ? (float)(rs[o] / (double)cols) : tbeta;
    S[o] = beta;
    for (uint32_t wi = 0; wi < wng; wi++) {
      uint32_t word = 0;
      for (uint32_t f = 0; f < 16; f++) {
        uint32_t c = 16 * wi + f;
        int t = c < cols ? trit_q(W[(size_t)o * cols + c], beta) : 0;
        word |= (uint32_t)(t == 1 ? 1 : (t == -1 ? 3 : 0)) << (2 * f);
      }
      WP[(size_t)o * wng + wi] = word;
    }
  }
  free(rs);
}

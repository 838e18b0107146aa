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

/* ---- the training-side operators (kernels.el line numbers per function) ---- */
static float sigm_o(float x) { return 1.0f / (1.0f + expf(0.0f - x)); }

/* :132-140 transpose */
void nlo_transpose(const float *A, float *C, uint32_t R, uint32_t Co) {
  for (uint64_t idx = 0; idx < (uint64_t)R * Co; idx++) C[(idx % Co) * R + idx / Co] = A[idx];
}
/* :157-164 slice-cols, :166-173 set-cols (D in place) */
void nlo_slice_cols(const float *A, float *C, uint32_t seq, uint32_t dim, uint32_t hd, uint32_t c0) {
  for (uint64_t idx = 0; idx < (uint64_t)seq * hd; idx++) C[idx] = A[(idx / hd) * dim + c0 + idx % hd];
}
void nlo_set_cols(float *D, const float *S, uint32_t seq, uint32_t dim, uint32_t hd, uint32_t c0) {
  for (uint64_t idx = 0; idx < (uint64_t)seq * hd; idx++) D[(idx / hd) * dim + c0 + idx % hd] = S[idx];
}
/* :195-204 silu-mul-bwd */
void nlo_silu_mul_bwd(const float *G, const float *A, const float *B, float *DA, float *DB, uint32_t n) {
  for (uint32_t i = 0; i < n; i++) {
    float a = A[i], sg = sigm_o(a), g = G[i];
    DA[i] = (g * B[i]) * (sg * (1.0f + a * (1.0f - sg)));
    DB[i] = g * (a * sg);
  }
}
/* :1314-1320 silu-bwd */
void nlo_silu_bwd(const float *G, const float *X, float *D, uint32_t n) {
  for (uint32_t i = 0; i < n; i++) {
    float x = X[i], sg = sigm_o(x);
    D[i] = G[i] * (sg * (1.0f + x * (1.0f - sg)));
  }
}
/* :473-485 gelu-bwd */
void nlo_gelu_bwd(const float *G, const float *H, float *D, uint32_t n) {
  for (uint32_t i = 0; i < n; i++) {
    float x = H[i];
    float inner = 0.7978845608f * (x + 0.044715f * (x * (x * x)));
    float e = expf(2.0f * inner);
    float th = (e - 1.0f) / (e + 1.0f);
    float sech2 = 1.0f - th * th;
    float dudx = 0.7978845608f * (1.0f + 0.134145f * (x * x));
    float gp = 0.5f * (1.0f + th) + 0.5f * (x * (sech2 * dudx));
    D[i] = G[i] * gp;
  }
}
/* :455-460 sub-scale, :488-493 sgd (W in place) */
void nlo_sub_scale(const float *A, const float *B, const float *S, float *C, uint32_t n) {
  for (uint32_t i = 0; i < n; i++) C[i] = (A[i] - B[i]) * S[0];
}
void nlo_sgd(float *W, const float *G, const float *L, const float *S, uint32_t n) {
  for (uint32_t i = 0; i < n; i++) W[i] = W[i] - (L[0] * S[0]) * G[i];
}
/* :1338-1351 adam (W, M, V in place) */
void nlo_adam(float *W, const float *G, float *M, float *V, const float *H, const float *S,
              uint32_t n) {
  for (uint32_t i = 0; i < n; i++) {
    float g = S[0] * G[i], b1 = H[1], b2 = H[2];
    float m = b1 * M[i] + (1.0f - b1) * g;
    float v = b2 * V[i] + (1.0f - b2) * (g * g);
    M[i] = m;
    V[i] = v;
    W[i] = W[i] - H[0] * (m / (sqrtf(v) + H[3]));
  }
}
/* :463-470 colsum, :1280-1287 rmsnorm-dgamma */
void nlo_colsum(const float *G, float *D, uint32_t M, uint32_t N) {
  for (uint32_t o = 0; o < N; o++) {
    float acc = 0.0f;
    for (uint32_t r = 0; r < M; r++) acc = acc + G[(uint64_t)r * N + o];
    D[o] = acc;
  }
}
void nlo_rmsnorm_dgamma(const float *DY, const float *X, const float *S, float *DG, uint32_t M,
                        uint32_t N) {
  for (uint32_t j = 0; j < N; j++) {
    float acc = 0.0f;
    for (uint32_t r = 0; r < M; r++) {
      uint64_t k = (uint64_t)r * N + j;
      acc = acc + (DY[k] * X[k]) * S[r];
    }
    DG[j] = acc;
  }
}
/* :1267-1278 rmsnorm-dx */
void nlo_rmsnorm_dx(const float *DY, const float *X, const float *S, const float *G, float *DX,
                    uint32_t M, uint32_t N) {
  for (uint32_t r = 0; r < M; r++) {
    uint64_t base = (uint64_t)r * N;
    float is = S[r], a = 0.0f;
    for (uint32_t k = 0; k < N; k++) a = a + (DY[base + k] * G[k]) * X[base + k];
    float is3 = ((is * is) * is) / (float)N;
    for (uint32_t j = 0; j < N; j++)
      DX[base + j] = (is * DY[base + j]) * G[j] - (is3 * X[base + j]) * a;
  }
}
/* :1327-1335 softmax-bwd, :1373-1381 rowdot */
void nlo_softmax_bwd(const float *P, const float *G, float *DS, uint32_t M, uint32_t N) {
  for (uint32_t r = 0; r < M; r++) {
    uint64_t base = (uint64_t)r * N;
    float dot = 0.0f;
    for (uint32_t k = 0; k < N; k++) dot = dot + P[base + k] * G[base + k];
    for (uint32_t j = 0; j < N; j++) DS[base + j] = P[base + j] * (G[base + j] - dot);
  }
}
void nlo_rowdot(const float *G, const float *Y, float *D, uint32_t M, uint32_t N) {
  for (uint32_t r = 0; r < M; r++) {
    float acc = 0.0f;
    for (uint32_t j = 0; j < N; j++) acc = acc + G[(uint64_t)r * N + j] * Y[(uint64_t)r * N + j];
    D[r] = acc;
  }
}
/* :1407-1422 ce-grad-idx (IDX != 0, T = target indices) and :1425-1439 ce-grad (T one-hot) */
void nlo_ce_grad(const float *LG, const float *T, float *G, uint32_t M, uint32_t V, int idx) {
  for (uint32_t r = 0; r < M; r++) {
    uint64_t base = (uint64_t)r * V;
    float mx = LG[base];
    for (uint32_t j = 0; j < V; j++) if (LG[base + j] > mx) mx = LG[base + j];
    float s = 0.0f;
    for (uint32_t j = 0; j < V; j++) s = s + expf(LG[base + j] - mx);
    float invm = 1.0f / (float)M;
    uint32_t tgt = idx ? u_of(T[r]) : 0u;
    for (uint32_t j = 0; j < V; j++) {
      float sub = idx ? (j == tgt ? 1.0f : 0.0f) : T[base + j];
      G[base + j] = (expf(LG[base + j] - mx) / s - sub) * invm;
    }
  }
}
/* :1353-1363 topk-mask */
void nlo_topk_mask(const float *LG, float *MK, uint32_t M, uint32_t E, uint32_t K) {
  for (uint64_t idx = 0; idx < (uint64_t)M * E; idx++) {
    uint64_t base = idx / E * E;
    uint32_t cnt = 0;
    for (uint32_t j = 0; j < E; j++) if (LG[base + j] > LG[idx]) cnt++;
    MK[idx] = cnt < K ? 0.0f : -1.0e30f;
  }
}
/* :1395-1405 embed-bwd */
void nlo_embed_bwd(const float *TOK, const float *GX, float *DW, uint32_t seq, uint32_t dim,
                   uint32_t vocab) {
  for (uint64_t idx = 0; idx < (uint64_t)vocab * dim; idx++) {
    uint32_t tt = (uint32_t)(idx / dim), j = (uint32_t)(idx % dim);
    float acc = 0.0f;
    for (uint32_t i = 0; i < seq; i++)
      if (u_of(TOK[i]) == tt) acc = acc + GX[(uint64_t)i * dim + j];
    DW[idx] = acc;
  }
}
/* :569-576 gather-spike, :578-585 scatter-spike (POOL in place); indices past
 * the pool are skipped */
void nlo_gather_spike(const float *TABLE, const float *POOL, float *OUT, uint32_t n, uint32_t bs,
                      uint64_t pool_words) {
  for (uint64_t idx = 0; idx < (uint64_t)n * bs; idx++) {
    uint64_t src = (uint64_t)u_of(TABLE[idx / bs]) * bs + idx % bs;
    if (src < pool_words) OUT[idx] = POOL[src];
  }
}
void nlo_scatter_spike(const float *TABLE, const float *SRC, float *POOL, uint32_t n, uint32_t bs,
                       uint64_t pool_words) {
  for (uint64_t idx = 0; idx < (uint64_t)n * bs; idx++) {
    uint64_t dst = (uint64_t)u_of(TABLE[idx / bs]) * bs + idx % bs;
    if (dst < pool_words) POOL[dst] = SRC[idx];
  }
}
/* :673-698 gdn-step (S in place) */
void nlo_gdn_step(float *S, const float *Q, const float *K, const float *V, const float *G,
                  const float *B, float *OUT, uint32_t nv, uint32_t dk, uint32_t dv, uint32_t t) {
  for (uint64_t idx = 0; idx < (uint64_t)nv * dv; idx++) {
    uint32_t h = (uint32_t)(idx / dv), j = (uint32_t)(idx % dv);
    uint64_t sb = (uint64_t)h * dk * dv + j, qb = ((uint64_t)t * nv + h) * dk;
    uint64_t vb = ((uint64_t)t * nv + h) * dv + j;
    float gv = G[(uint64_t)t * nv + h], bv = B[(uint64_t)t * nv + h], mem = 0.0f;
    for (uint32_t i = 0; i < dk; i++) {
      uint64_t p = sb + (uint64_t)i * dv;
      float sv = S[p] * gv;
      S[p] = sv;
      mem = mem + sv * K[qb + i];
    }
    float d = bv * (V[vb] - mem), o = 0.0f;
    for (uint32_t i = 0; i < dk; i++) {
      uint64_t p = sb + (uint64_t)i * dv;
      float sv = S[p] + K[qb + i] * d;
      S[p] = sv;
      o = o + sv * Q[qb + i];
    }
    OUT[vb] = o;
  }
}
/* :237-290 attention backward: attn-sc-dq (DS K DQ), attn-sc-dk (DS Q DK),
 * attn-ctx-dp (DC V DP), attn-ctx-dv (DC P DV) */
void nlo_attn_sc_dq(const float *DS, const float *K, float *DQ, uint32_t seq, uint32_t dim,
                    uint32_t heads, uint32_t kvheads) {
  uint32_t hd = dim / heads, grp = heads / kvheads, kvdim = kvheads * hd;
  for (uint64_t idx = 0; idx < (uint64_t)seq * dim; idx++) {
    uint32_t i = (uint32_t)(idx / dim), c = (uint32_t)(idx % dim), h = c / hd, t = c % hd;
    uint64_t sb = (uint64_t)h * seq * seq + (uint64_t)i * seq;
    float acc = 0.0f;
    for (uint32_t j = 0; j < seq; j++) acc = acc + DS[sb + j] * K[(uint64_t)j * kvdim + (h / grp) * hd + t];
    DQ[idx] = acc * (1.0f / sqrtf((float)hd));
  }
}
void nlo_attn_sc_dk(const float *DS, const float *Q, float *DK, uint32_t seq, uint32_t dim,
                    uint32_t heads, uint32_t kvheads) {
  uint32_t hd = dim / heads, grp = heads / kvheads, kvdim = kvheads * hd;
  for (uint64_t idx = 0; idx < (uint64_t)seq * kvdim; idx++) {
    uint32_t j = (uint32_t)(idx / kvdim), rem = (uint32_t)(idx % kvdim), kvh = rem / hd, t = rem % hd;
    float acc = 0.0f;
    for (uint32_t hh = 0; hh < grp; hh++) {
      uint32_t h = kvh * grp + hh;
      for (uint32_t i = 0; i < seq; i++)
        acc = acc + DS[(uint64_t)h * seq * seq + j + (uint64_t)i * seq] * Q[(uint64_t)i * dim + h * hd + t];
    }
    DK[idx] = acc * (1.0f / sqrtf((float)hd));
  }
}
void nlo_attn_ctx_dp(const float *DC, const float *V, float *DP, uint32_t seq, uint32_t dim,
                     uint32_t heads, uint32_t kvheads) {
  uint32_t hd = dim / heads, grp = heads / kvheads, kvdim = kvheads * hd;
  for (uint64_t idx = 0; idx < (uint64_t)heads * seq * seq; idx++) {
    uint32_t h = (uint32_t)(idx / ((uint64_t)seq * seq));
    uint64_t rem = idx % ((uint64_t)seq * seq);
    uint32_t i = (uint32_t)(rem / seq), j = (uint32_t)(rem % seq);
    float acc = 0.0f;
    for (uint32_t t = 0; t < hd; t++)
      acc = acc + DC[(uint64_t)i * dim + h * hd + t] * V[(uint64_t)j * kvdim + (h / grp) * hd + t];
    DP[idx] = acc;
  }
}
void nlo_attn_ctx_dv(const float *DC, const float *P, float *DV, uint32_t seq, uint32_t dim,
                     uint32_t heads, uint32_t kvheads) {
  uint32_t hd = dim / heads, grp = heads / kvheads, kvdim = kvheads * hd;
  for (uint64_t idx = 0; idx < (uint64_t)seq * kvdim; idx++) {
    uint32_t j = (uint32_t)(idx / kvdim), rem = (uint32_t)(idx % kvdim), kvh = rem / hd, t = rem % hd;
    float acc = 0.0f;
    for (uint32_t hh = 0; hh < grp; hh++) {
      uint32_t h = kvh * grp + hh;
      for (uint32_t i = 0; i < seq; i++)
        acc = acc + DC[(uint64_t)i * dim + h * hd + t] * P[(uint64_t)h * seq * seq + j + (uint64_t)i * seq];
    }
    DV[idx] = acc;
  }
}
/* :1144-1180 tree-attn */
void nlo_tree_attn(const float *Q, const float *CK, const float *CV, const float *NK,
                   const float *NV, const float *PAR, const float *LEN, float *C, uint32_t M,
                   uint32_t dim, uint32_t heads, uint32_t kvheads, uint32_t maxdepth) {
  uint32_t hd = dim / heads, grp = heads / kvheads, kvdim = kvheads * hd;
  float coef = 1.0f / sqrtf((float)hd);
  uint32_t L = u_of(LEN[0]);
  for (uint64_t idx = 0; idx < (uint64_t)M * dim; idx++) {
    uint32_t i = (uint32_t)(idx / dim), c = (uint32_t)(idx % dim), h = c / hd, t = c % hd,
             kvh = h / grp;
    const float *q = Q + (uint64_t)i * dim + h * hd;
    float mx = -1.0e30f;
#define NLO_SCORE(KP, KB, OUTV)                                   \
    do {                                                          \
      float acc_ = 0.0f;                                          \
      for (uint32_t tt = 0; tt < hd; tt++) acc_ = acc_ + q[tt] * (KP)[(KB) + tt]; \
      OUTV = acc_ * coef;                                         \
    } while (0)
    for (uint32_t j = 0; j < L; j++) {
      float s;
      NLO_SCORE(CK, (uint64_t)j * kvdim + kvh * hd, s);
      if (s > mx) mx = s;
    }
    uint32_t cur = i;
    for (uint32_t d = 0; d < maxdepth && cur < M; d++) {
      float s;
      NLO_SCORE(NK, (uint64_t)cur * kvdim + kvh * hd, s);
      if (s > mx) mx = s;
      cur = u_of(PAR[cur]);
    }
    float z = 0.0f, ctx = 0.0f;
    for (uint32_t j = 0; j < L; j++) {
      uint64_t kb = (uint64_t)j * kvdim + kvh * hd;
      float s;
      NLO_SCORE(CK, kb, s);
      float e = expf(s - mx);
      z = z + e;
      ctx = ctx + e * CV[kb + t];
    }
    cur = i;
    for (uint32_t d = 0; d < maxdepth && cur < M; d++) {
      uint64_t kb = (uint64_t)cur * kvdim + kvh * hd;
      float s;
      NLO_SCORE(NK, kb, s);
      float e = expf(s - mx);
      z = z + e;
      ctx = ctx + e * NV[kb + t];
      cur = u_of(PAR[cur]);
    }
#undef NLO_SCORE
    C[idx] = ctx / z;
  }
}

/* nl_oracle_decoder.c -- CPU model of the ternary decoder.
 *
 * TEST INFRASTRUCTURE ONLY: the parity checker of the library's decoder and
 * the CPU baseline of its decode throughput.  No product code calls it.
 *
 * The reference repository holds this model's kernels but not the model, so
 * the composition is restated from the conventions its kernels document,
 * with each step done by the restated kernel of nl_oracle.c where one
 * exists: embed-gather (lisp/nelisp-gpu-kernels.el:1385-1392), RMSNorm as
 * rmsnorm-istd/-fwd (:1250-1265) with eps a parameter, the ternary linears as
 * ternary-rows (:713-746) with the row scale in every block, half-split RoPE
 * as rope-half (:857-882) at the absolute position, the KV cache as
 * cache-append-b (:358-365), attention as decode-attn-b (:368-390), SwiGLU as
 * silu-mul (:187-193), residuals as add2 (:816-821), the tied LM head as a
 * sequential f32 dot product, greedy argmax taking the lowest index on ties.
 *
 * Weights are regenerated from the seed with the same counter-based hash
 * the library uses (splitmix64 finaliser over (seed, tensor, element)),
 * restated here so the checker does not share code with what it checks.
 */
#define _POSIX_C_SOURCE 199309L   /* clock_gettime */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

#include "nl_oracle.h"

typedef struct {
  uint32_t hidden, layers, heads, kv_heads, head_dim, ffn, vocab, max_batch, max_seq;
  float rms_eps, rope_base;
  uint64_t seed;
} nlo_decoder_config;

static uint64_t mix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}
static uint64_t tkey(uint64_t seed, uint64_t t) {
  return mix64(seed ^ mix64(t * 0xD1B54A32D192ED03ull + 1u));
}
static uint32_t r24(uint64_t key, uint64_t i) { return (uint32_t)(mix64(key ^ i) >> 40); }
static float unit(uint64_t key, uint64_t i) { return (float)r24(key, i) * (1.0f / 16777216.0f); }
static int trit(uint64_t key, uint64_t i) { return (int)((r24(key, i) * 3u) >> 24) - 1; }

enum { WQ = 0, WK, WV, WO, WGATE, WUP, WDOWN, SQ, SK, SV, SO, SGATE, SUP, SDOWN, GATTN, GFFN };
#define T_EMBED 1000000u
#define T_FINAL 1000001u

/* Rows [r0, r0+rows) of a [* x K] ternary tensor, two-bit packed. */
static void pack_rows(uint32_t *W, uint64_t key, uint32_t rows, uint32_t K) {
  uint32_t wng = (K + 15) / 16;
#pragma omp parallel for schedule(static)
  for (long long r = 0; r < (long long)rows; r++)
    for (uint32_t w = 0; w < wng; w++) {
      uint32_t word = 0;
      for (uint32_t f = 0; f < 16 && 16 * w + f < K; f++) {
        int t = trit(key, (uint64_t)r * K + 16 * w + f);
        word |= (uint32_t)(t == 1 ? 1 : (t == -1 ? 3 : 0)) << (2 * f);
      }
      W[(size_t)r * wng + w] = word;
    }
}
static void scales(float *S, uint64_t key, uint32_t n, uint32_t K) {
  float rs = (float)(1.0 / sqrt(2.0 * (double)K / 3.0));
  for (uint32_t i = 0; i < n; i++) {
    float u = unit(key, i);
    float a = 0.5f + u;
    S[i] = a * rs;
  }
}
static void gains(float *G, uint64_t key, uint32_t n) {
  for (uint32_t i = 0; i < n; i++) {
    float u = unit(key, i);
    float h = 0.5f * u;
    G[i] = 0.75f + h;
  }
}

static void rmsnorm(const float *h, const float *g, float *x, uint32_t B, uint32_t H, float eps) {
  for (uint32_t b = 0; b < B; b++) {
    float ss = 0.0f;
    for (uint32_t i = 0; i < H; i++) {
      float v = h[(size_t)b * H + i];
      float sq = v * v;
      ss = ss + sq;
    }
    float mean = ss / (float)H;
    float rinv = 1.0f / sqrtf(mean + eps);
    for (uint32_t i = 0; i < H; i++) {
      float xs = h[(size_t)b * H + i] * rinv;
      x[(size_t)b * H + i] = xs * g[i];
    }
  }
}

typedef struct {
  uint32_t *wq, *wk, *wv, *wo, *wg, *wu, *wd;
  float *sq, *sk, *sv, *so, *sg, *su, *sd, *ga, *gf;
} Lw;

/* The model's weights and the activations of one position. */
typedef struct {
  Lw *L;
  float *E, *gfin;
  float *ck, *cv;           /* [layers][B][npos][kvd] */
  float *h, *x, *q, *k, *v, *qr, *kr, *ctx, *o, *g, *u, *a, *lg;
  uint32_t B, npos;
} Model;

static void model_free(const nlo_decoder_config *c, Model *M) {
  for (uint32_t l = 0; l < c->layers; l++) {
    Lw *W = &M->L[l];
    free(W->wq); free(W->wk); free(W->wv); free(W->wo); free(W->wg); free(W->wu);
    free(W->wd); free(W->sq); free(W->sk); free(W->sv); free(W->so); free(W->sg);
    free(W->su); free(W->sd); free(W->ga); free(W->gf);
  }
  free(M->L); free(M->E); free(M->gfin); free(M->ck); free(M->cv); free(M->h); free(M->x);
  free(M->q); free(M->k); free(M->v); free(M->qr); free(M->kr); free(M->ctx); free(M->o);
  free(M->g); free(M->u); free(M->a); free(M->lg);
}

static void model_init(const nlo_decoder_config *c, Model *M, uint32_t B, uint32_t npos) {
  const uint32_t H = c->hidden, hd = c->head_dim, nh = c->heads, kvh = c->kv_heads;
  const uint32_t F = c->ffn, V = c->vocab, qd = nh * hd, kvd = kvh * hd;
  M->B = B;
  M->npos = npos;
  M->L = (Lw *)calloc(c->layers, sizeof(Lw));
  for (uint32_t l = 0; l < c->layers; l++) {
    uint64_t T = (uint64_t)l * 16;
    Lw *W = &M->L[l];
    W->wq = malloc((size_t)qd * (H / 16) * 4);
    W->wk = malloc((size_t)kvd * (H / 16) * 4);
    W->wv = malloc((size_t)kvd * (H / 16) * 4);
    W->wo = malloc((size_t)H * ((qd + 15) / 16) * 4);
    W->wg = malloc((size_t)F * (H / 16) * 4);
    W->wu = malloc((size_t)F * (H / 16) * 4);
    W->wd = malloc((size_t)H * ((F + 15) / 16) * 4);
    pack_rows(W->wq, tkey(c->seed, T + WQ), qd, H);
    pack_rows(W->wk, tkey(c->seed, T + WK), kvd, H);
    pack_rows(W->wv, tkey(c->seed, T + WV), kvd, H);
    pack_rows(W->wo, tkey(c->seed, T + WO), H, qd);
    pack_rows(W->wg, tkey(c->seed, T + WGATE), F, H);
    pack_rows(W->wu, tkey(c->seed, T + WUP), F, H);
    pack_rows(W->wd, tkey(c->seed, T + WDOWN), H, F);
    W->sq = malloc((size_t)qd * 4); scales(W->sq, tkey(c->seed, T + SQ), qd, H);
    W->sk = malloc((size_t)kvd * 4); scales(W->sk, tkey(c->seed, T + SK), kvd, H);
    W->sv = malloc((size_t)kvd * 4); scales(W->sv, tkey(c->seed, T + SV), kvd, H);
    W->so = malloc((size_t)H * 4); scales(W->so, tkey(c->seed, T + SO), H, qd);
    W->sg = malloc((size_t)F * 4); scales(W->sg, tkey(c->seed, T + SGATE), F, H);
    W->su = malloc((size_t)F * 4); scales(W->su, tkey(c->seed, T + SUP), F, H);
    W->sd = malloc((size_t)H * 4); scales(W->sd, tkey(c->seed, T + SDOWN), H, F);
    W->ga = malloc((size_t)H * 4); gains(W->ga, tkey(c->seed, T + GATTN), H);
    W->gf = malloc((size_t)H * 4); gains(W->gf, tkey(c->seed, T + GFFN), H);
  }
  M->E = malloc((size_t)V * H * 4);
  {
    uint64_t k = tkey(c->seed, T_EMBED);
    float *E = M->E;
#pragma omp parallel for schedule(static)
    for (long long i = 0; i < (long long)V * H; i++) {
      float u = unit(k, (uint64_t)i);
      float t = 2.0f * u;
      E[i] = t - 1.0f;
    }
  }
  M->gfin = malloc((size_t)H * 4);
  gains(M->gfin, tkey(c->seed, T_FINAL), H);
  M->ck = calloc((size_t)c->layers * B * npos * kvd, 4);
  M->cv = calloc((size_t)c->layers * B * npos * kvd, 4);
  M->h = malloc((size_t)B * H * 4); M->x = malloc((size_t)B * H * 4);
  M->q = malloc((size_t)B * qd * 4); M->k = malloc((size_t)B * kvd * 4);
  M->v = malloc((size_t)B * kvd * 4);
  M->qr = malloc((size_t)B * qd * 4); M->kr = malloc((size_t)B * kvd * 4);
  M->ctx = malloc((size_t)B * qd * 4); M->o = malloc((size_t)B * H * 4);
  M->g = malloc((size_t)B * F * 4); M->u = malloc((size_t)B * F * 4);
  M->a = malloc((size_t)B * F * 4);
  M->lg = malloc((size_t)B * V * 4);
}

/* One position P for the B sequences whose tokens are TOK: every layer
 * (appending to the KV cache at P), then the LM head into M->lg [B x V]. */
static void model_position(const nlo_decoder_config *c, Model *M, uint32_t p, const int32_t *tok) {
  const uint32_t H = c->hidden, hd = c->head_dim, nh = c->heads, kvh = c->kv_heads;
  const uint32_t F = c->ffn, V = c->vocab, qd = nh * hd, kvd = kvh * hd;
  const uint32_t B = M->B, npos = M->npos;
  float *h = M->h, *x = M->x, *q = M->q, *k = M->k, *v = M->v, *qr = M->qr, *kr = M->kr;
  float *ctx = M->ctx, *o = M->o, *g = M->g, *u = M->u, *a = M->a;
  for (uint32_t b = 0; b < B; b++) memcpy(h + (size_t)b * H, M->E + (size_t)tok[b] * H, (size_t)H * 4);
  for (uint32_t l = 0; l < c->layers; l++) {
    const Lw *W = &M->L[l];
    rmsnorm(h, W->ga, x, B, H, c->rms_eps);
    nlo_ternary_gemv_rows(x, W->wq, W->sq, q, B, qd, H);
    nlo_ternary_gemv_rows(x, W->wk, W->sk, k, B, kvd, H);
    nlo_ternary_gemv_rows(x, W->wv, W->sv, v, B, kvd, H);
    /* rope-half at position p: the kernel's row index is the position, so
     * run it on a [p+1]-row buffer whose last row is this token. */
    for (uint32_t b = 0; b < B; b++) {
      for (uint32_t hh = 0; hh < nh + kvh; hh++) {
        const float *src = hh < nh ? q + (size_t)b * qd + (size_t)hh * hd
                                   : k + (size_t)b * kvd + (size_t)(hh - nh) * hd;
        float *dst = hh < nh ? qr + (size_t)b * qd + (size_t)hh * hd
                             : kr + (size_t)b * kvd + (size_t)(hh - nh) * hd;
        uint32_t half = hd / 2;
        for (uint32_t m = 0; m < half; m++) {
          float ex = (2.0f * (float)m) / (float)hd;
          float theta = (float)p / powf(c->rope_base, ex);
          float cc = cosf(theta), ss = sinf(theta);
          float a0 = src[m], a1 = src[m + half];
          float t0 = a0 * cc, t1 = a1 * ss, t2 = a1 * cc, t3 = a0 * ss;
          dst[m] = t0 - t1;
          dst[m + half] = t2 + t3;
        }
      }
    }
    float *ckl = M->ck + (size_t)l * B * npos * kvd, *cvl = M->cv + (size_t)l * B * npos * kvd;
    float posf = (float)p;
    nlo_cache_append_b(kr, &posf, ckl, B, kvd, npos);
    nlo_cache_append_b(v, &posf, cvl, B, kvd, npos);
    nlo_decode_attn_b(qr, ckl, cvl, &posf, ctx, B, qd, nh, kvh, npos);
    nlo_ternary_gemv_rows(ctx, W->wo, W->so, o, B, H, qd);
    nlo_add2(h, o, h, B * H);
    rmsnorm(h, W->gf, x, B, H, c->rms_eps);
    nlo_ternary_gemv_rows(x, W->wg, W->sg, g, B, F, H);
    nlo_ternary_gemv_rows(x, W->wu, W->su, u, B, F, H);
    nlo_silu_mul(g, u, a, B * F);
    nlo_ternary_gemv_rows(a, W->wd, W->sd, o, B, H, F);
    nlo_add2(h, o, h, B * H);
  }
  rmsnorm(h, M->gfin, x, B, H, c->rms_eps);
  const float *E = M->E;
  float *lg = M->lg;
#pragma omp parallel for schedule(static)
  for (long long idx = 0; idx < (long long)B * V; idx++) {
    uint32_t b = (uint32_t)(idx / V), row = (uint32_t)(idx % V);
    float acc = 0.0f;
    for (uint32_t i = 0; i < H; i++) {
      float pr = E[(size_t)row * H + i] * x[(size_t)b * H + i];
      acc = acc + pr;
    }
    lg[idx] = acc;
  }
}

/* One tensor of the CPU model's weights into OUT: per-layer tensor WHICH
 * (WQ .. GFFN, the library's tensor ids) of layer LAYER -- packed two-bit rows
 * of ceil(K/16) words for WQ .. WDOWN, f32 for the scales and gains -- or
 * the embedding (WHICH 16, f32 [vocab x hidden]) or the final gain (17).
 * Returns the number of 32-bit words written, 0 for a bad WHICH. */
uint64_t nlo_decoder_tensor(const nlo_decoder_config *c, uint32_t layer, uint32_t which,
                            void *out) {
  const uint32_t H = c->hidden, hd = c->head_dim, F = c->ffn;
  const uint32_t qd = c->heads * hd, kvd = c->kv_heads * hd;
  const uint64_t T = (uint64_t)layer * 16;
  uint32_t *W = (uint32_t *)out;
  float *S = (float *)out;
  switch (which) {
    case WQ: pack_rows(W, tkey(c->seed, T + WQ), qd, H); return (uint64_t)qd * ((H + 15) / 16);
    case WK: pack_rows(W, tkey(c->seed, T + WK), kvd, H); return (uint64_t)kvd * ((H + 15) / 16);
    case WV: pack_rows(W, tkey(c->seed, T + WV), kvd, H); return (uint64_t)kvd * ((H + 15) / 16);
    case WO: pack_rows(W, tkey(c->seed, T + WO), H, qd); return (uint64_t)H * ((qd + 15) / 16);
    case WGATE: pack_rows(W, tkey(c->seed, T + WGATE), F, H); return (uint64_t)F * ((H + 15) / 16);
    case WUP: pack_rows(W, tkey(c->seed, T + WUP), F, H); return (uint64_t)F * ((H + 15) / 16);
    case WDOWN: pack_rows(W, tkey(c->seed, T + WDOWN), H, F); return (uint64_t)H * ((F + 15) / 16);
    case SQ: scales(S, tkey(c->seed, T + SQ), qd, H); return qd;
    case SK: scales(S, tkey(c->seed, T + SK), kvd, H); return kvd;
    case SV: scales(S, tkey(c->seed, T + SV), kvd, H); return kvd;
    case SO: scales(S, tkey(c->seed, T + SO), H, qd); return H;
    case SGATE: scales(S, tkey(c->seed, T + SGATE), F, H); return F;
    case SUP: scales(S, tkey(c->seed, T + SUP), F, H); return F;
    case SDOWN: scales(S, tkey(c->seed, T + SDOWN), H, F); return H;
    case GATTN: gains(S, tkey(c->seed, T + GATTN), H); return H;
    case GFFN: gains(S, tkey(c->seed, T + GFFN), H); return H;
    case 16: {
      const uint64_t k = tkey(c->seed, T_EMBED);
      for (uint64_t i = 0; i < (uint64_t)c->vocab * H; i++) S[i] = 2.0f * unit(k, i) - 1.0f;
      return (uint64_t)c->vocab * H;
    }
    case 17: gains(S, tkey(c->seed, T_FINAL), H); return H;
    default: return 0;
  }
}

static uint32_t argmax_row(const float *lg, uint32_t V) {
  uint32_t best = 0;
  for (uint32_t r = 1; r < V; r++)
    if (lg[r] > lg[best]) best = r;
  return best;
}

int nlo_decoder_generate(const nlo_decoder_config *c, uint32_t B, uint32_t P,
                         const int32_t *prompt, uint32_t steps, int32_t *out_tokens,
                         float *logits) {
  const uint32_t V = c->vocab;
  const uint32_t npos = P + steps - 1;
  Model M;
  model_init(c, &M, B, npos);
  int32_t *tok = malloc((size_t)B * 4);
  for (uint32_t b = 0; b < B; b++) tok[b] = prompt[(size_t)b * P];
  for (uint32_t p = 0; p < npos; p++) {
    model_position(c, &M, p, tok);
    if (logits) memcpy(logits + (size_t)p * B * V, M.lg, (size_t)B * V * 4);
    for (uint32_t b = 0; b < B; b++) {
      uint32_t best = argmax_row(M.lg + (size_t)b * V, V);
      if (p + 1 < P) {
        tok[b] = prompt[(size_t)b * P + p + 1];
      } else {
        tok[b] = (int32_t)best;
        out_tokens[(size_t)b * steps + (p + 1 - P)] = (int32_t)best;
      }
    }
  }
  model_free(c, &M);
  free(tok);
  return 0;
}

/* The CPU baseline of decode throughput at a given context: after the
 * weights are generated, rows 0..CTX-1 of every layer's KV cache are filled
 * with seeded values in [-1, 1) (standing in for a prefilled prompt: the
 * per-position work does not depend on what the rows hold), then STEPS
 * greedy positions CTX .. CTX+STEPS-1 are decoded for B sequences with the
 * arithmetic of nlo_decoder_generate.  Returns the wall-clock seconds of
 * those positions only (weight generation excluded), or a negative value on
 * a bad argument. */
double nlo_decoder_time_positions(const nlo_decoder_config *c, uint32_t B, uint32_t ctx,
                                  uint32_t steps) {
  if (B == 0 || steps == 0) return -1.0;
  const uint32_t kvd = c->kv_heads * c->head_dim, V = c->vocab;
  const uint32_t npos = ctx + steps;
  Model M;
  model_init(c, &M, B, npos);
  {
    const uint64_t kk = tkey(c->seed, 2000000u), kv = tkey(c->seed, 2000001u);
    float *ck = M.ck, *cv = M.cv;
    const long long per = (long long)npos * kvd;
#pragma omp parallel for schedule(static)
    for (long long lb = 0; lb < (long long)c->layers * B; lb++)
      for (long long i = 0; i < (long long)ctx * kvd; i++) {
        const uint64_t at = (uint64_t)(lb * per + i);
        ck[at] = 2.0f * unit(kk, at) - 1.0f;
        cv[at] = 2.0f * unit(kv, at) - 1.0f;
      }
  }
  int32_t *tok = malloc((size_t)B * 4);
  for (uint32_t b = 0; b < B; b++) tok[b] = (int32_t)((7u + 131u * b) % V);
  struct timespec t0, t1;
  clock_gettime(CLOCK_MONOTONIC, &t0);
  for (uint32_t p = ctx; p < npos; p++) {
    model_position(c, &M, p, tok);
    for (uint32_t b = 0; b < B; b++) tok[b] = (int32_t)argmax_row(M.lg + (size_t)b * V, V);
  }
  clock_gettime(CLOCK_MONOTONIC, &t1);
  model_free(c, &M);
  free(tok);
  return (double)(t1.tv_sec - t0.tv_sec) + 1e-9 * (double)(t1.tv_nsec - t0.tv_nsec);
}

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
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

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

int nlo_decoder_generate(const nlo_decoder_config *c, uint32_t B, uint32_t P,
                         const int32_t *prompt, uint32_t steps, int32_t *out_tokens,
                         float *logits) {
  const uint32_t H = c->hidden, hd = c->head_dim, nh = c->heads, kvh = c->kv_heads;
  const uint32_t F = c->ffn, V = c->vocab, qd = nh * hd, kvd = kvh * hd;
  const uint32_t npos = P + steps - 1;
  Lw *L = (Lw *)calloc(c->layers, sizeof(Lw));
  for (uint32_t l = 0; l < c->layers; l++) {
    uint64_t T = (uint64_t)l * 16;
    L[l].wq = malloc((size_t)qd * (H / 16) * 4);
    L[l].wk = malloc((size_t)kvd * (H / 16) * 4);
    L[l].wv = malloc((size_t)kvd * (H / 16) * 4);
    L[l].wo = malloc((size_t)H * ((qd + 15) / 16) * 4);
    L[l].wg = malloc((size_t)F * (H / 16) * 4);
    L[l].wu = malloc((size_t)F * (H / 16) * 4);
    L[l].wd = malloc((size_t)H * ((F + 15) / 16) * 4);
    pack_rows(L[l].wq, tkey(c->seed, T + WQ), qd, H);
    pack_rows(L[l].wk, tkey(c->seed, T + WK), kvd, H);
    pack_rows(L[l].wv, tkey(c->seed, T + WV), kvd, H);
    pack_rows(L[l].wo, tkey(c->seed, T + WO), H, qd);
    pack_rows(L[l].wg, tkey(c->seed, T + WGATE), F, H);
    pack_rows(L[l].wu, tkey(c->seed, T + WUP), F, H);
    pack_rows(L[l].wd, tkey(c->seed, T + WDOWN), H, F);
    L[l].sq = malloc((size_t)qd * 4); scales(L[l].sq, tkey(c->seed, T + SQ), qd, H);
    L[l].sk = malloc((size_t)kvd * 4); scales(L[l].sk, tkey(c->seed, T + SK), kvd, H);
    L[l].sv = malloc((size_t)kvd * 4); scales(L[l].sv, tkey(c->seed, T + SV), kvd, H);
    L[l].so = malloc((size_t)H * 4); scales(L[l].so, tkey(c->seed, T + SO), H, qd);
    L[l].sg = malloc((size_t)F * 4); scales(L[l].sg, tkey(c->seed, T + SGATE), F, H);
    L[l].su = malloc((size_t)F * 4); scales(L[l].su, tkey(c->seed, T + SUP), F, H);
    L[l].sd = malloc((size_t)H * 4); scales(L[l].sd, tkey(c->seed, T + SDOWN), H, F);
    L[l].ga = malloc((size_t)H * 4); gains(L[l].ga, tkey(c->seed, T + GATTN), H);
    L[l].gf = malloc((size_t)H * 4); gains(L[l].gf, tkey(c->seed, T + GFFN), H);
  }
  float *E = malloc((size_t)V * H * 4);
  {
    uint64_t k = tkey(c->seed, T_EMBED);
#pragma omp parallel for schedule(static)
    for (long long i = 0; i < (long long)V * H; i++) {
      float u = unit(k, (uint64_t)i);
      float t = 2.0f * u;
      E[i] = t - 1.0f;
    }
  }
  float *gfin = malloc((size_t)H * 4);
  gains(gfin, tkey(c->seed, T_FINAL), H);
  float *ck = calloc((size_t)c->layers * B * npos * kvd, 4);
  float *cv = calloc((size_t)c->layers * B * npos * kvd, 4);
  float *h = malloc((size_t)B * H * 4), *x = malloc((size_t)B * H * 4);
  float *q = malloc((size_t)B * qd * 4), *k = malloc((size_t)B * kvd * 4), *v = malloc((size_t)B * kvd * 4);
  float *qr = malloc((size_t)B * qd * 4), *kr = malloc((size_t)B * kvd * 4);
  float *ctx = malloc((size_t)B * qd * 4), *o = malloc((size_t)B * H * 4);
  float *g = malloc((size_t)B * F * 4), *u = malloc((size_t)B * F * 4), *a = malloc((size_t)B * F * 4);
  float *lg = malloc((size_t)B * V * 4);
  int32_t *tok = malloc((size_t)B * 4);
  for (uint32_t b = 0; b < B; b++) tok[b] = prompt[(size_t)b * P];
  uint32_t one = 0x3f800000u, rb;
  memcpy(&rb, &c->rope_base, 4);
  for (uint32_t p = 0; p < npos; p++) {
    for (uint32_t b = 0; b < B; b++) memcpy(h + (size_t)b * H, E + (size_t)tok[b] * H, (size_t)H * 4);
    for (uint32_t l = 0; l < c->layers; l++) {
      rmsnorm(h, L[l].ga, x, B, H, c->rms_eps);
      nlo_ternary_gemv_rows(x, L[l].wq, L[l].sq, q, B, qd, H);
      nlo_ternary_gemv_rows(x, L[l].wk, L[l].sk, k, B, kvd, H);
      nlo_ternary_gemv_rows(x, L[l].wv, L[l].sv, v, B, kvd, H);
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
      (void)one; (void)rb;
      float *ckl = ck + (size_t)l * B * npos * kvd, *cvl = cv + (size_t)l * B * npos * kvd;
      float posf = (float)p;
      nlo_cache_append_b(kr, &posf, ckl, B, kvd, npos);
      nlo_cache_append_b(v, &posf, cvl, B, kvd, npos);
      nlo_decode_attn_b(qr, ckl, cvl, &posf, ctx, B, qd, nh, kvh, npos);
      nlo_ternary_gemv_rows(ctx, L[l].wo, L[l].so, o, B, H, qd);
      nlo_add2(h, o, h, B * H);
      rmsnorm(h, L[l].gf, x, B, H, c->rms_eps);
      nlo_ternary_gemv_rows(x, L[l].wg, L[l].sg, g, B, F, H);
      nlo_ternary_gemv_rows(x, L[l].wu, L[l].su, u, B, F, H);
      nlo_silu_mul(g, u, a, B * F);
      nlo_ternary_gemv_rows(a, L[l].wd, L[l].sd, o, B, H, F);
      nlo_add2(h, o, h, B * H);
    }
    rmsnorm(h, gfin, x, B, H, c->rms_eps);
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
    if (logits) memcpy(logits + (size_t)p * B * V, lg, (size_t)B * V * 4);
    for (uint32_t b = 0; b < B; b++) {
      uint32_t best = 0;
      for (uint32_t r = 1; r < V; r++)
        if (lg[(size_t)b * V + r] > lg[(size_t)b * V + best]) best = r;
      if (p + 1 < P) {
        tok[b] = prompt[(size_t)b * P + p + 1];
      } else {
        tok[b] = (int32_t)best;
        out_tokens[(size_t)b * steps + (p + 1 - P)] = (int32_t)best;
      }
    }
  }
  for (uint32_t l = 0; l < c->layers; l++) {
    free(L[l].wq); free(L[l].wk); free(L[l].wv); free(L[l].wo); free(L[l].wg); free(L[l].wu);
    free(L[l].wd); free(L[l].sq); free(L[l].sk); free(L[l].sv); free(L[l].so); free(L[l].sg);
    free(L[l].su); free(L[l].sd); free(L[l].ga); free(L[l].gf);
  }
  free(L); free(E); free(gfin); free(ck); free(cv); free(h); free(x); free(q); free(k); free(v);
  free(qr); free(kr); free(ctx); free(o); free(g); free(u); free(a); free(lg); free(tok);
  return 0;
}

// k_train.cu -- the reference's remaining operators: glue copies, the
// training kernels (gradients and optimizers), the MoE top-k mask, the paged
// gather / scatter spikes, the gated-delta-net step and tree attention.
//
// Reference operators (lisp/nelisp-gpu-kernels.el):
//   transpose :132-140, slice-cols :157-164, set-cols :166-173,
//   silu-mul-bwd :195-204, sub-scale :455-460, colsum :463-470,
//   gelu-bwd :473-485, sgd :488-493, gather-spike :569-576,
//   scatter-spike :578-585, gdn-step :673-698, tree-attn :1144-1180,
//   rmsnorm-dx :1267-1278, rmsnorm-dgamma :1280-1287, silu-bwd :1314-1320,
//   softmax-bwd :1327-1335, adam :1338-1351, topk-mask :1353-1363,
//   rowdot :1373-1381, embed-bwd :1395-1405, ce-grad-idx :1407-1422,
//   ce-grad :1425-1439.
// Elementwise operators keep the reference's f32 operation order (no
// contraction), so they are bit-identical but for expf.  Row reductions run
// one warp per row (the sum order differs from the reference's single
// thread); column reductions and the per-output loops keep one thread per
// output in the reference's order.  Gathers through a table skip indices
// outside the pool (the reference would read or write past it).

#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include <initializer_list>

#include "nl_internal.h"

namespace nl {
namespace {

size_t no_scr(const OpArgs &) { return 0; }
unsigned blocks_for(uint64_t n, unsigned t = 256) { return grid_for(n, t, 148u * 64u); }
__device__ __forceinline__ uint32_t f2u(float v) { return v > 0.0f ? __float2uint_rz(v) : 0u; }
__device__ __forceinline__ float sigm(float x) { return 1.0f / (1.0f + expf(0.0f - x)); }

#define NL_FOR(n, limit)                                                                  \
  for (uint64_t idx = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < (n) && idx < (limit); \
       idx += (uint64_t)gridDim.x * blockDim.x)

// Elementwise operators: one launcher shape, an index functor each.
template <typename F>
__global__ void k_each(uint64_t n, uint64_t limit, F f) {
  NL_FOR(n, limit) f(idx);
}
template <typename F>
cudaError_t launch_each(const OpArgs &a, uint64_t n, F f) {
  if (!n) return cudaSuccess;
  k_each<<<blocks_for(n), 256, 0, a.stream>>>(n, invocations(a.groups, 64), f);
  count_launches(1);
  return cudaPeekAtLastError();
}

const char *need_all(const OpArgs &a, std::initializer_list<uint64_t> words) {
  uint32_t b = 0;
  for (uint64_t w : words) {
    const char *m = need_words(a, b++, w, "buffer");
    if (m) return m;
  }
  return nullptr;
}

// ---- glue ------------------------------------------------------------------------
const char *chk_transpose(const OpArgs &a) {
  const uint64_t n = (uint64_t)a.push[0] * a.push[1];
  return need_all(a, {n, n});
}
cudaError_t run_transpose(const OpArgs &a) {
  const float *A = (const float *)a.buf[0];
  float *C = (float *)a.buf[1];
  const uint32_t R = a.push[0], Co = a.push[1];
  return launch_each(a, (uint64_t)R * Co, [=] __device__(uint64_t idx) {
    const uint64_t i = idx / Co, j = idx % Co;
    C[j * R + i] = A[idx];
  });
}
const char *chk_cols(const OpArgs &a, bool set) {
  const uint64_t seq = a.push[0], dim = a.push[1], hd = a.push[2], c0 = a.push[3];
  if (seq && (c0 + hd > dim)) return fmt_msg("columns %u..%u past dim %u", a.push[3],
                                               a.push[3] + a.push[2], a.push[1]);
  return set ? need_all(a, {seq * dim, seq * hd}) : need_all(a, {seq * dim, seq * hd});
}
const char *chk_slice(const OpArgs &a) { return chk_cols(a, false); }
const char *chk_set(const OpArgs &a) { return chk_cols(a, true); }
cudaError_t run_slice(const OpArgs &a) {
  const float *A = (const float *)a.buf[0];
  float *C = (float *)a.buf[1];
  const uint32_t dim = a.push[1], hd = a.push[2], c0 = a.push[3];
  return launch_each(a, (uint64_t)a.push[0] * hd, [=] __device__(uint64_t idx) {
    C[idx] = A[(idx / hd) * dim + c0 + idx % hd];
  });
}
cudaError_t run_set(const OpArgs &a) {
  float *D = (float *)a.buf[0];
  const float *S = (const float *)a.buf[1];
  const uint32_t dim = a.push[1], hd = a.push[2], c0 = a.push[3];
  return launch_each(a, (uint64_t)a.push[0] * hd, [=] __device__(uint64_t idx) {
    D[(idx / hd) * dim + c0 + idx % hd] = S[idx];
  });
}

// ---- elementwise gradients and optimizers -----------------------------------------
const char *chk_n5(const OpArgs &a) {
  const uint64_t n = a.push[0];
  return need_all(a, {n, n, n, n, n});
}
cudaError_t run_silu_mul_bwd(const OpArgs &a) {
  const float *G = (const float *)a.buf[0], *A = (const float *)a.buf[1],
              *B = (const float *)a.buf[2];
  float *DA = (float *)a.buf[3], *DB = (float *)a.buf[4];
  return launch_each(a, a.push[0], [=] __device__(uint64_t i) {
    const float x = A[i], sg = sigm(x), g = G[i];
    DA[i] = __fmul_rn(__fmul_rn(g, B[i]),
                      __fmul_rn(sg, __fadd_rn(1.0f, __fmul_rn(x, __fsub_rn(1.0f, sg)))));
    DB[i] = __fmul_rn(g, __fmul_rn(x, sg));
  });
}
const char *chk_n3(const OpArgs &a) {
  const uint64_t n = a.push[0];
  return need_all(a, {n, n, n});
}
cudaError_t run_silu_bwd(const OpArgs &a) {
  const float *G = (const float *)a.buf[0], *X = (const float *)a.buf[1];
  float *D = (float *)a.buf[2];
  return launch_each(a, a.push[0], [=] __device__(uint64_t i) {
    const float x = X[i], sg = sigm(x);
    D[i] = __fmul_rn(G[i], __fmul_rn(sg, __fadd_rn(1.0f, __fmul_rn(x, __fsub_rn(1.0f, sg)))));
  });
}
cudaError_t run_gelu_bwd(const OpArgs &a) {
  const float *G = (const float *)a.buf[0], *H = (const float *)a.buf[1];
  float *D = (float *)a.buf[2];
  return launch_each(a, a.push[0], [=] __device__(uint64_t i) {
    const float x = H[i];
    const float inner =
        __fmul_rn(0.7978845608f, __fadd_rn(x, __fmul_rn(0.044715f, __fmul_rn(x, __fmul_rn(x, x)))));
    const float e = expf(__fmul_rn(2.0f, inner));
    const float th = __fdiv_rn(__fsub_rn(e, 1.0f), __fadd_rn(e, 1.0f));
    const float sech2 = __fsub_rn(1.0f, __fmul_rn(th, th));
    const float dudx = __fmul_rn(0.7978845608f, __fadd_rn(1.0f, __fmul_rn(0.134145f, __fmul_rn(x, x))));
    const float gp = __fadd_rn(__fmul_rn(0.5f, __fadd_rn(1.0f, th)),
                               __fmul_rn(0.5f, __fmul_rn(x, __fmul_rn(sech2, dudx))));
    D[i] = __fmul_rn(G[i], gp);
  });
}
const char *chk_sub_scale(const OpArgs &a) {
  const uint64_t n = a.push[0];
  return need_all(a, {n, n, 1, n});
}
cudaError_t run_sub_scale(const OpArgs &a) {
  const float *A = (const float *)a.buf[0], *B = (const float *)a.buf[1],
              *S = (const float *)a.buf[2];
  float *C = (float *)a.buf[3];
  return launch_each(a, a.push[0], [=] __device__(uint64_t i) {
    C[i] = __fmul_rn(__fsub_rn(A[i], B[i]), S[0]);
  });
}
const char *chk_sgd(const OpArgs &a) {
  const uint64_t n = a.push[0];
  return need_all(a, {n, n, 1, 1});
}
cudaError_t run_sgd(const OpArgs &a) {
  float *W = (float *)a.buf[0];
  const float *G = (const float *)a.buf[1], *L = (const float *)a.buf[2],
              *S = (const float *)a.buf[3];
  return launch_each(a, a.push[0], [=] __device__(uint64_t i) {
    W[i] = __fsub_rn(W[i], __fmul_rn(__fmul_rn(L[0], S[0]), G[i]));
  });
}
const char *chk_adam(const OpArgs &a) {
  const uint64_t n = a.push[0];
  return need_all(a, {n, n, n, n, 4, 1});
}
cudaError_t run_adam(const OpArgs &a) {
  float *W = (float *)a.buf[0], *M = (float *)a.buf[2], *V = (float *)a.buf[3];
  const float *G = (const float *)a.buf[1], *H = (const float *)a.buf[4],
              *S = (const float *)a.buf[5];
  return launch_each(a, a.push[0], [=] __device__(uint64_t i) {
    const float g = __fmul_rn(S[0], G[i]);
    const float b1 = H[1], b2 = H[2];
    const float m = __fadd_rn(__fmul_rn(b1, M[i]), __fmul_rn(__fsub_rn(1.0f, b1), g));
    const float v = __fadd_rn(__fmul_rn(b2, V[i]), __fmul_rn(__fsub_rn(1.0f, b2), __fmul_rn(g, g)));
    M[i] = m;
    V[i] = v;
    W[i] = __fsub_rn(W[i], __fmul_rn(H[0], __fdiv_rn(m, __fadd_rn(sqrtf(v), H[3]))));
  });
}

// ---- reductions ----------------------------------------------------------------------
// colsum / rmsnorm-dgamma: one thread per column, rows in order (coalesced across threads).
const char *chk_colsum(const OpArgs &a) {
  return need_all(a, {(uint64_t)a.push[0] * a.push[1], a.push[1]});
}
cudaError_t run_colsum(const OpArgs &a) {
  const float *G = (const float *)a.buf[0];
  float *D = (float *)a.buf[1];
  const uint32_t M = a.push[0], N = a.push[1];
  return launch_each(a, N, [=] __device__(uint64_t o) {
    float acc = 0.0f;
    for (uint32_t r = 0; r < M; r++) acc = __fadd_rn(acc, G[(uint64_t)r * N + o]);
    D[o] = acc;
  });
}
const char *chk_dgamma(const OpArgs &a) {
  const uint64_t mn = (uint64_t)a.push[0] * a.push[1];
  return need_all(a, {mn, mn, a.push[0], a.push[1]});
}
cudaError_t run_dgamma(const OpArgs &a) {
  const float *DY = (const float *)a.buf[0], *X = (const float *)a.buf[1],
              *S = (const float *)a.buf[2];
  float *DG = (float *)a.buf[3];
  const uint32_t M = a.push[0], N = a.push[1];
  return launch_each(a, N, [=] __device__(uint64_t j) {
    float acc = 0.0f;
    for (uint32_t r = 0; r < M; r++) {
      const uint64_t k = (uint64_t)r * N + j;
      acc = __fadd_rn(acc, __fmul_rn(__fmul_rn(DY[k], X[k]), S[r]));
    }
    DG[j] = acc;
  });
}

// Row reductions: one warp per row.
__device__ __forceinline__ float warp_sum(float v) {
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
template <typename F>
__global__ void k_rows(uint32_t M, uint64_t limit, F f) {
  const uint64_t r = (uint64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (r >= M || r >= limit) return;
  f((uint32_t)r, threadIdx.x & 31);
}
template <typename F>
cudaError_t launch_rows(const OpArgs &a, uint32_t M, F f) {
  if (!M) return cudaSuccess;
  k_rows<<<(unsigned)ceil_div64(M, 8), 256, 0, a.stream>>>(M, invocations(a.groups, 64), f);
  count_launches(1);
  return cudaPeekAtLastError();
}
const char *chk_rmsnorm_dx(const OpArgs &a) {
  const uint64_t mn = (uint64_t)a.push[0] * a.push[1];
  return need_all(a, {mn, mn, a.push[0], a.push[1], mn});
}
cudaError_t run_rmsnorm_dx(const OpArgs &a) {
  const float *DY = (const float *)a.buf[0], *X = (const float *)a.buf[1],
              *S = (const float *)a.buf[2], *G = (const float *)a.buf[3];
  float *DX = (float *)a.buf[4];
  const uint32_t N = a.push[1];
  return launch_rows(a, a.push[0], [=] __device__(uint32_t r, int lane) {
    const uint64_t base = (uint64_t)r * N;
    const float is = S[r];
    float acc = 0.0f;
    for (uint32_t k = lane; k < N; k += 32)
      acc = __fadd_rn(acc, __fmul_rn(__fmul_rn(DY[base + k], G[k]), X[base + k]));
    const float s = warp_sum(acc);
    const float is3 = __fdiv_rn(__fmul_rn(__fmul_rn(is, is), is), (float)N);
    for (uint32_t j = lane; j < N; j += 32)
      DX[base + j] = __fsub_rn(__fmul_rn(__fmul_rn(is, DY[base + j]), G[j]),
                               __fmul_rn(__fmul_rn(is3, X[base + j]), s));
  });
}
const char *chk_softmax_bwd(const OpArgs &a) {
  const uint64_t mn = (uint64_t)a.push[0] * a.push[1];
  return need_all(a, {mn, mn, mn});
}
cudaError_t run_softmax_bwd(const OpArgs &a) {
  const float *P = (const float *)a.buf[0], *G = (const float *)a.buf[1];
  float *DS = (float *)a.buf[2];
  const uint32_t N = a.push[1];
  return launch_rows(a, a.push[0], [=] __device__(uint32_t r, int lane) {
    const uint64_t base = (uint64_t)r * N;
    float acc = 0.0f;
    for (uint32_t k = lane; k < N; k += 32) acc = __fadd_rn(acc, __fmul_rn(P[base + k], G[base + k]));
    const float dot = warp_sum(acc);
    for (uint32_t j = lane; j < N; j += 32)
      DS[base + j] = __fmul_rn(P[base + j], __fsub_rn(G[base + j], dot));
  });
}
const char *chk_rowdot(const OpArgs &a) {
  const uint64_t mn = (uint64_t)a.push[0] * a.push[1];
  return need_all(a, {mn, mn, a.push[0]});
}
cudaError_t run_rowdot(const OpArgs &a) {
  const float *G = (const float *)a.buf[0], *Y = (const float *)a.buf[1];
  float *D = (float *)a.buf[2];
  const uint32_t N = a.push[1];
  return launch_rows(a, a.push[0], [=] __device__(uint32_t r, int lane) {
    const uint64_t base = (uint64_t)r * N;
    float acc = 0.0f;
    for (uint32_t j = lane; j < N; j += 32) acc = __fadd_rn(acc, __fmul_rn(G[base + j], Y[base + j]));
    const float s = warp_sum(acc);
    if (lane == 0) D[r] = s;
  });
}
// ce-grad (OH one-hot) / ce-grad-idx (TG target index): (softmax - target) / M.
template <bool IDX>
const char *chk_ce(const OpArgs &a) {
  const uint64_t mv = (uint64_t)a.push[0] * a.push[1];
  return need_all(a, {mv, IDX ? (uint64_t)a.push[0] : mv, mv});
}
template <bool IDX>
cudaError_t run_ce(const OpArgs &a) {
  const float *LG = (const float *)a.buf[0], *T = (const float *)a.buf[1];
  float *G = (float *)a.buf[2];
  const uint32_t M = a.push[0], V = a.push[1];
  return launch_rows(a, M, [=] __device__(uint32_t r, int lane) {
    const uint64_t base = (uint64_t)r * V;
    float mx = V ? LG[base] : 0.0f;
    for (uint32_t j = lane; j < V; j += 32) mx = fmaxf(mx, LG[base + j]);
    mx = warp_max(mx);
    float acc = 0.0f;
    for (uint32_t j = lane; j < V; j += 32) acc = __fadd_rn(acc, expf(__fsub_rn(LG[base + j], mx)));
    const float s = warp_sum(acc);
    const float invm = __fdiv_rn(1.0f, (float)M);
    const uint32_t tgt = IDX ? f2u(T[r]) : 0u;
    for (uint32_t j = lane; j < V; j += 32) {
      const float sub = IDX ? (j == tgt ? 1.0f : 0.0f) : T[base + j];
      G[base + j] = __fmul_rn(__fsub_rn(__fdiv_rn(expf(__fsub_rn(LG[base + j], mx)), s), sub), invm);
    }
  });
}

// ---- MoE top-k mask ------------------------------------------------------------
const char *chk_topk(const OpArgs &a) {
  const uint64_t me = (uint64_t)a.push[0] * a.push[1];
  return need_all(a, {me, me});
}
cudaError_t run_topk(const OpArgs &a) {
  const float *LG = (const float *)a.buf[0];
  float *MK = (float *)a.buf[1];
  const uint32_t E = a.push[1], K = a.push[2];
  return launch_each(a, (uint64_t)a.push[0] * E, [=] __device__(uint64_t idx) {
    const uint64_t base = idx / E * E;
    const float ve = LG[idx];
    uint32_t cnt = 0;
    for (uint32_t j = 0; j < E; j++) cnt += LG[base + j] > ve ? 1u : 0u;
    MK[idx] = cnt < K ? 0.0f : -1.0e30f;
  });
}

// ---- embedding backward ---------------------------------------------------------
const char *chk_embed_bwd(const OpArgs &a) {
  const uint64_t seq = a.push[0], dim = a.push[1], vocab = a.push[2];
  return need_all(a, {seq, seq * dim, vocab * dim});
}
cudaError_t run_embed_bwd(const OpArgs &a) {
  const float *TOK = (const float *)a.buf[0], *GX = (const float *)a.buf[1];
  float *DW = (float *)a.buf[2];
  const uint32_t seq = a.push[0], dim = a.push[1];
  return launch_each(a, (uint64_t)a.push[2] * dim, [=] __device__(uint64_t idx) {
    const uint32_t tt = (uint32_t)(idx / dim), j = (uint32_t)(idx % dim);
    float acc = 0.0f;
    for (uint32_t i = 0; i < seq; i++)
      if (f2u(TOK[i]) == tt) acc = __fadd_rn(acc, GX[(uint64_t)i * dim + j]);
    DW[idx] = acc;
  });
}

// ---- paged gather / scatter spikes -------------------------------------------------
const char *chk_spike(const OpArgs &a, bool scatter) {
  const uint64_t n = a.push[0], bs = a.push[1];
  return scatter ? need_all(a, {n, n * bs, 0}) : need_all(a, {n, 0, n * bs});
}
const char *chk_gather_spike(const OpArgs &a) { return chk_spike(a, false); }
const char *chk_scatter_spike(const OpArgs &a) { return chk_spike(a, true); }
cudaError_t run_gather_spike(const OpArgs &a) {
  const float *TABLE = (const float *)a.buf[0], *POOL = (const float *)a.buf[1];
  float *OUT = (float *)a.buf[2];
  const uint32_t bs = a.push[1];
  const uint64_t pool = a.words[1];
  return launch_each(a, (uint64_t)a.push[0] * bs, [=] __device__(uint64_t idx) {
    const uint64_t src = (uint64_t)f2u(TABLE[idx / bs]) * bs + idx % bs;
    if (src < pool) OUT[idx] = POOL[src];
  });
}
cudaError_t run_scatter_spike(const OpArgs &a) {
  const float *TABLE = (const float *)a.buf[0], *SRC = (const float *)a.buf[1];
  float *POOL = (float *)a.buf[2];
  const uint32_t bs = a.push[1];
  const uint64_t pool = a.words[2];
  return launch_each(a, (uint64_t)a.push[0] * bs, [=] __device__(uint64_t idx) {
    const uint64_t dst = (uint64_t)f2u(TABLE[idx / bs]) * bs + idx % bs;
    if (dst < pool) POOL[dst] = SRC[idx];
  });
}

// ---- gated delta-net step (one token t of a linear-attention recurrence) --------
// S [nv x dk x dv] in place: decay by G, delta-rule update with B, read out by Q.
const char *chk_gdn(const OpArgs &a) {
  const uint64_t nv = a.push[0], dk = a.push[1], dv = a.push[2], t = a.push[3];
  return need_all(a, {nv * dk * dv, (t + 1) * nv * dk, (t + 1) * nv * dk, (t + 1) * nv * dv,
                      (t + 1) * nv, (t + 1) * nv, (t + 1) * nv * dv});
}
cudaError_t run_gdn(const OpArgs &a) {
  float *S = (float *)a.buf[0], *OUT = (float *)a.buf[6];
  const float *Q = (const float *)a.buf[1], *K = (const float *)a.buf[2],
              *V = (const float *)a.buf[3], *G = (const float *)a.buf[4],
              *B = (const float *)a.buf[5];
  const uint32_t nv = a.push[0], dk = a.push[1], dv = a.push[2], t = a.push[3];
  return launch_each(a, (uint64_t)nv * dv, [=] __device__(uint64_t idx) {
    const uint32_t h = (uint32_t)(idx / dv), j = (uint32_t)(idx % dv);
    const uint64_t sb = (uint64_t)h * dk * dv + j, qb = ((uint64_t)t * nv + h) * dk;
    const uint64_t vb = ((uint64_t)t * nv + h) * dv + j;
    const float gv = G[(uint64_t)t * nv + h], bv = B[(uint64_t)t * nv + h];
    float mem = 0.0f;
    for (uint32_t i = 0; i < dk; i++) {
      const uint64_t p = sb + (uint64_t)i * dv;
      const float sv = __fmul_rn(S[p], gv);
      S[p] = sv;
      mem = __fadd_rn(mem, __fmul_rn(sv, K[qb + i]));
    }
    const float d = __fmul_rn(bv, __fsub_rn(V[vb], mem));
    float o = 0.0f;
    for (uint32_t i = 0; i < dk; i++) {
      const uint64_t p = sb + (uint64_t)i * dv;
      const float sv = __fadd_rn(S[p], __fmul_rn(K[qb + i], d));
      S[p] = sv;
      o = __fadd_rn(o, __fmul_rn(sv, Q[qb + i]));
    }
    OUT[vb] = o;
  });
}

// ---- tree attention (a speculative-decoding token tree over a cached prefix) ------
// Row i attends to the LEN[0] cached keys and to its ancestors in the tree
// (PAR links, at most maxdepth of them, a parent index >= M ends the walk).
const char *chk_tree(const OpArgs &a) {
  const uint64_t M = a.push[0], dim = a.push[1], heads = a.push[2], kvheads = a.push[3];
  if (!heads || !kvheads || dim % heads || heads % kvheads)
    return fmt_msg("tree-attn: dim %u, heads %u, kvheads %u do not divide", a.push[1],
                   a.push[2], a.push[3]);
  const uint64_t kvdim = kvheads * (dim / heads);
  return need_all(a, {M * dim, 0, 0, M * kvdim, M * kvdim, M, 1, M * dim});
}
cudaError_t run_tree(const OpArgs &a) {
  const float *Q = (const float *)a.buf[0], *CK = (const float *)a.buf[1],
              *CV = (const float *)a.buf[2], *NK = (const float *)a.buf[3],
              *NV = (const float *)a.buf[4], *PAR = (const float *)a.buf[5],
              *LEN = (const float *)a.buf[6];
  float *C = (float *)a.buf[7];
  const uint32_t M = a.push[0], dim = a.push[1], heads = a.push[2], kvheads = a.push[3],
                 maxdepth = a.push[4];
  const uint64_t cache_words = a.words[1] < a.words[2] ? a.words[1] : a.words[2];
  return launch_each(a, (uint64_t)M * dim, [=] __device__(uint64_t idx) {
    const uint32_t hd = dim / heads, grp = heads / kvheads, kvdim = kvheads * hd;
    const uint32_t i = (uint32_t)(idx / dim), c = (uint32_t)(idx % dim);
    const uint32_t h = c / hd, t = c % hd, kvh = h / grp;
    uint32_t L = f2u(LEN[0]);
    if ((uint64_t)L * kvdim > cache_words) L = (uint32_t)(cache_words / kvdim);
    const uint64_t c0q = (uint64_t)i * dim + (uint64_t)h * hd;
    const float coef = __fdiv_rn(1.0f, sqrtf((float)hd));
    auto score = [&](const float *Kp, uint64_t kb) {
      float acc = 0.0f;
      for (uint32_t tt = 0; tt < hd; tt++) acc = __fadd_rn(acc, __fmul_rn(Q[c0q + tt], Kp[kb + tt]));
      return __fmul_rn(acc, coef);
    };
    float mx = -1.0e30f;
    for (uint32_t j = 0; j < L; j++) mx = fmaxf(mx, score(CK, (uint64_t)j * kvdim + kvh * hd));
    uint32_t cur = i;
    for (uint32_t d = 0; d < maxdepth && cur < M; d++) {
      mx = fmaxf(mx, score(NK, (uint64_t)cur * kvdim + kvh * hd));
      cur = f2u(PAR[cur]);
    }
    float z = 0.0f, ctx = 0.0f;
    for (uint32_t j = 0; j < L; j++) {
      const uint64_t kb = (uint64_t)j * kvdim + kvh * hd;
      const float e = expf(__fsub_rn(score(CK, kb), mx));
      z = __fadd_rn(z, e);
      ctx = __fadd_rn(ctx, __fmul_rn(e, CV[kb + t]));
    }
    cur = i;
    for (uint32_t d = 0; d < maxdepth && cur < M; d++) {
      const uint64_t kb = (uint64_t)cur * kvdim + kvh * hd;
      const float e = expf(__fsub_rn(score(NK, kb), mx));
      z = __fadd_rn(z, e);
      ctx = __fadd_rn(ctx, __fmul_rn(e, NV[kb + t]));
      cur = f2u(PAR[cur]);
    }
    C[idx] = __fdiv_rn(ctx, z);
  });
}

}  // namespace

const OpSpec kTrainOps[] = {
    {"transpose", 2, 2, chk_transpose, no_scr, run_transpose},
    {"slice-cols", 2, 4, chk_slice, no_scr, run_slice},
    {"set-cols", 2, 4, chk_set, no_scr, run_set},
    {"silu-mul-bwd", 5, 1, chk_n5, no_scr, run_silu_mul_bwd},
    {"silu-bwd", 3, 1, chk_n3, no_scr, run_silu_bwd},
    {"gelu-bwd", 3, 1, chk_n3, no_scr, run_gelu_bwd},
    {"sub-scale", 4, 1, chk_sub_scale, no_scr, run_sub_scale},
    {"sgd", 4, 1, chk_sgd, no_scr, run_sgd},
    {"adam", 6, 1, chk_adam, no_scr, run_adam},
    {"colsum", 2, 2, chk_colsum, no_scr, run_colsum},
    {"rmsnorm-dgamma", 4, 2, chk_dgamma, no_scr, run_dgamma},
    {"rmsnorm-dx", 5, 2, chk_rmsnorm_dx, no_scr, run_rmsnorm_dx},
    {"softmax-bwd", 3, 2, chk_softmax_bwd, no_scr, run_softmax_bwd},
    {"rowdot", 3, 2, chk_rowdot, no_scr, run_rowdot},
    {"ce-grad", 3, 2, chk_ce<false>, no_scr, run_ce<false>},
    {"ce-grad-idx", 3, 2, chk_ce<true>, no_scr, run_ce<true>},
    {"topk-mask", 2, 3, chk_topk, no_scr, run_topk},
    {"embed-bwd", 3, 3, chk_embed_bwd, no_scr, run_embed_bwd},
    {"gather-spike", 3, 2, chk_gather_spike, no_scr, run_gather_spike},
    {"scatter-spike", 3, 2, chk_scatter_spike, no_scr, run_scatter_spike},
    {"gdn-step", 7, 4, chk_gdn, no_scr, run_gdn},
    {"tree-attn", 8, 5, chk_tree, no_scr, run_tree},
};
const int kTrainOpsCount = sizeof(kTrainOps) / sizeof(kTrainOps[0]);

}  // namespace nl

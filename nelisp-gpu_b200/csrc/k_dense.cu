// k_dense.cu -- f32 matmul family for sm_100a.
//
// Reference operators (lisp/nelisp-gpu-kernels.el):
//   matmul       :17-27   C = A B, row-major, one invocation per output
//   linear       :71-81   C = X W^T + B
//   matmul-tiled :82-107  the same product with 16x16 workgroup tiles
//   matmul-reg   :129     4x4 outputs per invocation (M, N multiples of 4)
//
// The product is computed in f32 on the CUDA cores (FFMA): the parity bar is
// 1e-4 of the output scale, which plain TF32 tensor-core products miss at
// these depths.  Register-blocked tiles staged through shared memory; the
// tile size is chosen so that the grid fills the 148 SMs.  `groups` keeps
// each operator's own meaning for the short-grid emulation (elements for
// matmul/linear, 16x16 tiles for matmul-tiled, 4x4 blocks for matmul-reg).

#include <cuda_runtime.h>
#include <stdint.h>

#include "nl_internal.h"

namespace nl {
namespace {

enum Cover { kElem = 0, kTile16 = 1, kReg4 = 2 };

template <int BM, int BN, int BK, int TM, int TN, bool TRANS_B, bool TRANS_A = false>
__global__ void __launch_bounds__((BM / TM) * (BN / TN))
sgemm_kernel(const float *__restrict__ A, const float *__restrict__ B,
             const float *__restrict__ bias, float *__restrict__ C,
             uint32_t M, uint32_t K, uint32_t N, int cover, uint64_t limit) {
  constexpr int TX = BN / TN, TY = BM / TM, NT = TX * TY;
  __shared__ float As[BK][BM + 4];
  __shared__ float Bs[BK][BN + 4];
  const int tid = threadIdx.x, tx = tid % TX, ty = tid / TX;
  const uint32_t m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
  float acc[TM][TN];
#pragma unroll
  for (int i = 0; i < TM; i++)
#pragma unroll
    for (int j = 0; j < TN; j++) acc[i][j] = 0.0f;

  for (uint32_t k0 = 0; k0 < K; k0 += BK) {
    if (TRANS_A) {
      // A is [K x M] (matmul-at); tile element (kk, r) = A[k0 + kk, m0 + r]
      for (int e = tid; e < BM * BK; e += NT) {
        int kk = e / BM, r = e % BM;
        uint32_t gr = m0 + r, gk = k0 + kk;
        As[kk][r] = (gr < M && gk < K) ? __ldg(A + (uint64_t)gk * M + gr) : 0.0f;
      }
    } else {
      for (int e = tid; e < BM * BK; e += NT) {
        int r = e / BK, kk = e % BK;
        uint32_t gr = m0 + r, gk = k0 + kk;
        As[kk][r] = (gr < M && gk < K) ? __ldg(A + (uint64_t)gr * K + gk) : 0.0f;
      }
    }
    if (TRANS_B) {
      // B is [N x K] (a linear layer's weight); tile element (kk, c) = B[c, kk]
      for (int e = tid; e < BN * BK; e += NT) {
        int c = e / BK, kk = e % BK;
        uint32_t gc = n0 + c, gk = k0 + kk;
        Bs[kk][c] = (gc < N && gk < K) ? __ldg(B + (uint64_t)gc * K + gk) : 0.0f;
      }
    } else {
      for (int e = tid; e < BN * BK; e += NT) {
        int kk = e / BN, c = e % BN;
        uint32_t gc = n0 + c, gk = k0 + kk;
        Bs[kk][c] = (gc < N && gk < K) ? __ldg(B + (uint64_t)gk * N + gc) : 0.0f;
      }
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < BK; kk++) {
      float a[TM], b[TN];
#pragma unroll
      for (int i = 0; i < TM; i++) a[i] = As[kk][ty * TM + i];
#pragma unroll
      for (int j = 0; j < TN; j++) b[j] = Bs[kk][tx * TN + j];
#pragma unroll
      for (int i = 0; i < TM; i++)
#pragma unroll
        for (int j = 0; j < TN; j++) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
  const uint32_t tiles16 = (N + 15) / 16, blocks4 = (N + 3) / 4;
#pragma unroll
  for (int i = 0; i < TM; i++) {
    uint32_t r = m0 + ty * TM + i;
    if (r >= M) continue;
#pragma unroll
    for (int j = 0; j < TN; j++) {
      uint32_t c = n0 + tx * TN + j;
      if (c >= N) continue;
      uint64_t unit;
      if (cover == kTile16) unit = (uint64_t)(r / 16) * tiles16 + c / 16;
      else if (cover == kReg4) unit = (uint64_t)(r / 4) * blocks4 + c / 4;
      else unit = (uint64_t)r * N + c;
      if (unit >= limit) continue;
      float v = acc[i][j];
      if (bias) v = __ldg(bias + c) + v;
      C[(uint64_t)r * N + c] = v;
    }
  }
}

template <bool TRANS_B, bool TRANS_A = false>
cudaError_t sgemm(const float *A, const float *B, const float *bias, float *C,
                  uint32_t M, uint32_t K, uint32_t N, int cover,
                  uint64_t limit, cudaStream_t st) {
  if (M == 0 || N == 0) return cudaSuccess;
  uint64_t big = (uint64_t)M * N;
  if (big >= (uint64_t)148 * 64 * 64) {
    dim3 grid((N + 63) / 64, (M + 63) / 64);
    sgemm_kernel<64, 64, 16, 4, 4, TRANS_B, TRANS_A><<<grid, 256, 0, st>>>(A, B, bias, C, M, K, N, cover, limit);
  } else if (big >= (uint64_t)148 * 32 * 32) {
    dim3 grid((N + 31) / 32, (M + 31) / 32);
    sgemm_kernel<32, 32, 32, 2, 2, TRANS_B, TRANS_A><<<grid, 256, 0, st>>>(A, B, bias, C, M, K, N, cover, limit);
  } else {
    // Small products (the reference's 256^3 vkmatmul case): latency-bound,
    // so each CTA stages 256 columns of K at once (one load round and one
    // barrier for K <= 256, instead of eight) and runs its sequential-k
    // dot products from shared memory.
    dim3 grid((N + 15) / 16, (M + 15) / 16);
    sgemm_kernel<16, 16, 256, 1, 1, TRANS_B, TRANS_A><<<grid, 256, 0, st>>>(A, B, bias, C, M, K, N, cover, limit);
  }
  count_launches(1);
  return cudaPeekAtLastError();
}

size_t no_scratch(const OpArgs &) { return 0; }

const char *chk_matmul(const OpArgs &a) {
  uint64_t M = a.push[0], K = a.push[1], N = a.push[2];
  const char *m;
  if ((m = need_words(a, 0, (M * N) != 0 ? M * K : 0, "A"))) return m;
  if ((m = need_words(a, 1, (M * N) != 0 ? K * N : 0, "B"))) return m;
  return need_words(a, 2, M * N, "C");
}
const char *chk_matmul_reg(const OpArgs &a) {
  if (a.push[0] % 4 || a.push[2] % 4)
    return fmt_msg("matmul-reg: M (%u) and N (%u) must be multiples of 4",
                   a.push[0], a.push[2]);
  return chk_matmul(a);
}
template <int COVER>
cudaError_t run_matmul(const OpArgs &a) {
  uint64_t lim = COVER == kTile16 ? (uint64_t)a.groups : invocations(a.groups, 64);
  return sgemm<false>((const float *)a.buf[0], (const float *)a.buf[1], nullptr,
                      (float *)a.buf[2], a.push[0], a.push[1], a.push[2], COVER,
                      lim, a.stream);
}

const char *chk_linear(const OpArgs &a) {
  // (X W B C) push (M IN OUT)
  uint64_t M = a.push[0], IN = a.push[1], OUT = a.push[2];
  const char *m;
  if ((m = need_words(a, 0, (M * OUT) != 0 ? M * IN : 0, "X"))) return m;
  if ((m = need_words(a, 1, (M * OUT) != 0 ? OUT * IN : 0, "W"))) return m;
  if ((m = need_words(a, 2, (M * OUT) != 0 ? OUT : 0, "B"))) return m;
  return need_words(a, 3, M * OUT, "C");
}
cudaError_t run_linear(const OpArgs &a) {
  return sgemm<true>((const float *)a.buf[0], (const float *)a.buf[1],
                     (const float *)a.buf[2], (float *)a.buf[3], a.push[0],
                     a.push[1], a.push[2], kElem, invocations(a.groups, 64),
                     a.stream);
}

}  // namespace

// matmul-at (kernels.el:177-186): C[m, n] = sum_k A[k, m] B[k, n], A [K x M].
const char *chk_matmul_at(const OpArgs &a) {
  const uint64_t M = a.push[0], K = a.push[1], N = a.push[2];
  const char *m;
  const bool any = M != 0 && N != 0;
  if ((m = need_words(a, 0, any ? K * M : 0, "A"))) return m;
  if ((m = need_words(a, 1, any ? K * N : 0, "B"))) return m;
  return need_words(a, 2, M * N, "C");
}
cudaError_t run_matmul_at(const OpArgs &a) {
  return sgemm<false, true>((const float *)a.buf[0], (const float *)a.buf[1], nullptr,
                            (float *)a.buf[2], a.push[0], a.push[1], a.push[2], kElem,
                            invocations(a.groups, 64), a.stream);
}

const OpSpec kDenseOps[] = {
    {"matmul-at", 3, 3, chk_matmul_at, no_scratch, run_matmul_at},
    {"matmul", 3, 3, chk_matmul, no_scratch, run_matmul<kElem>},
    {"matmul-tiled", 3, 3, chk_matmul, no_scratch, run_matmul<kTile16>},
    {"matmul-reg", 3, 3, chk_matmul_reg, no_scratch, run_matmul<kReg4>},
    {"linear", 4, 3, chk_linear, no_scratch, run_linear},
};
const int kDenseOpsCount = sizeof(kDenseOps) / sizeof(kDenseOps[0]);

}  // namespace nl

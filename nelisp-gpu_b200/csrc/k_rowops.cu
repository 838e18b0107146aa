// k_rowops.cu -- row reductions and elementwise kernels for sm_100a.
//
// Reference operators (lisp/nelisp-gpu-kernels.el):
//   softmax      :28-42     per row: m = max, s = sum exp(a-m), c = exp(a-m)/s
//   silu-mul     :187-193   C = (a * 1/(1+exp(-a))) * B
//   add2         :816-821   C = A + B           (vadd :12-16 is the same op)
//   scale        :141       C = A * S[0]
//   rmsnorm-istd :1250-1256 S[r] = 1/sqrt(sum x^2 / N + 1e-6)
//   rmsnorm-fwd  :1259-1265 C = (X * S[r]) * G[j]
//   embed-gather :1385-1392 C[i,j] = WTE[uint(TOK[i]) * dim + j]
//
// All are HBM-bound.  The reference runs softmax and rmsnorm-istd with ONE
// invocation per row (64 rows per workgroup), serial over the row; here a
// CTA owns a row, holds it in registers when it fits (one HBM read, one
// write) and reduces with warp shuffles.  Elementwise kernels use 128-bit
// loads when every buffer is 16-byte aligned.

#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include "nl_internal.h"

namespace nl {
namespace {

constexpr int kRowThreads = 256;

__device__ __forceinline__ float warp_max(float v) {
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float warp_sum(float v) {
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
// CTA-wide reductions through shared memory; every thread gets the result.
__device__ float block_max(float v, float *red) {
  v = warp_max(v);
  const int w = threadIdx.x >> 5, nw = blockDim.x >> 5;
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[w] = v;
  __syncthreads();
  float r = red[0];
  for (int i = 1; i < nw; i++) r = fmaxf(r, red[i]);
  return r;
}
__device__ float block_sum(float v, float *red) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, nw = blockDim.x >> 5;
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[w] = v;
  __syncthreads();
  float r = 0.0f;
  for (int i = 0; i < nw; i++) r += red[i];
  return r;
}

// ---- softmax ---------------------------------------------------------------
// One CTA per row; VPT floats per thread held in registers (rows up to
// VPT*256 columns).  The reference's max starts at A[base] and only a
// strictly larger value replaces it; a NaN element therefore never becomes
// the max there, as with fmaxf here.  The exponentials use the hardware
// exp2 (__expf) and the normalisation one reciprocal per row: a few
// instructions an element instead of a few dozen, so the kernel streams
// HBM instead of issuing math; the error stays within 1e-5 relative for
// exponents down to -60, below the reference's 1e-4 bar.
template <int VPT>
__global__ void __launch_bounds__(kRowThreads)
softmax_reg_kernel(const float *__restrict__ A, float *__restrict__ C,
                   uint32_t M, uint32_t N, uint64_t limit, int vec) {
  __shared__ float red[32];
  const uint32_t row = blockIdx.x;
  if (row >= M || row >= limit) return;
  const float *a = A + (uint64_t)row * N;
  float *c = C + (uint64_t)row * N;
  float v[VPT];
  float m = -INFINITY;
  if (vec) {
#pragma unroll
    for (int k = 0; k < VPT / 4; k++) {
      uint32_t i = 4u * (threadIdx.x + (uint32_t)k * kRowThreads);
      float4 x = (i < N) ? __ldcs(reinterpret_cast<const float4 *>(a + i))
                         : make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
      v[4 * k] = x.x; v[4 * k + 1] = x.y; v[4 * k + 2] = x.z; v[4 * k + 3] = x.w;
    }
  } else {
#pragma unroll
    for (int k = 0; k < VPT; k++) {
      uint32_t i = threadIdx.x + (uint32_t)k * kRowThreads;
      v[k] = (i < N) ? __ldcs(a + i) : -INFINITY;
    }
  }
#pragma unroll
  for (int k = 0; k < VPT; k++) m = fmaxf(m, v[k]);
  m = block_max(m, red);
  if (!(m > -INFINITY)) m = __ldg(a);  // all -inf/NaN: the reference keeps A[base]
  float s = 0.0f;
#pragma unroll
  for (int k = 0; k < VPT; k++) {
    v[k] = __expf(v[k] - m);
    s += v[k];
  }
  // Padding lanes held -inf and contribute exp(-inf) = 0.
  s = block_sum(s, red);
  const float inv = 1.0f / s;
  if (vec) {
#pragma unroll
    for (int k = 0; k < VPT / 4; k++) {
      uint32_t i = 4u * (threadIdx.x + (uint32_t)k * kRowThreads);
      if (i < N)
        __stcs(reinterpret_cast<float4 *>(c + i),
               make_float4(v[4 * k] * inv, v[4 * k + 1] * inv, v[4 * k + 2] * inv,
                           v[4 * k + 3] * inv));
    }
  } else {
#pragma unroll
    for (int k = 0; k < VPT; k++) {
      uint32_t i = threadIdx.x + (uint32_t)k * kRowThreads;
      if (i < N) __stcs(c + i, v[k] * inv);
    }
  }
}

// Rows longer than the register budget: an online max/sum pass, then a
// second read that writes.
__global__ void __launch_bounds__(kRowThreads)
softmax_long_kernel(const float *__restrict__ A, float *__restrict__ C,
                    uint32_t M, uint32_t N, uint64_t limit) {
  __shared__ float red[32];
  const uint32_t row = blockIdx.x;
  if (row >= M || row >= limit) return;
  const float *a = A + (uint64_t)row * N;
  float *c = C + (uint64_t)row * N;
  float m = -INFINITY, s = 0.0f;
  for (uint32_t i = threadIdx.x; i < N; i += blockDim.x) {
    float x = __ldg(a + i);
    if (x > m) { s = s * expf(m - x) + 1.0f; m = x; }
    else s += expf(x - m);
  }
  float gm = block_max(m, red);
  float part = (m > -INFINITY) ? s * expf(m - gm) : 0.0f;
  if (!(gm > -INFINITY)) gm = __ldg(a);
  float gs = block_sum(part, red);
  for (uint32_t i = threadIdx.x; i < N; i += blockDim.x) c[i] = expf(__ldg(a + i) - gm) / gs;
}

// ---- rmsnorm -----------------------------------------------------------------
__global__ void __launch_bounds__(kRowThreads)
rmsnorm_istd_kernel(const float *__restrict__ X, float *__restrict__ S,
                    uint32_t M, uint32_t N, uint64_t limit) {
  __shared__ float red[32];
  const uint32_t r = blockIdx.x;
  if (r >= M || r >= limit) return;
  const float *x = X + (uint64_t)r * N;
  float ss = 0.0f;
  for (uint32_t i = threadIdx.x; i < N; i += blockDim.x) {
    float v = __ldg(x + i);
    ss = fmaf(v, v, ss);
  }
  ss = block_sum(ss, red);
  if (threadIdx.x == 0) S[r] = 1.0f / sqrtf(ss / (float)N + 0.000001f);
}

__global__ void rmsnorm_fwd_kernel(const float *__restrict__ X,
                                   const float *__restrict__ S,
                                   const float *__restrict__ G,
                                   float *__restrict__ C, uint32_t M,
                                   uint32_t N, uint64_t n) {
  for (uint64_t idx = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < n;
       idx += (uint64_t)gridDim.x * blockDim.x) {
    uint32_t r = (uint32_t)(idx / N), j = (uint32_t)(idx % N);
    C[idx] = (__ldg(X + idx) * __ldg(S + r)) * __ldg(G + j);
  }
}

// ---- elementwise -------------------------------------------------------------
enum Ew { kAdd = 0, kSiluMul = 1, kScale = 2, kMul = 3 };

template <int OP>
__device__ __forceinline__ float ew(float a, float b) {
  if (OP == kAdd) return a + b;
  if (OP == kMul || OP == kScale) return a * b;
  // silu-mul: (a * sigmoid(a)) * b, sigmoid = 1/(1+exp(-a))
  float sg = 1.0f / (1.0f + expf(-a));
  return (a * sg) * b;
}

template <int OP>
__global__ void ew_kernel(const float *__restrict__ A, const float *__restrict__ B,
                          float *__restrict__ C, uint64_t n, int vec) {
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  uint64_t t = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (vec) {
    const uint64_t n4 = n / 4;
    for (uint64_t i = t; i < n4; i += stride) {
      float4 a = __ldcs(reinterpret_cast<const float4 *>(A) + i);
      float4 b = (OP == kScale) ? make_float4(0, 0, 0, 0)
                                : __ldcs(reinterpret_cast<const float4 *>(B) + i);
      if (OP == kScale) { float s = __ldg(B); b = make_float4(s, s, s, s); }
      float4 c = make_float4(ew<OP>(a.x, b.x), ew<OP>(a.y, b.y), ew<OP>(a.z, b.z),
                             ew<OP>(a.w, b.w));
      __stcs(reinterpret_cast<float4 *>(C) + i, c);
    }
    for (uint64_t i = 4 * n4 + t; i < n; i += stride)
      C[i] = ew<OP>(A[i], OP == kScale ? __ldg(B) : B[i]);
  } else {
    for (uint64_t i = t; i < n; i += stride)
      C[i] = ew<OP>(A[i], OP == kScale ? __ldg(B) : B[i]);
  }
}

__global__ void embed_gather_kernel(const float *__restrict__ TOK,
                                    const float *__restrict__ WTE,
                                    float *__restrict__ C, uint32_t dim,
                                    uint64_t n, uint64_t wte_words) {
  // The row index is uint32 arithmetic as in the reference; a token id past
  // the table reads zero (Vulkan's robust buffer access) instead of faulting.
  for (uint64_t idx = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < n;
       idx += (uint64_t)gridDim.x * blockDim.x) {
    uint32_t i = (uint32_t)(idx / dim), j = (uint32_t)(idx % dim);
    uint32_t tk = __float2uint_rz(__ldg(TOK + i));
    uint32_t w = tk * dim + j;
    C[idx] = (w < wte_words) ? __ldg(WTE + w) : 0.0f;
  }
}

// ---- registry glue -------------------------------------------------------------
size_t no_scratch(const OpArgs &) { return 0; }

const char *chk_softmax(const OpArgs &a) {
  uint64_t n = (uint64_t)a.push[0] * a.push[1];
  const char *m;
  if ((m = need_words(a, 0, n, "A"))) return m;
  return need_words(a, 1, n, "C");
}
cudaError_t run_softmax(const OpArgs &a) {
  uint32_t M = a.push[0], N = a.push[1];
  if (M == 0 || N == 0) return cudaSuccess;
  uint64_t lim = invocations(a.groups, 64);
  int vec = aligned16(a.buf[0]) && aligned16(a.buf[1]) && (N % 4 == 0);
  const float *A = (const float *)a.buf[0];
  float *C = (float *)a.buf[1];
  if (N <= 1024u)
    softmax_reg_kernel<4><<<M, kRowThreads, 0, a.stream>>>(A, C, M, N, lim, vec);
  else if (N <= 2048u)
    softmax_reg_kernel<8><<<M, kRowThreads, 0, a.stream>>>(A, C, M, N, lim, vec);
  else if (N <= 4096u)
    softmax_reg_kernel<16><<<M, kRowThreads, 0, a.stream>>>(A, C, M, N, lim, vec);
  else if (N <= 8192u)
    softmax_reg_kernel<32><<<M, kRowThreads, 0, a.stream>>>(A, C, M, N, lim, vec);
  else
    softmax_long_kernel<<<M, kRowThreads, 0, a.stream>>>(A, C, M, N, lim);
  count_launches(1);
  return cudaPeekAtLastError();
}

template <int OP>
const char *chk_ew(const OpArgs &a) {
  uint64_t n = a.push[0];
  const char *m;
  if ((m = need_words(a, 0, n, "A"))) return m;
  if ((m = need_words(a, 1, OP == kScale ? (n ? 1 : 0) : n, OP == kScale ? "S" : "B"))) return m;
  return need_words(a, 2, n, "C");
}
template <int OP>
cudaError_t run_ew(const OpArgs &a) {
  uint64_t n = a.push[0];
  uint64_t lim = invocations(a.groups, 64);
  if (lim < n) n = lim;
  if (n == 0) return cudaSuccess;
  int vec = aligned16(a.buf[0]) && aligned16(a.buf[2]) && (OP == kScale || aligned16(a.buf[1]));
  ew_kernel<OP><<<grid_for(vec ? (n + 3) / 4 : n, 256), 256, 0, a.stream>>>(
      (const float *)a.buf[0], (const float *)a.buf[1], (float *)a.buf[2], n, vec);
  count_launches(1);
  return cudaPeekAtLastError();
}

const char *chk_rms_istd(const OpArgs &a) {
  const char *m;
  if ((m = need_words(a, 0, (uint64_t)a.push[0] * a.push[1], "X"))) return m;
  return need_words(a, 1, a.push[0], "S");
}
cudaError_t run_rms_istd(const OpArgs &a) {
  if (a.push[0] == 0) return cudaSuccess;
  rmsnorm_istd_kernel<<<a.push[0], kRowThreads, 0, a.stream>>>(
      (const float *)a.buf[0], (float *)a.buf[1], a.push[0], a.push[1],
      invocations(a.groups, 64));
  count_launches(1);
  return cudaPeekAtLastError();
}

const char *chk_rms_fwd(const OpArgs &a) {
  uint64_t M = a.push[0], N = a.push[1];
  const char *m;
  if ((m = need_words(a, 0, M * N, "X"))) return m;
  if ((m = need_words(a, 1, (M * N) != 0 ? M : 0, "S"))) return m;
  if ((m = need_words(a, 2, (M * N) != 0 ? N : 0, "G"))) return m;
  return need_words(a, 3, M * N, "C");
}
cudaError_t run_rms_fwd(const OpArgs &a) {
  uint64_t n = (uint64_t)a.push[0] * a.push[1];
  uint64_t lim = invocations(a.groups, 64);
  if (lim < n) n = lim;
  if (n == 0) return cudaSuccess;
  rmsnorm_fwd_kernel<<<grid_for(n, 256), 256, 0, a.stream>>>(
      (const float *)a.buf[0], (const float *)a.buf[1], (const float *)a.buf[2],
      (float *)a.buf[3], a.push[0], a.push[1], n);
  count_launches(1);
  return cudaPeekAtLastError();
}

const char *chk_embed(const OpArgs &a) {
  // (TOK WTE C) push (seq dim); the WTE rows read depend on TOK's data and
  // are bounds-checked on the device side by the caller's table size.
  uint64_t seq = a.push[0], dim = a.push[1];
  const char *m;
  if ((m = need_words(a, 0, (seq * dim) != 0 ? seq : 0, "TOK"))) return m;
  return need_words(a, 2, seq * dim, "C");
}
cudaError_t run_embed(const OpArgs &a) {
  uint64_t n = (uint64_t)a.push[0] * a.push[1];
  uint64_t lim = invocations(a.groups, 64);
  if (lim < n) n = lim;
  if (n == 0) return cudaSuccess;
  embed_gather_kernel<<<grid_for(n, 256), 256, 0, a.stream>>>(
      (const float *)a.buf[0], (const float *)a.buf[1], (float *)a.buf[2],
      a.push[1], n, (uint64_t)a.words[1]);
  count_launches(1);
  return cudaPeekAtLastError();
}

}  // namespace

const OpSpec kRowOps[] = {
    {"softmax", 2, 2, chk_softmax, no_scratch, run_softmax},
    {"silu-mul", 3, 1, chk_ew<kSiluMul>, no_scratch, run_ew<kSiluMul>},
    {"add2", 3, 1, chk_ew<kAdd>, no_scratch, run_ew<kAdd>},
    {"vadd", 3, 1, chk_ew<kAdd>, no_scratch, run_ew<kAdd>},
    {"mul", 3, 1, chk_ew<kMul>, no_scratch, run_ew<kMul>},
    {"scale", 3, 1, chk_ew<kScale>, no_scratch, run_ew<kScale>},
    {"rmsnorm-istd", 2, 2, chk_rms_istd, no_scratch, run_rms_istd},
    {"rmsnorm-fwd", 4, 2, chk_rms_fwd, no_scratch, run_rms_fwd},
    {"embed-gather", 3, 2, chk_embed, no_scratch, run_embed},
};
const int kRowOpsCount = sizeof(kRowOps) / sizeof(kRowOps[0]);

}  // namespace nl

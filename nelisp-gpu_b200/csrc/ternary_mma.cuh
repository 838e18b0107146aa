// ternary_mma.cuh -- the exact int8 tensor-core step of the ternary GEMV:
// mma.m16n8k32.s8 and the two-bit weight codes turned into its A operands.
// Shared by the GEMV kernels (k_ternary.cu) and the decoder's step kernel
// (nl_step.cu).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace nl {

__device__ __forceinline__ void mma_s8(int (&d)[4], uint32_t a0, uint32_t a1,
                                       uint32_t a2, uint32_t a3, uint2 b) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b.x), "r"(b.y));
}

// Two-bit codes -> int8 operands of four m16n8k32 steps, with no lookup.
// Byte b of word w holds codes 4b..4b+3, code i in field i % 4 (bits
// 2(i%4)..2(i%4)+1 of the byte).  MMA step j takes field j of every byte of
// the lane's two words (a0/a2 = the first / second word of row g, a1/a3 the
// same of row g+8; the activation fragments follow the same column order,
// see ternary_prep.cuh).  Two forms:
//
// unpack_signed: a code moved to bits 6..7 of a byte, the bits below
//   cleared, IS the int8 value 64*t of its trit (00 -> 0, 01 -> 64,
//   10 -> -128 = 64*(-2), 11 -> -64), the reference's sign-extending decode
//   scaled by 64: (w << 2(3-j)) & 0xC0C0C0C0, two instructions a register.
//   Every step carries 64*t, so the dot products come out multiplied by 64.
//
// unpack_offset: one LOP3 a register.  A code XOR 0b10 is t + 2 (00 -> 2,
//   01 -> 3, 11 -> 1, 10 -> 0), so (w ^ 0xAAAAAAAA) & (3 << 2j) * 0x01010101
//   gives bytes 4^j (t + 2) <= 48 for fields j = 0..2, still non-negative
//   int8; field 3 keeps the signed form 64 t (w & 0xC0C0C0C0, one AND).  Each
//   step accumulates into its own chain, whose sum is an exact multiple of
//   4^j; chain j >> 2j then holds sum (t + 2) x (j < 3) or sum t x (j = 3),
//   and the epilogue removes 2 * sum x over fields 0..2 exactly with the
//   prep's XSUM.
constexpr uint32_t kTop2 = 0xC0C0C0C0u;
__device__ __forceinline__ uint2 lo2(uint4 v) { return make_uint2(v.x, v.y); }
__device__ __forceinline__ uint2 hi2(uint4 v) { return make_uint2(v.z, v.w); }
__device__ __forceinline__ void unpack_signed(uint2 a, uint2 c, uint32_t (&A)[4][4]) {
#pragma unroll
  for (int j = 0; j < 4; j++) {
    const int sh = 6 - 2 * j;
    A[j][0] = (a.x << sh) & kTop2;
    A[j][1] = (c.x << sh) & kTop2;
    A[j][2] = (a.y << sh) & kTop2;
    A[j][3] = (c.y << sh) & kTop2;
  }
}
// (w ^ x) & M in one instruction: lop3 with the truth table of (a ^ c) & b
// (0x48 for a = 0xF0, b = 0xCC, c = 0xAA).
template <uint32_t M>
__device__ __forceinline__ uint32_t xor_and(uint32_t w, uint32_t x) {
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, 0x48;\n" : "=r"(d) : "r"(w), "n"(M), "r"(x));
  return d;
}
// X holds 0xAAAAAAAA (kept in a register by the caller: lop3 takes one
// immediate).
__device__ __forceinline__ void unpack_offset(uint2 a, uint2 c, uint32_t x,
                                              uint32_t (&A)[4][4]) {
  A[0][0] = xor_and<0x03030303u>(a.x, x); A[0][1] = xor_and<0x03030303u>(c.x, x);
  A[0][2] = xor_and<0x03030303u>(a.y, x); A[0][3] = xor_and<0x03030303u>(c.y, x);
  A[1][0] = xor_and<0x0C0C0C0Cu>(a.x, x); A[1][1] = xor_and<0x0C0C0C0Cu>(c.x, x);
  A[1][2] = xor_and<0x0C0C0C0Cu>(a.y, x); A[1][3] = xor_and<0x0C0C0C0Cu>(c.y, x);
  A[2][0] = xor_and<0x30303030u>(a.x, x); A[2][1] = xor_and<0x30303030u>(c.x, x);
  A[2][2] = xor_and<0x30303030u>(a.y, x); A[2][3] = xor_and<0x30303030u>(c.y, x);
  A[3][0] = a.x & kTop2; A[3][1] = c.x & kTop2;
  A[3][2] = a.y & kTop2; A[3][3] = c.y & kTop2;
}
__device__ __forceinline__ uint32_t offset_key() {
  uint32_t x;
  asm("mov.b32 %0, 0xAAAAAAAA;\n" : "=r"(x));
  return x;
}
// The four step chains of one output column of unpack_offset, unscaled:
// sum (t + 2) x over fields 0..2 plus sum t x over field 3 (exact).
__device__ __forceinline__ int offset_combine(int a0, int a1, int a2, int a3) {
  return a0 + (a1 >> 2) + (a2 >> 4) + (a3 >> 6);
}
}  // namespace nl

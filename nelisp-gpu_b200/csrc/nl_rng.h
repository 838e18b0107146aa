// nl_rng.h -- the counter-based generator the decoder's synthetic weights
// come from.  Every value is a pure function of (seed, tensor id, element
// index), so each tensor-parallel rank generates exactly its own shard from
// global indices, and a CPU model can regenerate the same numbers.
//
// mix64 is the splitmix64 finaliser (Steele, Lea and Flood, "Fast splittable
// pseudorandom number generators", OOPSLA 2014).
#pragma once

#include <stdint.h>

#if defined(__CUDACC__)
#define NL_HD __host__ __device__ __forceinline__
#else
#define NL_HD static inline
#endif

NL_HD uint64_t nl_mix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

// Per-tensor key.
NL_HD uint64_t nl_tensor_key(uint64_t seed, uint64_t tensor) {
  return nl_mix64(seed ^ nl_mix64(tensor * 0xD1B54A32D192ED03ull + 1u));
}

// 24 uniform bits for element I of a tensor.
NL_HD uint32_t nl_rand24(uint64_t key, uint64_t i) {
  return (uint32_t)(nl_mix64(key ^ i) >> 40);
}

// Uniform in [0, 1), exactly representable in f32.
NL_HD float nl_unit(uint64_t key, uint64_t i) {
  return (float)nl_rand24(key, i) * (1.0f / 16777216.0f);
}

// A trit -1, 0 or +1, each with probability 1/3 (up to 2^-24).
NL_HD int nl_trit(uint64_t key, uint64_t i) {
  return (int)((nl_rand24(key, i) * 3u) >> 24) - 1;
}

// Tensor ids of the decoder's parameters: per layer L, 16 ids from L*16.
enum {
  NL_T_WQ = 0, NL_T_WK = 1, NL_T_WV = 2, NL_T_WO = 3, NL_T_WGATE = 4, NL_T_WUP = 5,
  NL_T_WDOWN = 6, NL_T_SQ = 7, NL_T_SK = 8, NL_T_SV = 9, NL_T_SO = 10, NL_T_SGATE = 11,
  NL_T_SUP = 12, NL_T_SDOWN = 13, NL_T_ATTN_NORM = 14, NL_T_FFN_NORM = 15
};
#define NL_T_EMBED 1000000u
#define NL_T_FINAL_NORM 1000001u

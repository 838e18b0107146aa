// nl_step.h -- the decoder's decode step as one persistent kernel (nl_step.cu):
// its arguments and the shared-memory layout both sides compute.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace nl {

// Per-layer weights and caches of this rank (device pointers).
struct StepLayer {
  const uint32_t *wqkv, *wo, *wgu, *wd;
  const float *sqkv, *so, *sgu, *sd, *gattn, *gffn;
  float *ck, *cv;
};

struct StepArgs {
  const StepLayer *layers;          // [L], device memory
  uint32_t L, B, H, hd, hr, kvr, fr, maxseq, max_batch, qkv_rows;
  float eps, coef;
  uint32_t nsplit, chunk;           // attention split geometry (attn_geom)
  uint32_t dch;                     // K chunks of the down GEMV
  uint32_t nst;                     // ring stages the launch's shared memory holds
  const float *embed, *gfinal;
  const float2 *rope;               // [maxseq][hd/2] (cos, sin)
  float *hbuf;                      // [2][B][H] residual stream, two buffers
  float *qkv, *ctx, *o, *a;         // [B][qkv_rows], [B][hr*hd], [B][H], [B][fr]
  float *x_final;                   // [B][H] the LM head's input
  float *apart;                     // attention partials [B][hr][nsplit][hd + 2]
  unsigned *acnt;                   // [B * kvr] finished splits, reset by the merger
  unsigned *amax;                   // [B] max |a| (float bits)
  long long *dpart;                 // [dch][B][H] exact partial sums of the down GEMV
  const int *tok, *pos;
  unsigned long long *bar;          // grid barrier arrivals (never reset)
  unsigned long long *sep;          // step-kernel launches completed
  int *err;                         // a bounded wait gave up
};

// Shared memory of the step kernel, in bytes from a 128-byte-aligned base.
constexpr uint32_t kStepMaxK = 2560;                 // columns of one weight stage
constexpr uint32_t kStepRowPad = 4;                  // words of padding per staged row
constexpr uint32_t kStepStageBytes = 16u * (kStepMaxK / 16u + kStepRowPad) * 4u;   // 10496
constexpr uint32_t kStepMaxB = 8;
constexpr uint32_t kStepMaxStages = 32;

struct StepSmem {
  uint32_t ring, act, red, sacc, pre, total;
};

__host__ __device__ inline uint32_t step_align(uint32_t b) { return (b + 127u) & ~127u; }

// Offsets of the step kernel's shared memory for NST ring stages: the
// mbarriers, the ring, ACT (the activation fragments of one K chunk and the
// rows they are made from, or the attention merge scratch), RED / SACC (the cross-warp sums of a tile) and
// PRE (the prep's per-word partials and row statistics).
// Activation fragments of one K chunk: NT n-tiles of int8 limbs.
__host__ __device__ inline uint32_t step_frag_bytes(uint32_t NT) { return NT * kStepMaxK * 8u; }
// Sequence rows NT n-tiles hold at most (three limbs a row; four for up to four rows).
__host__ __device__ inline uint32_t step_rows(uint32_t NT) { return 8u * NT / 3u; }

__host__ __device__ inline StepSmem step_layout(uint32_t NT, uint32_t hd, uint32_t grp,
                                                uint32_t nst) {
  StepSmem s;
  // the fragments, then the staged rows they are made from
  uint32_t act = step_frag_bytes(NT) + step_rows(NT) * kStepMaxK * 4u;
  const uint32_t attn = 2u * (4u * grp * hd + 8u * grp) * 4u;
  if (attn > act) act = attn;
  s.ring = 2u * kStepMaxStages * 8u;
  s.act = s.ring + nst * kStepStageBytes;
  s.red = s.act + step_align(act);
  s.sacc = s.red + step_align(8u * NT * 4u * 32u * 4u);
  s.pre = s.sacc + step_align(2u * 16u * (8u * NT + 1u) * 4u);
  s.total = s.pre + step_align(kStepMaxB * (kStepMaxK / 16u) * 4u * 2u + 1024u);
  return s;
}
// Ring stages that fit in BUDGET bytes (at most kStepMaxStages).
__host__ __device__ inline uint32_t step_stages(uint32_t NT, uint32_t hd, uint32_t grp,
                                                uint32_t budget) {
  const uint32_t fixed = step_layout(NT, hd, grp, 0).total;
  uint32_t n = budget > fixed ? (budget - fixed) / kStepStageBytes : 0u;
  return n > kStepMaxStages ? kStepMaxStages : n;
}

// Grid barriers of one step: five per layer.
__host__ __device__ inline uint32_t step_barriers(uint32_t L) { return 5u * L; }

// Host side (nl_step.cu).
bool step_supported(uint32_t B, uint32_t H, uint32_t hd, uint32_t hr, uint32_t kvr, uint32_t fr,
                    int tp);
size_t step_dpart_bytes(uint32_t B, uint32_t H, uint32_t fr);
uint32_t step_down_chunks(uint32_t fr);
cudaError_t step_launch(const StepArgs &a, cudaStream_t st);
cudaError_t step_launch_h128(const StepArgs &a, cudaStream_t st);   // nl_step_h128.cu
cudaError_t step_launch_h64(const StepArgs &a, cudaStream_t st);    // nl_step_h64.cu

}  // namespace nl

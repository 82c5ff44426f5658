// Host interface of the sampler kernels (kernels/sampler.cu).
#pragma once
#include <cuda_runtime.h>
#include <cstdint>

namespace b200 {

struct SampleArgs {
  const float* temperature;  // [B]; < 1e-3 = greedy row
  const int* top_k;          // [B] or null; -1 = off
  const float* top_p;        // [B] or null
  const float* min_p;        // [B] or null
  const int64_t* seeds;      // [B] Philox key per row
  const int64_t* offsets;    // [B] Philox counter word (step index) or null
  // allowed-token bitmasks (guided decoding): row b uses mask allow_row[b]
  // (-1 = unconstrained) of `allow` [n_masks, mask_words]; both null = none
  const uint32_t* allow;
  const int* allow_row;
  int mask_words;
  // log-probabilities of the distribution each row samples from (greedy rows:
  // the raw logits under the mask): the lp_k most likely tokens (value, id),
  // best first, and the chosen token's; lp_k = 0 = none, at most kMaxLogprobs
  int lp_k;
  float* lp_top_v;           // [B, lp_k]
  int* lp_top_i;             // [B, lp_k]; -1 where fewer than lp_k tokens survive
  float* lp_chosen;          // [B]
};

constexpr int kMaxLogprobs = 20;

void argmax_rows(const float* logits, int B, int V, int64_t ld, int* out, cudaStream_t s);
void sample_rows(const float* logits, int B, int V, int64_t ld, const SampleArgs& a, int* out, cudaStream_t s);
void apply_penalties(float* logits, int64_t ld, const int* rows, const int* ids, const int* gen_counts,
                     const float* presence, const float* frequency, const float* repetition, int n,
                     cudaStream_t s);

}  // namespace b200

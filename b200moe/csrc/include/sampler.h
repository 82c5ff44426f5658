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
};

void argmax_rows(const float* logits, int B, int V, int64_t ld, int* out, cudaStream_t s);
void sample_rows(const float* logits, int B, int V, int64_t ld, const SampleArgs& a, int* out, cudaStream_t s);
void apply_penalties(float* logits, int64_t ld, const int* rows, const int* ids, const int* gen_counts,
                     const float* presence, const float* frequency, const float* repetition, int n,
                     cudaStream_t s);

}  // namespace b200

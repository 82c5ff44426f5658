// Host interface of the tensor-parallel sums over NVLink peer memory (kernels/tp_comm.cu).
#pragma once
#include <cuda_runtime.h>
#include <cstdint>

namespace b200 {

constexpr int kTpMaxWorld = 8;

// One all-reduce step of the tensor-parallel attention path.  Every rank holds its
// fp32 partial [splits, T, H] in `part[rank]`; all ranks' buffers are mapped here.
struct TpArgs {
  int world;
  int rank;
  const float* part[kTpMaxWorld];  // each rank's partial buffer (peer mappings; part[rank] is local)
  int splits;                      // partials per rank (split-K GEMM), summed with the ranks
  long long split_stride;          // floats between splits
  uint32_t* flags[kTpMaxWorld];    // each rank's flag array [world]; rank s releases into flags[r][s]
  uint32_t* epoch;                 // local: all-reduce steps completed
  int* counter;                    // local CTA counter, zero between launches
  int* status;
  unsigned long long* wait_ns;     // [world] ns waited on each rank, or null
};

// part[rank][t] = sum_k slots[t * topk + k] in fp32 (fixed order), then the last CTA
// releases *epoch + 1 into every rank's flags[.][rank].
void tp_slots_partial(const TpArgs& a, const void* slots, int topk, int T, int H, cudaStream_t s);

// Waits (bounded) until every rank released *epoch + 1, then per token:
//   residual += bf16(sum over ranks r = 0..W-1, splits s of part[r][s][t])   (fixed order)
//   out = rmsnorm(residual) * w
// and the last CTA sets *epoch += 1.  Every rank computes the same sum in the same
// order, so the replicated residual stream stays bit-identical across ranks.
void tp_allreduce_rmsnorm(const TpArgs& a, void* residual, const void* w, void* out, int T, int H, float eps,
                          cudaStream_t s);

}  // namespace b200

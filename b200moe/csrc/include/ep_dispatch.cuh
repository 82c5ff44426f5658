// Device side of the expert-parallel dispatch, shared by ep_dispatch_kernel
// (kernels/ep_p2p.cu) and the router kernel that dispatches its own top-k rows
// (router_fused_kernel, kernels/fused_ops.cu):
//
//   ep_claim        one routed (token, k) row claims a position in the owner's
//                   segment for this source and an index among this source's rows
//                   for the expert (one thread per row: a token's rows claim together)
//   ep_store_row    the row and its metadata as plain 16-byte stores into the
//                   owner's memory (warp-collective); ep_send_row / ep_send_token
//                   combine the two for one row or for all of one token's rows
//   ep_block_arrive every block that sent rows arrives on a grid counter; true in
//                   every thread of the last one (block-collective)
//   ep_publish      the last block writes this source's per-expert row counts into
//                   every owner's count matrix, releases the epoch flags and
//                   resets the scratch for the next layer (block-collective)
//
// Publication takes one system-scope acq_rel fence per block: the block barrier
// orders the block's stores before the fencing thread, and fences are cumulative.
#pragma once
#include <cuda_bf16.h>
#include <cstdint>

#include "sm100.cuh"
#include "ep_sync.cuh"
#include "ep_p2p.h"

namespace b200 {

// A claimed position for one routed row: the owner, the row in the owner's segment
// for this source, and the row's index among this source's rows for the expert.
struct EpClaim {
  int dest, pos, idx;
};

// Called by one thread per routed row (independent rows claim in parallel).
__device__ __forceinline__ EpClaim ep_claim(const EpArgs& a, int ge) {
  EpClaim c{0, a.cap, 0};  // pos == cap: nothing is written
  if (ge < 0 || ge >= a.num_experts) {
    record_status(a.status, kStatusBadShape);
    return c;
  }
  c.dest = a.owner[ge];
  c.pos = atomicAdd(&a.send_cursor[c.dest], 1);
  c.idx = atomicAdd(&a.ecur[ge], 1);
  if (c.pos >= a.cap) record_status(a.status, kStatusBadShape);  // the host sizes cap for the worst case
  return c;
}

// Warp-collective: store the claimed row (16-byte stores into the owner's memory) and
// its metadata.  p = token * topk + k (the combine slot); every argument is warp-uniform.
__device__ __forceinline__ void ep_store_row(const EpArgs& a, const __nv_bfloat16* __restrict__ xrow, int p, int ge,
                                             float wt, EpClaim c, int lane) {
  if (c.pos >= a.cap) return;
  const int64_t row = (int64_t)a.rank * a.cap + c.pos;
  const uint4* src = reinterpret_cast<const uint4*>(xrow);
  uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(a.recv_x[c.dest]) + row * a.hidden);
  for (int i = lane; i < a.hidden / 8; i += 32) dst[i] = src[i];
  if (lane == 0) reinterpret_cast<int4*>(a.recv_meta[c.dest])[row] = make_int4(ge, p, __float_as_int(wt), c.idx);
}

// One routed row per warp (lane 0 claims).
__device__ __forceinline__ void ep_send_row(const EpArgs& a, const __nv_bfloat16* __restrict__ xrow, int p, int ge,
                                            float wt, int lane) {
  EpClaim c{0, 0, 0};
  if (lane == 0) c = ep_claim(a, ge);
  c.dest = __shfl_sync(0xffffffffu, c.dest, 0);
  c.pos = __shfl_sync(0xffffffffu, c.pos, 0);
  c.idx = __shfl_sync(0xffffffffu, c.idx, 0);
  ep_store_row(a, xrow, p, ge, wt, c, lane);
}

// All of one token's routed rows by one warp: lane k < topk holds the token's k-th
// expert (ge) and weight (wt); the topk claims go out together, then the rows.
__device__ __forceinline__ void ep_send_token(const EpArgs& a, const __nv_bfloat16* __restrict__ xrow, int tok,
                                              int topk, int ge, float wt, int lane) {
  EpClaim c{0, 0, 0};
  if (lane < topk) c = ep_claim(a, ge);
  for (int k = 0; k < topk; ++k) {
    EpClaim ck;
    ck.dest = __shfl_sync(0xffffffffu, c.dest, k);
    ck.pos = __shfl_sync(0xffffffffu, c.pos, k);
    ck.idx = __shfl_sync(0xffffffffu, c.idx, k);
    ep_store_row(a, xrow, tok * topk + k, __shfl_sync(0xffffffffu, ge, k), __shfl_sync(0xffffffffu, wt, k), ck, lane);
  }
}

// All threads of every participating block call it once, after their rows; `nblocks`
// blocks participate.  `last_s` is a shared int.
__device__ __forceinline__ bool ep_block_arrive(const EpArgs& a, int nblocks, int* last_s) {
  __syncthreads();
  if (threadIdx.x == 0) {
    fence_acq_rel_sys();
    const bool last = atomicAdd(a.done_blocks, 1) == nblocks - 1;
    if (last) fence_acq_rel_sys();  // every other block's rows, seen through the counter
    *last_s = last;
  }
  __syncthreads();
  return *last_s != 0;
}

// Called by every thread of the last block only.
__device__ __forceinline__ void ep_publish(const EpArgs& a, uint32_t epoch) {
  for (int ge = threadIdx.x; ge < a.num_experts; ge += blockDim.x) {
    const int dest = a.owner[ge];
    volatile int* cnt = reinterpret_cast<volatile int*>(a.counts[dest]);
    cnt[a.rank * a.num_local + a.ge_local[ge]] = atomicAdd(&a.ecur[ge], 0);
    a.ecur[ge] = 0;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    fence_acq_rel_sys();
    for (int r = 0; r < a.world; ++r) st_release_sys(reinterpret_cast<uint32_t*>(a.flags[r]) + a.rank, epoch);
    for (int r = 0; r < a.world; ++r) a.send_cursor[r] = 0;
    *a.done_blocks = 0;
    *a.epoch = epoch;
  }
}

}  // namespace b200

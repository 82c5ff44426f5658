// Device side of the expert-parallel dispatch, shared by ep_dispatch_kernel
// (kernels/ep_p2p.cu) and the router kernel that dispatches its own top-k rows
// (router_fused_kernel, kernels/fused_ops.cu):
//
//   ep_send_row     one routed (token, k) row: claim a position in the owner's
//                   segment for this source and an index among this source's rows
//                   for the expert, store the row and its metadata with plain
//                   16-byte stores into the owner's memory (warp-collective)
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

// p = token * topk + k (the combine slot); ge / wt are warp-uniform.
__device__ __forceinline__ void ep_send_row(const EpArgs& a, const __nv_bfloat16* __restrict__ xrow, int p, int ge,
                                            float wt, int lane) {
  if (ge < 0 || ge >= a.num_experts) {
    if (lane == 0) record_status(a.status, kStatusBadShape);
    return;
  }
  const int dest = a.owner[ge];
  int pos = 0, idx = 0;
  if (lane == 0) {
    pos = atomicAdd(&a.send_cursor[dest], 1);
    idx = atomicAdd(&a.ecur[ge], 1);
  }
  pos = __shfl_sync(0xffffffffu, pos, 0);
  idx = __shfl_sync(0xffffffffu, idx, 0);
  if (pos >= a.cap) {  // the host sizes cap for the worst case; never write past it
    if (lane == 0) record_status(a.status, kStatusBadShape);
    return;
  }
  const int64_t row = (int64_t)a.rank * a.cap + pos;
  const uint4* src = reinterpret_cast<const uint4*>(xrow);
  uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(a.recv_x[dest]) + row * a.hidden);
  for (int i = lane; i < a.hidden / 8; i += 32) dst[i] = src[i];
  if (lane == 0) reinterpret_cast<int4*>(a.recv_meta[dest])[row] = make_int4(ge, p, __float_as_int(wt), idx);
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

// Expert-parallel dispatch / combine over NVLink peer memory (sm_100a).
//
// Every rank owns a symmetric set of buffers (same layout on all ranks, peers'
// copies mapped into this process):
//   recv_x    [W * cap, H] bf16   rows routed to this rank's experts, segment per source
//   recv_meta [W * cap, 4] int32  (global expert, source slot, weight bits, index among
//                                 the source's rows for that expert)
//   counts    [W * El] int32      rows from each source for each local expert
//   flags     [W] uint32          dispatch epoch written by each source
//   done      [W] uint32          combine epoch written by each expert owner
//   slots     [cap, H] bf16       this rank's (token, k) slots, written by owners
//
// Per MoE layer: five stream-ordered launches, no host sync, graph-capturable.
//   ep_dispatch   warp per routed (token, k): claim a position in the owner's
//                 segment for this source and an index among this source's rows
//                 for the expert, store the row and its metadata with plain
//                 16-byte stores into the peer's memory; the last block writes
//                 this source's per-expert counts into every owner's count
//                 matrix and releases the epoch flag (release, system scope).
//   ep_scatter    owner side: every block waits (bounded) for every source's
//                 flag, derives expert offsets from the count matrix (no
//                 counting pass), and copies each received row straight to its
//                 expert-sorted position with its combine address and weight;
//                 block 0 publishes the per-expert counts and offsets.
//   gemm_tc x 2   gate/up + SiLU, then down whose epilogue writes each weighted
//                 row straight into the source rank's slots (peer stores); the
//                 down GEMM's last CTA releases this rank's done epoch to every
//                 source.
//   moe_combine   source side: waits (bounded) for every owner's done epoch, then
//                 the fixed-order top-k sum + residual + next RMSNorm on local memory.
//
// Epochs live in device memory (incremented by ep_dispatch), so a replayed CUDA
// graph keeps advancing them.  All waits are bounded (%globaltimer); on expiry
// the kernel records a status code and returns.  Peer memory is accessed with
// plain ld/st only (no TMA).  ep_signal / ep_wait_done are the stand-alone forms
// of the release and the wait.
//
// Reference: the replicated-hidden all_reduce combine of
// nanovllm/models/qwen3_moe.py:414-418 (one NCCL all-reduce per layer).
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <algorithm>
#include <cstdint>
#include <stdexcept>
#include <string>

#include "sm100.cuh"
#include "ep_sync.cuh"
#include "ep_p2p.h"
#include "ep_dispatch.cuh"

namespace b200 {

__global__ void ep_dispatch_kernel(const EpArgs a, const __nv_bfloat16* __restrict__ x, const int* __restrict__ ids,
                                   const float* __restrict__ w, int T, int topk) {
  __shared__ uint32_t epoch_s;
  __shared__ int last_s;
  if (threadIdx.x == 0) epoch_s = *a.epoch + 1;
  __syncthreads();
  const uint32_t epoch = epoch_s;
  const int warps = blockDim.x >> 5;
  const int lane = threadIdx.x & 31;
  for (int p = blockIdx.x * warps + (threadIdx.x >> 5); p < T * topk; p += gridDim.x * warps)
    ep_send_row(a, x + (int64_t)(p / topk) * a.hidden, p, ids[p], w[p], lane);
  if (ep_block_arrive(a, gridDim.x, &last_s)) ep_publish(a, epoch);
}

// Owner side.  Every block waits for every source, then places each received row at
//   offset[expert] + (rows of that expert from lower-numbered sources) + its index
// among its source's rows for the expert, all read from the count matrix: the layout
// is the same whatever the arrival order.  One warp per row.
__global__ void ep_scatter_kernel(const EpArgs a, int* __restrict__ local_counts, __nv_bfloat16* __restrict__ x_perm,
                                  int* __restrict__ slot_code, float* __restrict__ slot_w,
                                  int* __restrict__ offsets_out) {
  __shared__ int offs[kEpMaxLocalExperts + 1];
  __shared__ int base[kEpMaxWorld * kEpMaxLocalExperts];  // rows of expert e from sources < s, at s * El + e
  __shared__ int seg[kEpMaxWorld + 1];
  __shared__ int src_rows[kEpMaxWorld];
  __shared__ int ok_s;
  const int W = a.world, El = a.num_local;
  const uint32_t epoch = *a.epoch;
  const uint32_t* my_flags = reinterpret_cast<const uint32_t*>(a.flags[a.rank]);
  if (threadIdx.x == 0) ok_s = 1;
  __syncthreads();
  if (threadIdx.x < W) {
    // block 0 charges the wait to the source it waited for (the wait accounting)
    if (!wait_epoch(my_flags + threadIdx.x, epoch, a.status,
                    (blockIdx.x == 0 && a.wait_ns) ? a.wait_ns + threadIdx.x : nullptr))
      ok_s = 0;
  }
  __syncthreads();
  if (!ok_s) {  // a source never arrived (status recorded): leave the layer's expert work empty
    if (blockIdx.x == 0)
      for (int e = threadIdx.x; e <= El; e += blockDim.x) {
        if (offsets_out != nullptr) offsets_out[e] = 0;
        if (e < El) local_counts[e] = 0;
      }
    return;
  }
  const volatile int* cnt = reinterpret_cast<const volatile int*>(a.counts[a.rank]);
  if (threadIdx.x < W) src_rows[threadIdx.x] = 0;
  __syncthreads();
  // per expert: sources in order (rank-major prefix), then the expert prefix.  Each
  // count is read once, by the thread of its expert (the W loads are independent);
  // the per-source row totals are summed in shared memory, not by one thread.
  for (int e = threadIdx.x; e < El; e += blockDim.x) {
    int c[kEpMaxWorld];
#pragma unroll
    for (int src = 0; src < kEpMaxWorld; ++src) c[src] = src < W ? cnt[src * El + e] : 0;
    int run = 0;
#pragma unroll
    for (int src = 0; src < kEpMaxWorld; ++src) {
      if (src < W) {
        base[src * El + e] = run;
        run += c[src];
        atomicAdd(&src_rows[src], c[src]);
      }
    }
    offs[e] = run;  // total of expert e, turned into the prefix below
  }
  __syncthreads();
  if (threadIdx.x < 32) {  // expert prefix by one warp (shared memory), source segments by lane 0
    const int lane = threadIdx.x;
    int carry = 0;
    for (int e0 = 0; e0 < El; e0 += 32) {
      const int e = e0 + lane;
      const int n = e < El ? offs[e] : 0;
      int incl = n;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
      }
      if (e < El) offs[e] = carry + incl - n;
      carry += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (lane == 0) {
      offs[El] = carry;
      int r = 0;
      for (int src = 0; src < W; ++src) {
        seg[src] = r;
        r += min(src_rows[src], a.cap);
      }
      seg[W] = r;
    }
  }
  __syncthreads();
  if (blockIdx.x == 0) {
    for (int e = threadIdx.x; e <= El; e += blockDim.x) {
      if (offsets_out != nullptr) offsets_out[e] = offs[e];
      if (e < El) local_counts[e] = offs[e + 1] - offs[e];
    }
  }
  const int lane = threadIdx.x & 31;
  const int total = seg[W];
  const int H8 = a.hidden / 8;
  for (int i = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); i < total; i += gridDim.x * (blockDim.x >> 5)) {
    int src = 0;
    while (seg[src + 1] <= i) ++src;
    const int64_t row = (int64_t)src * a.cap + (i - seg[src]);
    const int4 m = reinterpret_cast<const int4*>(a.recv_meta[a.rank])[row];
    const int le = (m.x >= 0 && m.x < a.num_experts) ? a.g2l[m.x] : -1;
    if (le < 0) {
      if (lane == 0) record_status(a.status, kStatusBadShape);
      continue;
    }
    const int pos = offs[le] + base[src * El + le] + m.w;
    if (m.w < 0 || pos >= offs[le + 1]) {
      if (lane == 0) record_status(a.status, kStatusBadShape);
      continue;
    }
    const uint4* s = reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(a.recv_x[a.rank]) +
                                                    row * a.hidden);
    uint4* d = reinterpret_cast<uint4*>(x_perm + (int64_t)pos * a.hidden);
    for (int j = lane; j < H8; j += 32) d[j] = s[j];
    if (lane == 0) {
      slot_code[pos] = src * a.slot_cap + m.y;   // combine target: (source rank, slot)
      slot_w[pos] = __int_as_float(m.z);
    }
  }
}

__global__ void ep_signal_kernel(const EpArgs a) {
  const int r = threadIdx.x;
  const uint32_t epoch = *a.epoch;
  fence_acq_rel_sys();
  if (r < a.world) st_release_sys(reinterpret_cast<uint32_t*>(a.done[r]) + a.rank, epoch);
}

__global__ void ep_wait_done_kernel(const EpArgs a) {
  const int r = threadIdx.x;
  const uint32_t epoch = *a.epoch;
  if (r < a.world)
    wait_epoch(reinterpret_cast<const uint32_t*>(a.done[a.rank]) + r, epoch, a.status,
               a.wait_ns ? a.wait_ns + a.world + r : nullptr);
  __syncthreads();
}

static void check(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

static void check_args(const EpArgs& a) {
  if (a.world < 1 || a.world > kEpMaxWorld) throw std::runtime_error("ep: world size out of range");
  if (a.hidden % 8) throw std::runtime_error("ep: hidden % 8");
}

void ep_dispatch(const EpArgs& a, const void* x, const int* ids, const float* w, int T, int topk, cudaStream_t s) {
  check_args(a);
  const int warps = 8;
  const int blocks = std::max(1, std::min(1024, (T * topk + warps - 1) / warps));
  ep_dispatch_kernel<<<blocks, warps * 32, 0, s>>>(a, static_cast<const __nv_bfloat16*>(x), ids, w, T, topk);
  check("ep_dispatch");
}

void ep_scatter(const EpArgs& a, int* local_counts, void* x_perm, int* slot_code, float* slot_w, int* offsets_out,
                int max_rows, cudaStream_t s) {
  check_args(a);
  if (a.num_local < 1 || a.num_local > kEpMaxLocalExperts) throw std::runtime_error("ep: local experts out of range");
  // two blocks per SM walk the rows grid-stride: every block waits and reads the
  // count matrix, so fewer blocks mean less redundant work at decode sizes
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int blocks = std::max(1, std::min(2 * sms, (max_rows + 7) / 8));
  ep_scatter_kernel<<<blocks, 256, 0, s>>>(a, local_counts, static_cast<__nv_bfloat16*>(x_perm), slot_code, slot_w,
                                           offsets_out);
  check("ep_scatter");
}

void ep_signal(const EpArgs& a, cudaStream_t s) {
  ep_signal_kernel<<<1, 32, 0, s>>>(a);
  check("ep_signal");
}

void ep_wait_done(const EpArgs& a, cudaStream_t s) {
  ep_wait_done_kernel<<<1, 32, 0, s>>>(a);
  check("ep_wait_done");
}

}  // namespace b200

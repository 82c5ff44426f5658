// Expert-parallel dispatch / combine over NVLink peer memory (sm_100a).
//
// Every rank owns a symmetric set of buffers (same layout on all ranks, peers'
// copies mapped into this process):
//   recv_x    [W * cap, H] bf16   rows routed to this rank's experts, segment per source
//   recv_meta [W * cap, 4] int32  (global expert, source slot, weight bits, -)
//   counts    [W] int32           rows received from each source
//   flags     [W] uint32          dispatch epoch written by each source
//   done      [W] uint32          combine epoch written by each expert owner
//   slots     [cap, H] bf16       this rank's (token, k) slots, written by owners
//
// Per MoE layer (all launches stream-ordered, no host sync, graph-capturable):
//   ep_dispatch   warp per routed (token, k): claim a position in the owner's
//                 segment for this source, store the row and its metadata with
//                 plain 16-byte stores into the peer's memory; the last block
//                 publishes counts and the epoch flag (release, system scope).
//   ep_count      owner side: bounded wait for every source's flag, count the
//                 received rows per local expert.
//   ep_scatter    owner side: expert-sorted copy of the received rows (local)
//                 plus the combine address (source, slot) and routing weight.
//   gemm_tc x 2   gate/up + SiLU, then down whose epilogue writes each weighted
//                 row straight into the source rank's slots (peer stores).
//   ep_signal     owner side: release the done epoch to every source.
//   ep_wait_done  source side: bounded wait for every owner's done epoch; then
//                 the usual fixed-order moe_combine runs on local memory.
//
// Epochs live in device memory (incremented by ep_dispatch), so a replayed CUDA
// graph keeps advancing them.  All waits are bounded (%globaltimer); on expiry
// the kernel records a status code and returns.  Peer memory is accessed with
// plain ld/st only (no TMA).
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
#include "ep_p2p.h"

namespace b200 {

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Bounded wait until *p >= want (wrap-safe compare).  False on timeout.  The
// time spent is added to *waited (when not null).
__device__ __forceinline__ bool wait_epoch(const uint32_t* p, uint32_t want, int* status,
                                           unsigned long long* waited) {
  const uint64_t t0 = globaltimer_ns();
  bool ok = true;
  while ((int32_t)(ld_acquire_sys(p) - want) < 0) {
    if (globaltimer_ns() - t0 > kWaitLimitNs) {
      record_status(status, kStatusTimeoutFlag);
      ok = false;
      break;
    }
    __nanosleep(64);
  }
  if (waited != nullptr) atomicAdd(waited, (unsigned long long)(globaltimer_ns() - t0));
  return ok;
}

__global__ void ep_dispatch_kernel(const EpArgs a, const __nv_bfloat16* __restrict__ x, const int* __restrict__ ids,
                                   const float* __restrict__ w, int T, int topk) {
  __shared__ uint32_t epoch_s;
  __shared__ int last_s;
  if (threadIdx.x == 0) epoch_s = *a.epoch + 1;
  __syncthreads();
  const uint32_t epoch = epoch_s;
  const int warps = blockDim.x >> 5;
  const int lane = threadIdx.x & 31;
  const int H8 = a.hidden / 8;
  for (int p = blockIdx.x * warps + (threadIdx.x >> 5); p < T * topk; p += gridDim.x * warps) {
    const int ge = ids[p];
    const int dest = a.owner[ge];
    int pos = 0;
    if (lane == 0) pos = atomicAdd(&a.send_cursor[dest], 1);
    pos = __shfl_sync(0xffffffffu, pos, 0);
    if (pos >= a.cap) {  // the host sizes cap for the worst case; never write past it
      if (lane == 0) record_status(a.status, kStatusBadShape);
      continue;
    }
    const int64_t row = (int64_t)a.rank * a.cap + pos;
    const uint4* src = reinterpret_cast<const uint4*>(x + (int64_t)(p / topk) * a.hidden);
    uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(a.recv_x[dest]) + row * a.hidden);
    for (int i = lane; i < H8; i += 32) dst[i] = src[i];
    if (lane == 0) {
      int4 m = make_int4(ge, p, __float_as_int(w[p]), 0);
      reinterpret_cast<int4*>(a.recv_meta[dest])[row] = m;
    }
  }
  __threadfence_system();  // every thread orders its own peer stores before the block's arrival
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    last_s = atomicAdd(a.done_blocks, 1) == (int)gridDim.x - 1;
  }
  __syncthreads();
  if (last_s && threadIdx.x == 0) {
    __threadfence_system();
    for (int r = 0; r < a.world; ++r) {
      const int n = min(atomicAdd(&a.send_cursor[r], 0), a.cap);
      volatile int* cnt = reinterpret_cast<volatile int*>(a.counts[r]);
      cnt[a.rank] = n;
    }
    __threadfence_system();
    for (int r = 0; r < a.world; ++r) st_release_sys(reinterpret_cast<uint32_t*>(a.flags[r]) + a.rank, epoch);
    for (int r = 0; r < a.world; ++r) a.send_cursor[r] = 0;
    *a.done_blocks = 0;
    *a.epoch = epoch;
  }
}

// One block per source segment: wait for the source's epoch, count rows per local expert.
__global__ void ep_count_kernel(const EpArgs a, int* __restrict__ local_counts) {
  __shared__ int ok_s;
  __shared__ int n_s;
  const int src = blockIdx.x;
  const uint32_t epoch = *a.epoch;
  uint32_t* my_flags = reinterpret_cast<uint32_t*>(a.flags[a.rank]);
  if (threadIdx.x == 0) {
    ok_s = wait_epoch(my_flags + src, epoch, a.status, a.wait_ns ? a.wait_ns + src : nullptr) ? 1 : 0;
    n_s = ok_s ? reinterpret_cast<volatile int*>(a.counts[a.rank])[src] : 0;
  }
  __syncthreads();
  const int n = n_s;
  const int4* meta = reinterpret_cast<const int4*>(a.recv_meta[a.rank]) + (int64_t)src * a.cap;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const int le = a.g2l[meta[i].x];
    if (le >= 0) atomicAdd(&local_counts[le], 1);
  }
}

// Expert-sorted copy of the received rows; one warp per row.
__global__ void ep_scatter_kernel(const EpArgs a, const int* __restrict__ local_counts, int* __restrict__ cursor,
                                  int num_local, __nv_bfloat16* __restrict__ x_perm, int* __restrict__ slot_code,
                                  float* __restrict__ slot_w, int* __restrict__ offsets_out) {
  __shared__ int offs[kEpMaxLocalExperts + 1];
  __shared__ int seg[kEpMaxWorld + 1];
  if (threadIdx.x == 0) {
    int s = 0;
    for (int e = 0; e < num_local; ++e) { offs[e] = s; s += local_counts[e]; }
    offs[num_local] = s;
    int r = 0;
    const volatile int* cnt = reinterpret_cast<const volatile int*>(a.counts[a.rank]);
    for (int src = 0; src < a.world; ++src) { seg[src] = r; r += cnt[src]; }
    seg[a.world] = r;
  }
  __syncthreads();
  if (blockIdx.x == 0 && offsets_out != nullptr)
    for (int e = threadIdx.x; e <= num_local; e += blockDim.x) offsets_out[e] = offs[e];
  const int lane = threadIdx.x & 31;
  const int total = seg[a.world];
  const int H8 = a.hidden / 8;
  for (int i = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); i < total; i += gridDim.x * (blockDim.x >> 5)) {
    int src = 0;
    while (seg[src + 1] <= i) ++src;
    const int64_t row = (int64_t)src * a.cap + (i - seg[src]);
    const int4 m = reinterpret_cast<const int4*>(a.recv_meta[a.rank])[row];
    const int le = a.g2l[m.x];
    if (le < 0) continue;
    int pos = 0;
    if (lane == 0) pos = offs[le] + atomicAdd(&cursor[le], 1);
    pos = __shfl_sync(0xffffffffu, pos, 0);
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
  __threadfence_system();
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

void ep_count(const EpArgs& a, int* local_counts, cudaStream_t s) {
  check_args(a);
  ep_count_kernel<<<a.world, 256, 0, s>>>(a, local_counts);
  check("ep_count");
}

void ep_scatter(const EpArgs& a, const int* local_counts, int* cursor, int num_local, void* x_perm, int* slot_code,
                float* slot_w, int* offsets_out, int max_rows, cudaStream_t s) {
  check_args(a);
  if (num_local > kEpMaxLocalExperts) throw std::runtime_error("ep: too many local experts");
  const int blocks = std::max(1, std::min(2048, (max_rows + 7) / 8));
  ep_scatter_kernel<<<blocks, 256, 0, s>>>(a, local_counts, cursor, num_local,
                                           static_cast<__nv_bfloat16*>(x_perm), slot_code, slot_w, offsets_out);
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

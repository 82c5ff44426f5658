// Tensor-parallel all-reduce fused into its consumer, over NVLink peer memory (sm_100a).
//
// In tensor-parallel attention every rank holds all T tokens and a slice of the
// heads (and of the experts), so after the O projection and after the MoE each
// rank has a partial sum of the layer's output that all ranks need in full.  The
// reference all-reduces it with NCCL and then runs the residual RMSNorm
// (nanovllm/layers/linear.py:152-160, nanovllm/models/qwen3_moe.py:414-418).
// Here the producer writes its fp32 partial into a buffer every peer has mapped
// and releases an epoch; the consumer -- the residual RMSNorm -- waits for every
// rank's epoch, reads the W partials of its token over NVLink with plain 16-byte
// loads, sums them in rank order, adds the residual and normalises:
//
//   O GEMM (split-K fp32 partials, last CTA releases)    -> tp_allreduce_rmsnorm
//   MoE down GEMM -> tp_slots_partial (k-sum, release)   -> tp_allreduce_rmsnorm
//
// Bytes over NVLink per rank and step: (W - 1) * T * H * 4 (every rank reads every
// peer's partial of every token), which is what keeps the residual replicated
// without a second exchange; the caller uses this path for decode-size batches
// and NCCL for large prefill batches.  Buffers are double-buffered by the caller
// (a peer can be at most one step ahead), waits are bounded by %globaltimer and
// record a status code, and no TMA or library kernel touches peer memory.
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cstdint>
#include <stdexcept>
#include <string>

#include "sm100.cuh"
#include "pdl.cuh"
#include "ep_sync.cuh"
#include "tp_comm.h"

namespace b200 {

namespace {

using bf16 = __nv_bfloat16;

__device__ __forceinline__ float bf16r(float x) { return __bfloat162float(__float2bfloat16(x)); }

__device__ __forceinline__ void unpack8(const uint4 u, float* f) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 v = __bfloat1622float2(h[i]);
    f[2 * i] = v.x;
    f[2 * i + 1] = v.y;
  }
}

__device__ __forceinline__ uint4 pack8(const float* f) {
  uint4 u;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
  return u;
}

constexpr int kInFlight = 8;  // partial loads in flight per thread

template <int NT>
__device__ __forceinline__ float block_sum(float v, float* red) {
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) red[w] = v;
  __syncthreads();
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < NT / 32; ++i) s += red[i];
  return s;
}

// The last CTA of the grid to get here runs `fn`.  SYS: every CTA's stores are
// published at system scope first (fn releases them to peers) -- the barrier orders
// the CTA's stores before thread 0's fence, which is cumulative, so one fence per
// CTA suffices; otherwise fn only needs every CTA to have arrived.
template <bool SYS, typename F>
__device__ __forceinline__ void last_cta(int* counter, F fn) {
  __syncthreads();
  if (threadIdx.x == 0) {
    if constexpr (SYS) fence_acq_rel_sys();
    else __threadfence();
    if (atomicAdd(counter, 1) == (int)gridDim.x - 1) {
      *counter = 0;
      if constexpr (SYS) fence_acq_rel_sys();
      fn();
    }
  }
}

template <int NT, int VPT>
__global__ void __launch_bounds__(NT) tp_slots_partial_kernel(TpArgs a, const bf16* __restrict__ slots, int topk,
                                                              int T, int H) {
  pdl_enter();
  const int t = blockIdx.x;
  if (t < T) {
    float* dst = const_cast<float*>(a.part[a.rank]) + (size_t)t * H;
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      const int idx = (threadIdx.x + j * NT) * 8;
      float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      for (int k = 0; k < topk; ++k) {
        float s[8];
        unpack8(*reinterpret_cast<const uint4*>(slots + ((size_t)t * topk + k) * H + idx), s);
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[e] += s[e];
      }
      *reinterpret_cast<float4*>(dst + idx) = make_float4(acc[0], acc[1], acc[2], acc[3]);
      *reinterpret_cast<float4*>(dst + idx + 4) = make_float4(acc[4], acc[5], acc[6], acc[7]);
    }
  }
  last_cta<true>(a.counter, [&] {
    const uint32_t e = *a.epoch + 1;
    for (int r = 0; r < a.world; ++r) st_release_sys(a.flags[r] + a.rank, e);
  });
  pdl_trigger();
}

template <int NT, int VPT>
__global__ void __launch_bounds__(NT) tp_allreduce_rmsnorm_kernel(TpArgs a, bf16* residual, const bf16* __restrict__ w,
                                                                  bf16* __restrict__ out, int T, int H, float eps) {
  pdl_enter();
  __shared__ float red[NT / 32];
  const uint32_t want = *a.epoch + 1;
  if (threadIdx.x < a.world)
    wait_epoch(a.flags[a.rank] + threadIdx.x, want, a.status,
               (blockIdx.x == 0 && a.wait_ns) ? a.wait_ns + threadIdx.x : nullptr);
  __syncthreads();
  const int t = blockIdx.x;
  if (t < T) {
    const size_t base = (size_t)t * H;
    float v[VPT][8];
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      const int idx = (threadIdx.x + j * NT) * 8;
      float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      // partial p = rank * splits + split, summed in that order; a batch of kInFlight
      // loads is issued before any add, so peer round trips overlap
      const int np = a.world * a.splits;
      for (int p0 = 0; p0 < np; p0 += kInFlight) {
        float4 x0[kInFlight], x1[kInFlight];
#pragma unroll
        for (int i = 0; i < kInFlight; ++i) {
          const int pi = p0 + i;
          if (pi < np) {
            const int r = pi / a.splits, sp = pi - r * a.splits;
            const float* p = a.part[r] + sp * a.split_stride + base + idx;
            x0[i] = *reinterpret_cast<const float4*>(p);
            x1[i] = *reinterpret_cast<const float4*>(p + 4);
          }
        }
#pragma unroll
        for (int i = 0; i < kInFlight; ++i) {
          if (p0 + i < np) {
            acc[0] += x0[i].x; acc[1] += x0[i].y; acc[2] += x0[i].z; acc[3] += x0[i].w;
            acc[4] += x1[i].x; acc[5] += x1[i].y; acc[6] += x1[i].z; acc[7] += x1[i].w;
          }
        }
      }
      float rr[8];
      unpack8(*reinterpret_cast<const uint4*>(residual + base + idx), rr);
#pragma unroll
      for (int e = 0; e < 8; ++e) v[j][e] = bf16r(acc[e]) + rr[e];
      *reinterpret_cast<uint4*>(residual + base + idx) = pack8(v[j]);
#pragma unroll
      for (int e = 0; e < 8; ++e) ss += v[j][e] * v[j][e];
    }
    const float inv = rsqrtf(block_sum<NT>(ss, red) / H + eps);
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      const int idx = (threadIdx.x + j * NT) * 8;
      float wf[8], o[8];
      unpack8(*reinterpret_cast<const uint4*>(w + idx), wf);
#pragma unroll
      for (int e = 0; e < 8; ++e) o[e] = bf16r(v[j][e] * inv) * wf[e];
      *reinterpret_cast<uint4*>(out + base + idx) = pack8(o);
    }
  }
  // the epoch is read only by this GPU's later launches: a device-scope arrival suffices
  last_cta<false>(a.counter, [&] { *a.epoch = want; });
  pdl_trigger();
}

void check_args(const TpArgs& a, int H) {
  if (a.world < 1 || a.world > kTpMaxWorld || a.rank < 0 || a.rank >= a.world)
    throw std::runtime_error("tp: bad world / rank");
  if (a.splits < 1) throw std::runtime_error("tp: splits must be >= 1");
  for (int r = 0; r < a.world; ++r)
    if (a.part[r] == nullptr || a.flags[r] == nullptr || (reinterpret_cast<uintptr_t>(a.part[r]) & 15))
      throw std::runtime_error("tp: every rank needs a 16-byte aligned partial buffer and a flag array");
  if (a.epoch == nullptr || a.counter == nullptr || a.status == nullptr) throw std::runtime_error("tp: null scratch");
  if (H != 2048 && H != 4096 && H != 1024 && H != 512 && H != 256)
    throw std::runtime_error("tp: unsupported hidden size " + std::to_string(H));
}

void check(const char* what) {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

}  // namespace

void tp_slots_partial(const TpArgs& a, const void* slots, int topk, int T, int H, cudaStream_t s) {
  check_args(a, H);
  const bf16* S = static_cast<const bf16*>(slots);
  const int G = T > 0 ? T : 1;  // an empty batch still releases its epoch
  if (H == 2048) pdl_launch(tp_slots_partial_kernel<256, 1>, G, 256, 0, s, a, S, topk, T, H);
  else if (H == 4096) pdl_launch(tp_slots_partial_kernel<256, 2>, G, 256, 0, s, a, S, topk, T, H);
  else if (H == 1024) pdl_launch(tp_slots_partial_kernel<128, 1>, G, 128, 0, s, a, S, topk, T, H);
  else if (H == 512) pdl_launch(tp_slots_partial_kernel<64, 1>, G, 64, 0, s, a, S, topk, T, H);
  else pdl_launch(tp_slots_partial_kernel<32, 1>, G, 32, 0, s, a, S, topk, T, H);
  check("tp_slots_partial");
}

void tp_allreduce_rmsnorm(const TpArgs& a, void* residual, const void* w, void* out, int T, int H, float eps,
                          cudaStream_t s) {
  check_args(a, H);
  bf16* R = static_cast<bf16*>(residual);
  const bf16* W = static_cast<const bf16*>(w);
  bf16* O = static_cast<bf16*>(out);
  const int G = T > 0 ? T : 1;
  if (H == 2048) pdl_launch(tp_allreduce_rmsnorm_kernel<256, 1>, G, 256, 0, s, a, R, W, O, T, H, eps);
  else if (H == 4096) pdl_launch(tp_allreduce_rmsnorm_kernel<256, 2>, G, 256, 0, s, a, R, W, O, T, H, eps);
  else if (H == 1024) pdl_launch(tp_allreduce_rmsnorm_kernel<128, 1>, G, 128, 0, s, a, R, W, O, T, H, eps);
  else if (H == 512) pdl_launch(tp_allreduce_rmsnorm_kernel<64, 1>, G, 64, 0, s, a, R, W, O, T, H, eps);
  else pdl_launch(tp_allreduce_rmsnorm_kernel<32, 1>, G, 32, 0, s, a, R, W, O, T, H, eps);
  check("tp_allreduce_rmsnorm");
}

}  // namespace b200

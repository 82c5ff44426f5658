// Memory-bound fused ops of the Qwen3-MoE layer (sm_100a).
//
//   embed_gather             token-id row gather (reference: VocabParallelEmbedding,
//                            nanovllm/layers/embed_head.py:34-42)
//   rmsnorm / add_rmsnorm    reference numerics of nanovllm/layers/layernorm.py:18-38:
//                            fp32 statistics, bf16 round, then bf16 weight multiply
//   moe_combine_add_rmsnorm  fixed-order top-k slot sum (nanovllm/kernels/moe_fusion.py:31-50)
//                            + residual add + the next RMSNorm, one pass over the row
//   qknorm_rope_kvstore      per-head q/k RMSNorm, neox RoPE and the paged KV store in
//                            one kernel (qwen3.py:82-86, rotary_embedding.py:7-16,
//                            attention.py:9-30); int8 KV gets a per-(token, head) scale
//   router_topk              fp32 softmax over experts, top-k, renormalise, bf16-round
//                            the weights, per-expert counts (qwen3_moe.py:389-395)
//   moe_permute              expert-sorted copy of the routed rows (qwen3_moe.py:219-245)
//
// Rows are processed with 16-byte vector accesses; one CTA (or warp) per token.
#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <vector>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <algorithm>
#include <cstdint>
#include <stdexcept>
#include <string>

#include "sm100.cuh"
#include "pdl.cuh"
#include "ep_sync.cuh"
#include "ep_dispatch.cuh"
#include "fused_ops.h"

namespace b200 {

using bf16 = __nv_bfloat16;

__device__ __forceinline__ void unpack8(const uint4& u, float (&f)[8]) {
  const __nv_bfloat162* p = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 t = __bfloat1622float2(p[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}
__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
  uint4 u;
  __nv_bfloat162* p = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) p[i] = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
  return u;
}
__device__ __forceinline__ float bf16r(float x) { return __bfloat162float(__float2bfloat16(x)); }

template <int NT>
__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) red[w] = v;
  __syncthreads();
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < NT / 32; ++i) s += red[i];
  __syncthreads();
  return s;
}

// ------------------------------------------------------------ embedding
// feed_src (optional): token t reads its id from feed_tokens[feed_src[t]] when
// feed_src[t] >= 0 -- the previous step's sampled token, still on the device, so a
// decode step can be launched before the host has read that token back.
__global__ void embed_gather_kernel(const int* __restrict__ ids, const bf16* __restrict__ table,
                                    bf16* __restrict__ out, int H, int V, int* status,
                                    const int* __restrict__ feed_src, const int* __restrict__ feed_tokens) {
  pdl_enter();
  const int t = blockIdx.x;
  int id = ids[t];
  if (feed_src != nullptr) {
    const int f = feed_src[t];
    if (f >= 0) id = feed_tokens[f];
  }
  if (id < 0 || id >= V) {  // the host validates ids; never read out of bounds
    record_status(status, kStatusBadShape);
    id = 0;
  }
  const uint4* src = reinterpret_cast<const uint4*>(table + (size_t)id * H);
  uint4* dst = reinterpret_cast<uint4*>(out + (size_t)t * H);
  for (int i = threadIdx.x; i < H / 8; i += blockDim.x) dst[i] = src[i];
  pdl_trigger();
}

// ------------------------------------------------------------- RMSNorm
// H = NT * 8 * VPT; one CTA per token.
template <int NT, int VPT>
__global__ void __launch_bounds__(NT) rmsnorm_kernel(const bf16* __restrict__ x, const bf16* res_in,
                                                     const bf16* __restrict__ w, bf16* __restrict__ out,
                                                     bf16* res_out, int H, float eps, const float* __restrict__ part,
                                                     int splits, size_t split_stride) {
  pdl_enter();
  __shared__ float red[NT / 32];
  const size_t base = (size_t)blockIdx.x * H;
  float v[VPT][8];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int idx = (threadIdx.x + j * NT) * 8;
    if (part != nullptr) {
      // x is the split-K GEMM's fp32 partial sums: reduce them and round to bf16
      // (the value the separate reduce kernel would have stored)
      float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      for (int sp = 0; sp < splits; ++sp) {
        const float4* q = reinterpret_cast<const float4*>(part + sp * split_stride + base + idx);
        const float4 lo = q[0], hi = q[1];
        acc[0] += lo.x; acc[1] += lo.y; acc[2] += lo.z; acc[3] += lo.w;
        acc[4] += hi.x; acc[5] += hi.y; acc[6] += hi.z; acc[7] += hi.w;
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) v[j][e] = bf16r(acc[e]);
    } else {
      unpack8(*reinterpret_cast<const uint4*>(x + base + idx), v[j]);
    }
    if (res_in != nullptr) {
      float r[8];
      unpack8(*reinterpret_cast<const uint4*>(res_in + base + idx), r);
#pragma unroll
      for (int e = 0; e < 8; ++e) v[j][e] += r[e];
      *reinterpret_cast<uint4*>(res_out + base + idx) = pack8(v[j]);
    }
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
  pdl_trigger();
}

// Combine the top-k expert slots of each token in fixed order, add the
// residual, and normalise with the next RMSNorm.
template <int NT, int VPT>
__global__ void __launch_bounds__(NT) moe_combine_kernel(const bf16* __restrict__ slots, int topk,
                                                         bf16* residual, const bf16* __restrict__ w,
                                                         bf16* __restrict__ out, int H, float eps,
                                                         int* __restrict__ zero_buf, int zero_n, int T,
                                                         CombineWait cw) {
  pdl_enter();
  // expert parallel: the slots are written by the experts' owners; wait for every
  // owner's done epoch first (block 0 charges the wait to the owner it waited for)
  if (cw.flags != nullptr) {
    const uint32_t epoch = *cw.epoch;
    if (threadIdx.x < cw.world)
      wait_epoch(cw.flags + threadIdx.x, epoch, cw.status,
                 (blockIdx.x == 0 && cw.wait_ns) ? cw.wait_ns + cw.world + threadIdx.x : nullptr);
    __syncthreads();
  }
  // the layer's routing counters are dead once the down GEMM has run: clear them
  // for the next layer here instead of in a separate fill launch
  if (blockIdx.x == 0 && zero_buf != nullptr)
    for (int i = threadIdx.x; i < zero_n; i += NT) zero_buf[i] = 0;
  __shared__ float red[NT / 32];
  const int t = blockIdx.x;
  if (t >= T) return;  // the one block of an empty batch that only waits
  const size_t base = (size_t)t * H;
  float v[VPT][8];
  float ss = 0.f;
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
    float r[8];
    unpack8(*reinterpret_cast<const uint4*>(residual + base + idx), r);
#pragma unroll
    for (int e = 0; e < 8; ++e) v[j][e] = bf16r(acc[e]) + r[e];
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
  pdl_trigger();
}

// ------------------------------------------------ q/k norm + RoPE + KV store
// One CTA per token, one warp per head (q heads, then k heads, then v heads).
// Lane l owns elements {l*E2 .. l*E2+E2-1} of each half (E2 = D/64).
template <int D>
__global__ void qknorm_rope_kvstore_kernel(const QkvArgs a) {
  pdl_enter();
  constexpr int E2 = D / 64;
  const int t = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nq = a.num_q_heads, nkv = a.num_kv_heads;
  const int pos = a.positions[t];
  const int slot = a.slot_mapping[t];
  const bf16* row = static_cast<const bf16*>(a.qkv) + (size_t)t * a.qkv_stride;
  const float* prow = a.part != nullptr ? a.part + (size_t)t * a.qkv_stride : nullptr;
  const float* cs = a.cos_sin + (size_t)pos * D;  // [cos(D/2) | sin(D/2)]
  for (int h = warp; h < nq + 2 * nkv; h += blockDim.x >> 5) {
    const bool is_q = h < nq, is_k = !is_q && h < nq + nkv;
    float x1[E2], x2[E2];
    if (prow != nullptr) {  // split-K partials: sum in split order, round to bf16
      const float* p = prow + (size_t)h * D;
#pragma unroll
      for (int e = 0; e < E2; ++e) {
        float s1 = p[lane * E2 + e], s2 = p[D / 2 + lane * E2 + e];
        for (int sp = 1; sp < a.splits; ++sp) {
          s1 += p[sp * a.part_stride + lane * E2 + e];
          s2 += p[sp * a.part_stride + D / 2 + lane * E2 + e];
        }
        x1[e] = bf16r(s1);
        x2[e] = bf16r(s2);
      }
    } else {
      const bf16* src = row + (size_t)h * D;
#pragma unroll
      for (int e = 0; e < E2; ++e) {
        x1[e] = __bfloat162float(src[lane * E2 + e]);
        x2[e] = __bfloat162float(src[D / 2 + lane * E2 + e]);
      }
    }
    if (is_q || is_k) {
      const bf16* nw = static_cast<const bf16*>(is_q ? a.q_norm_w : a.k_norm_w);
      float ss = 0.f;
#pragma unroll
      for (int e = 0; e < E2; ++e) ss += x1[e] * x1[e] + x2[e] * x2[e];
      const float inv = rsqrtf(warp_sum(ss) / D + a.eps);
#pragma unroll
      for (int e = 0; e < E2; ++e) {
        const int i1 = lane * E2 + e, i2 = D / 2 + i1;
        // the norm output is bf16 (normalise, round, bf16 weight multiply, round)
        x1[e] = bf16r(bf16r(x1[e] * inv) * __bfloat162float(nw[i1]));
        x2[e] = bf16r(bf16r(x2[e] * inv) * __bfloat162float(nw[i2]));
        const float c = cs[i1], s = cs[D / 2 + i1];
        const float y1 = x1[e] * c - x2[e] * s;
        const float y2 = x2[e] * c + x1[e] * s;
        x1[e] = y1;
        x2[e] = y2;
      }
    }
    if (is_q) {
      bf16* dst = static_cast<bf16*>(a.q_out) + ((size_t)t * nq + h) * D;
#pragma unroll
      for (int e = 0; e < E2; ++e) {
        dst[lane * E2 + e] = __float2bfloat16(x1[e]);
        dst[D / 2 + lane * E2 + e] = __float2bfloat16(x2[e]);
      }
    } else if (slot >= 0) {
      const int kvh = is_k ? h - nq : h - nq - nkv;
      const int blk = slot / a.block_size, bo = slot % a.block_size;
      const int64_t off = (int64_t)blk * a.block_stride + ((int64_t)kvh * a.block_size + bo) * D;
      const int64_t soff = (int64_t)blk * a.scale_block_stride + (int64_t)kvh * a.block_size + bo;
      if (a.kv_int8 == 2) {
        // channel mode: q = clamp(floor(x / scale[d] + 0.5), +-127) per channel; the head's
        // outlier dims store 0 and their exact bf16 value goes to the side pool
        const int kv = is_k ? 0 : 1;
        const float* sc = a.ch_scale + ((size_t)kv * nkv + kvh) * D;
        int8_t* dst = reinterpret_cast<int8_t*>(is_k ? a.k_cache : a.v_cache) + off;
        bf16* side = reinterpret_cast<bf16*>(is_k ? a.side_k : a.side_v) +
                     (int64_t)blk * a.side_block_stride + ((int64_t)kvh * a.block_size + bo) * 4;
        const int n_out = a.n_out[kvh];
        int od[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) od[i] = i < n_out ? a.out_idx[kvh * 4 + i] : -1;
        float* cmax = a.calib_amax != nullptr ? a.calib_amax + ((size_t)kv * nkv + kvh) * D : nullptr;
        float* csum = a.calib_sum != nullptr ? a.calib_sum + ((size_t)kv * nkv + kvh) * D : nullptr;
#pragma unroll
        for (int half = 0; half < 2; ++half) {
#pragma unroll
          for (int e = 0; e < E2; ++e) {
            const int d = half * (D / 2) + lane * E2 + e;
            const float xv = bf16r(half ? x2[e] : x1[e]);
            int q = (int)fmaxf(-127.f, fminf(127.f, floorf(xv / sc[d] + 0.5f)));
#pragma unroll
            for (int i = 0; i < 4; ++i)
              if (od[i] == d) {
                q = 0;
                side[i] = __float2bfloat16(xv);
              }
            dst[d] = (int8_t)q;
            if (cmax != nullptr) {  // |x| >= 0: its float bits order like the values
              atomicMax(reinterpret_cast<int*>(cmax + d), __float_as_int(fabsf(xv)));
              atomicAdd(csum + d, fabsf(xv));
            }
          }
        }
      } else if (a.kv_int8) {
        // per-(token, head) absmax scale, round-to-nearest into [-127, 127]
        float m = 0.f;
#pragma unroll
        for (int e = 0; e < E2; ++e) m = fmaxf(m, fmaxf(fabsf(bf16r(x1[e])), fabsf(bf16r(x2[e]))));
        m = warp_max(m);
        const float scale = m > 0.f ? m / 127.f : 1.f;
        int8_t* dst = reinterpret_cast<int8_t*>(is_k ? a.k_cache : a.v_cache) + off;
#pragma unroll
        for (int e = 0; e < E2; ++e) {
          dst[lane * E2 + e] = (int8_t)max(-127, min(127, __float2int_rn(bf16r(x1[e]) / scale)));
          dst[D / 2 + lane * E2 + e] = (int8_t)max(-127, min(127, __float2int_rn(bf16r(x2[e]) / scale)));
        }
        if (lane == 0) (is_k ? a.k_scale : a.v_scale)[soff] = scale;
      } else {
        bf16* dst = reinterpret_cast<bf16*>(is_k ? a.k_cache : a.v_cache) + off;
#pragma unroll
        for (int e = 0; e < E2; ++e) {
          dst[lane * E2 + e] = __float2bfloat16(x1[e]);
          dst[D / 2 + lane * E2 + e] = __float2bfloat16(x2[e]);
        }
      }
    }
  }
  pdl_trigger();
}

// --------------------------------------------------------------- router
// One warp per token; E <= 32 * EPL.  Logits are rounded to bf16 first: the
// reference's gate GEMM returns bf16 (qwen3_moe.py:390).
// Softmax over E logits of one token held by one warp (EPL per lane, already
// rounded to bf16 like the reference's bf16 gate output), top-k with the lowest
// expert id winning ties, optional renormalisation, bf16-rounded weights.
template <int EPL>
__device__ __forceinline__ void topk_row(float (&p)[EPL], int E, int topk, int renorm, int tok, int lane,
                                         int* __restrict__ ids, float* __restrict__ weights, int* __restrict__ counts,
                                         int* ev_out = nullptr, float* wv_out = nullptr) {
  float mx = -INFINITY;
#pragma unroll
  for (int j = 0; j < EPL; ++j) mx = fmaxf(mx, p[j]);
  mx = warp_max(mx);
  float sum = 0.f;
#pragma unroll
  for (int j = 0; j < EPL; ++j) {
    const int e = j * 32 + lane;
    p[j] = e < E ? __expf(p[j] - mx) : 0.f;
    sum += p[j];
  }
  sum = warp_sum(sum);
  const float inv = 1.f / sum;
#pragma unroll
  for (int j = 0; j < EPL; ++j) p[j] = j * 32 + lane < E ? p[j] * inv : -1.f;
  float sel_w[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  int sel_e[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  float wsum = 0.f;
#pragma unroll
  for (int k = 0; k < 8; ++k) {  // static indices keep sel_* in registers (topk <= 8)
    if (k >= topk) break;
    float bv = -2.f;
    int be = 1 << 30;
#pragma unroll
    for (int j = 0; j < EPL; ++j) {
      const int e = j * 32 + lane;
      if (p[j] > bv || (p[j] == bv && e < be)) { bv = p[j]; be = e; }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oe = __shfl_xor_sync(0xffffffffu, be, o);
      if (ov > bv || (ov == bv && oe < be)) { bv = ov; be = oe; }
    }
    sel_w[k] = bv;
    sel_e[k] = be;
    wsum += bv;
#pragma unroll
    for (int j = 0; j < EPL; ++j)
      if (j * 32 + lane == be) p[j] = -1.f;
  }
  if (lane < topk) {
    float wv = 0.f;
    int ev = 0;
#pragma unroll
    for (int k = 0; k < 8; ++k)
      if (k == lane) { wv = sel_w[k]; ev = sel_e[k]; }
    if (renorm) wv = wv / wsum;
    ids[(size_t)tok * topk + lane] = ev;
    weights[(size_t)tok * topk + lane] = bf16r(wv);  // the reference casts weights to bf16
    if (counts != nullptr) atomicAdd(&counts[ev], 1);
    if (ev_out != nullptr) {  // lane k < topk: the token's k-th expert and its weight
      *ev_out = ev;
      *wv_out = bf16r(wv);
    }
  }
}

template <int EPL>
__global__ void router_topk_kernel(const float* __restrict__ logits, int ld, int T, int E, int topk, int renorm,
                                   int* __restrict__ ids, float* __restrict__ weights, int* __restrict__ counts) {
  pdl_enter();
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= T) return;
  const float* row = logits + (size_t)warp * ld;
  float p[EPL];
#pragma unroll
  for (int j = 0; j < EPL; ++j) {
    const int e = j * 32 + lane;
    p[j] = e < E ? bf16r(row[e]) : -INFINITY;
  }
  topk_row<EPL>(p, E, topk, renorm, warp, lane, ids, weights, counts);
  pdl_trigger();
}

// ------------------------------------------------------------ fused router
// Router GEMM + softmax + top-k in one launch (replaces GEMM, split-K reduce and
// top-k).  CTA = 16 tokens x all experts (<= 128); warp w owns experts
// [16w, 16w + 16).  One thread streams 64-wide K chunks of x (box 64 x 16) and of
// the router weight (box 64 x 128) with TMA into an 8-deep mbarrier ring
// (128-byte swizzle: 16-byte unit u of row r at u ^ (r & 7), which the ldmatrix
// addressing below reads without bank conflicts); the warp-level bf16 MMAs
// accumulate in fp32 and the logits go through shared memory to one warp per
// token for the top-k.  Per-thread 16-byte cp.async (about 1150 requests per
// chunk) held a CTA near 20 GB/s; a TMA box is one request.
constexpr int kRtTok = 16, kRtE = 128, kRtK = 64;
constexpr int kRtStages = 8;
constexpr int kRtChunkBytes = (kRtTok + kRtE) * 128;
constexpr int kRtSmem = 1024 + kRtStages * kRtChunkBytes + kRtTok * (kRtE + 1) * 4 + kRtStages * 8 + 16;

__device__ __forceinline__ uint32_t rt_off(int row, int chunk) { return row * 128 + ((chunk ^ (row & 7)) << 4); }

// Decode-size batches have too few 16-token tiles to fill the SMs, and each CTA
// would walk all H / 64 chunks serially: the grid's y dimension then splits K.
// Each CTA writes its fp32 partial logits to `part`; the last CTA of a tile
// (per-tile counter) adds the partials in K order -- the same on every run --
// and does the top-k.
__global__ void __launch_bounds__(256) router_fused_kernel(const __grid_constant__ CUtensorMap xmap,
                                                           const __grid_constant__ CUtensorMap wmap, int T, int H,
                                                           int E, int topk, int renorm, int* __restrict__ ids,
                                                           float* __restrict__ weights, int* __restrict__ counts,
                                                           int* __restrict__ status, float* __restrict__ part,
                                                           int* __restrict__ tile_cnt,
                                                           const __nv_bfloat16* __restrict__ xg, const EpArgs ep,
                                                           int ep_on) {
  pdl_enter();
  constexpr int XB = kRtTok * 128;  // bytes of one x chunk (the W chunk follows it)
  extern __shared__ __align__(1024) uint8_t rt_raw[];
  uint8_t* ring = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(rt_raw) + 1023) & ~uintptr_t(1023));
  float(*logit)[kRtE + 1] = reinterpret_cast<float(*)[kRtE + 1]>(ring + kRtStages * kRtChunkBytes);
  uint64_t* full = reinterpret_cast<uint64_t*>(ring + kRtStages * kRtChunkBytes + kRtTok * (kRtE + 1) * 4);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(full + kRtStages);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t0 = blockIdx.x * kRtTok;
  const int KS = gridDim.y, ks = blockIdx.y;
  const int c_begin = (int)((int64_t)(H / kRtK) * ks / KS), c_end = (int)((int64_t)(H / kRtK) * (ks + 1) / KS);
  const int nchunks = c_end - c_begin;  // this CTA's K chunks; chunk j of them is global chunk c_begin + j
  if (threadIdx.x == 0) {
    for (int i = 0; i < kRtStages; ++i) mbar_init(&full[i], 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();
  auto issue = [&](int c) {
    uint8_t* dst = ring + (c % kRtStages) * kRtChunkBytes;
    mbar_arrive_expect_tx(&full[c % kRtStages], kRtChunkBytes);
    tma_load_2d(dst, &xmap, &full[c % kRtStages], (c_begin + c) * kRtK, t0);  // rows >= T come back zero-filled
    tma_load_2d(dst + XB, &wmap, &full[c % kRtStages], (c_begin + c) * kRtK, 0);
  };
  if (threadIdx.x == 0) {
    tma_prefetch_desc(&xmap);
    tma_prefetch_desc(&wmap);
    for (int c = 0; c < kRtStages - 1 && c < nchunks; ++c) issue(c);
  }
  float acc[2][4];
#pragma unroll
  for (int n = 0; n < 2; ++n)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[n][e] = 0.f;
  bool ok = true;
  for (int c = 0; c < nchunks; ++c) {
    // chunk c - 1's buffer was released by the barrier that ended the previous iteration
    if (threadIdx.x == 0 && c + kRtStages - 1 < nchunks) issue(c + kRtStages - 1);
    ok = mbar_wait(&full[c % kRtStages], (c / kRtStages) & 1, status, kStatusTimeoutFull, abort_flag);
    if (!__syncthreads_and(ok)) { ok = false; break; }
    const uint32_t xs = static_cast<uint32_t>(__cvta_generic_to_shared(ring + (c % kRtStages) * kRtChunkBytes));
    const uint32_t ws = xs + XB;
#pragma unroll
    for (int ks = 0; ks < kRtK / 16; ++ks) {
      const int mi = lane >> 3, rr = lane & 7;
      uint32_t a[4];
      {
        const int row = (mi & 1) * 8 + rr, chunk = ks * 2 + (mi >> 1);
        asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                     : "=r"(a[0]), "=r"(a[1]), "=r"(a[2]), "=r"(a[3]) : "r"(xs + rt_off(row, chunk)));
      }
      uint32_t b0, b1, b2, b3;
      {
        const int e = warp * 16 + (mi >> 1) * 8 + rr, chunk = ks * 2 + (mi & 1);
        asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                     : "=r"(b0), "=r"(b1), "=r"(b2), "=r"(b3) : "r"(ws + rt_off(e, chunk)));
      }
      asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                   "{%0,%1,%2,%3};"
                   : "+f"(acc[0][0]), "+f"(acc[0][1]), "+f"(acc[0][2]), "+f"(acc[0][3])
                   : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
      asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                   "{%0,%1,%2,%3};"
                   : "+f"(acc[1][0]), "+f"(acc[1][1]), "+f"(acc[1][2]), "+f"(acc[1][3])
                   : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b2), "r"(b3));
    }
    __syncthreads();  // every warp is done with chunk c: its buffer may be refilled
  }
  if (!ok) {
    if (threadIdx.x == 0) {
      // a wait gave up: let the copies already issued land before the CTA exits
      const uint64_t tw = globaltimer_ns();
      while (globaltimer_ns() - tw < 1000000ull) __nanosleep(1000);
    }
    return;
  }
  if (KS == 1) {
#pragma unroll
    for (int n = 0; n < 2; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int row = (lane >> 2) + 8 * (e >> 1), col = warp * 16 + n * 8 + 2 * (lane & 3) + (e & 1);
        logit[row][col] = acc[n][e];
      }
  } else {
    float* mine = part + ((size_t)blockIdx.x * KS + ks) * (kRtTok * kRtE);
#pragma unroll
    for (int n = 0; n < 2; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int row = (lane >> 2) + 8 * (e >> 1), col = warp * 16 + n * 8 + 2 * (lane & 3) + (e & 1);
        mine[row * kRtE + col] = acc[n][e];
      }
    __threadfence();
    __syncthreads();
    __shared__ int last_s;
    if (threadIdx.x == 0) last_s = atomicAdd(&tile_cnt[blockIdx.x], 1) == KS - 1;
    __syncthreads();
    if (!last_s) return;
    __threadfence();
    const float* all = part + (size_t)blockIdx.x * KS * (kRtTok * kRtE);
    for (int i = threadIdx.x; i < kRtTok * kRtE; i += blockDim.x) {
      float v = 0.f;
      for (int j = 0; j < KS; ++j) v += __ldcg(all + (size_t)j * (kRtTok * kRtE) + i);
      logit[i / kRtE][i % kRtE] = v;
    }
    if (threadIdx.x == 0) tile_cnt[blockIdx.x] = 0;  // ready for the next launch
  }
  __shared__ uint32_t ep_epoch_s;
  __shared__ int ep_last_s;
  if (ep_on && threadIdx.x == 0) ep_epoch_s = *ep.epoch + 1;
  __syncthreads();
  for (int r = warp; r < kRtTok; r += 8) {
    const int tok = t0 + r;
    if (tok >= T) break;
    float p[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int e = j * 32 + lane;
      p[j] = e < E ? bf16r(logit[r][e]) : -INFINITY;
    }
    int ev = 0;
    float wv = 0.f;
    topk_row<4>(p, E, topk, renorm, tok, lane, ids, weights, counts, &ev, &wv);
    if (ep_on) {
      // expert parallelism: send the token's rows to their experts' owners right here
      // (the stand-alone ep_dispatch_kernel does the same from ids / weights)
      ep_send_token(ep, xg + (int64_t)tok * H, tok, topk, ev, wv, lane);
    }
  }
  // one CTA per token tile gets here (split-K: the tile's last); the grid's last publishes
  if (ep_on && ep_block_arrive(ep, gridDim.x, &ep_last_s)) ep_publish(ep, ep_epoch_s);
  pdl_trigger();
}

// Each warp copies one routed (token, k) row to its expert-sorted position.
__global__ void moe_permute_kernel(const bf16* __restrict__ x, const int* __restrict__ ids, int T, int topk,
                                   int E, int H, const int* __restrict__ counts, int* __restrict__ cursor,
                                   bf16* __restrict__ x_perm, int* __restrict__ slot_of_row,
                                   int* __restrict__ offsets_out) {
  pdl_enter();
  __shared__ int offs[kMaxExperts + 1];
  if (threadIdx.x < 32) {
    const int per = (E + 31) / 32;
    const int lane = threadIdx.x;
    int e0 = lane * per, e1 = min(E, e0 + per), s = 0;
    for (int e = e0; e < e1; ++e) s += counts[e];
    int incl = s;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      int v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    int pre = incl - s;
    for (int e = e0; e < e1; ++e) { offs[e] = pre; pre += counts[e]; }
    if (lane == 31) offs[E] = incl;
  }
  __syncthreads();
  if (blockIdx.x == 0 && offsets_out != nullptr)
    for (int e = threadIdx.x; e <= E; e += blockDim.x) offsets_out[e] = offs[e];
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= T * topk) return;
  const int t = warp / topk;
  const int e = ids[warp];
  if (e < 0 || e >= E) return;
  int pos = 0;
  if (lane == 0) pos = offs[e] + atomicAdd(&cursor[e], 1);
  pos = __shfl_sync(0xffffffffu, pos, 0);
  if (lane == 0) slot_of_row[pos] = warp;
  const uint4* src = reinterpret_cast<const uint4*>(x + (size_t)t * H);
  uint4* dst = reinterpret_cast<uint4*>(x_perm + (size_t)pos * H);
  for (int i = lane; i < H / 8; i += 32) dst[i] = src[i];
  pdl_trigger();
}

// --------------------------------------------------------------- launchers
static void check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

// Split-K reduction: 4 consecutive outputs per thread (float4 loads of each
// partial; the partials of a decode-size GEMM sit in L2).
template <bool BF16>
__global__ void splitk_reduce_kernel(const float* __restrict__ part, int splits, int T, int N, void* out,
                                     int ld_out) {
  pdl_enter();
  const int n4 = N / 4;
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (int64_t)T * n4) return;
  const int t = (int)(idx / n4), c = (int)(idx % n4) * 4;
  const size_t stride = (size_t)T * N;
  const float* p = part + (size_t)t * N + c;
  float4 acc = *reinterpret_cast<const float4*>(p);
  for (int s = 1; s < splits; ++s) {
    const float4 v = *reinterpret_cast<const float4*>(p + s * stride);
    acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
  }
  if constexpr (BF16) {
    __nv_bfloat162 lo = __floats2bfloat162_rn(acc.x, acc.y), hi = __floats2bfloat162_rn(acc.z, acc.w);
    uint2 packed = make_uint2(*reinterpret_cast<uint32_t*>(&lo), *reinterpret_cast<uint32_t*>(&hi));
    *reinterpret_cast<uint2*>(static_cast<bf16*>(out) + (size_t)t * ld_out + c) = packed;
  } else {
    *reinterpret_cast<float4*>(static_cast<float*>(out) + (size_t)t * ld_out + c) = acc;
  }
  pdl_trigger();
}

// KV handoff: grid (blocks, chunks); each CTA streams a contiguous part of one
// block slab.  Used for prefill -> decode transfers into a peer's pool.
__global__ void kv_blocks_copy_kernel(const uint4* __restrict__ src, const int* __restrict__ src_ids,
                                      uint4* __restrict__ dst, const int* __restrict__ dst_ids, int64_t vecs) {
  pdl_enter();
  const int64_t s0 = (int64_t)src_ids[blockIdx.x] * vecs, d0 = (int64_t)dst_ids[blockIdx.x] * vecs;
  const int64_t per = (vecs + gridDim.y - 1) / gridDim.y;
  const int64_t lo = blockIdx.y * per, hi = min(vecs, lo + per);
  for (int64_t i = lo + threadIdx.x; i < hi; i += blockDim.x) dst[d0 + i] = src[s0 + i];
  pdl_trigger();
}

// e4m3 [G, N, K] (row-major, or tile-major as ops.tile_fp8 lays it out) with
// 128x128 block scales -> bf16 [G, N, K] row-major, bf16(float(q) * scale): the
// GEMM's per-tile dequantisation done once (large prefill batches re-read each
// expert's weights for every token tile).  One thread per 16 consecutive K.
__global__ void dequant_weights_kernel(const uint8_t* __restrict__ q, const float* __restrict__ scale,
                                       bf16* __restrict__ out, int G, int N, int K, int tiled) {
  pdl_enter();
  const int64_t chunks = (int64_t)G * N * (K / 16);
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= chunks) return;
  const int kc = (int)(i % (K / 16));
  const int64_t gn = i / (K / 16);
  const int n = (int)(gn % N), g = (int)(gn / N);
  const int k = kc * 16;
  size_t src;
  if (tiled) {
    const int r = n & 127, u = (k & 63) >> 4;
    const size_t blk = ((size_t)g * (N / 128) + (n >> 7)) * (K / 64) + (k >> 6);
    src = blk * 8192 + r * 64 + ((u ^ ((r >> 1) & 3)) << 4);
  } else {
    src = ((size_t)g * N + n) * K + k;
  }
  const uint4 v = *reinterpret_cast<const uint4*>(q + src);
  const float sc = scale[((size_t)g * (N / 128) + (n >> 7)) * (K / 128) + (k >> 7)];
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
  uint32_t o[8];
#pragma unroll
  for (int h = 0; h < 4; ++h) {
    // e4m3 -> f16 -> f32 are exact; one fp32 rounding of the product, then bf16
    __half2_raw lo = __nv_cvt_fp8x2_to_halfraw2(static_cast<__nv_fp8x2_storage_t>(w[h] & 0xFFFFu), __NV_E4M3);
    __half2_raw hi = __nv_cvt_fp8x2_to_halfraw2(static_cast<__nv_fp8x2_storage_t>(w[h] >> 16), __NV_E4M3);
    const float2 flo = __half22float2(*reinterpret_cast<__half2*>(&lo));
    const float2 fhi = __half22float2(*reinterpret_cast<__half2*>(&hi));
    __nv_bfloat162 b0 = __floats2bfloat162_rn(__fmul_rn(flo.x, sc), __fmul_rn(flo.y, sc));
    __nv_bfloat162 b1 = __floats2bfloat162_rn(__fmul_rn(fhi.x, sc), __fmul_rn(fhi.y, sc));
    o[2 * h] = *reinterpret_cast<uint32_t*>(&b0);
    o[2 * h + 1] = *reinterpret_cast<uint32_t*>(&b1);
  }
  uint4* dst = reinterpret_cast<uint4*>(out + ((size_t)g * N + n) * K + k);
  dst[0] = make_uint4(o[0], o[1], o[2], o[3]);
  dst[1] = make_uint4(o[4], o[5], o[6], o[7]);
  pdl_trigger();
}

void dequant_weights(const void* q, const float* scale, void* out, int G, int N, int K, bool tiled, cudaStream_t s) {
  if (N % 128 || K % 128) throw std::runtime_error("dequant_weights: N and K must be multiples of 128");
  const int64_t chunks = (int64_t)G * N * (K / 16);
  if (chunks == 0) return;
  pdl_launch(dequant_weights_kernel, (unsigned)((chunks + 255) / 256), 256, 0, s, 
      static_cast<const uint8_t*>(q), scale, static_cast<bf16*>(out), G, N, K, tiled ? 1 : 0);
  check_launch("dequant_weights");
}

void kv_blocks_copy(const void* src_base, const int* src_ids, void* dst_base, const int* dst_ids, int n,
                    int64_t block_bytes, cudaStream_t s) {
  if (n == 0) return;
  if (block_bytes % 16 || (reinterpret_cast<uintptr_t>(src_base) & 15) || (reinterpret_cast<uintptr_t>(dst_base) & 15))
    throw std::runtime_error("kv_blocks_copy: 16-byte aligned pools and block sizes required");
  const int64_t vecs = block_bytes / 16;
  const int chunks = (int)std::min<int64_t>(64, std::max<int64_t>(1, vecs / 4096));
  pdl_launch(kv_blocks_copy_kernel, dim3(n, chunks), 256, 0, s, static_cast<const uint4*>(src_base), src_ids,
                                                        static_cast<uint4*>(dst_base), dst_ids, vecs);
  check_launch("kv_blocks_copy");
}

void splitk_reduce(const float* part, int splits, int T, int N, void* out, int ld_out, bool out_bf16,
                   cudaStream_t s) {
  if (T == 0) return;
  if (N % 4 || ld_out % 4) throw std::runtime_error("splitk_reduce: N and ld_out must be multiples of 4");
  const int64_t work = (int64_t)T * (N / 4);
  const int blocks = (int)((work + 255) / 256);
  if (out_bf16) pdl_launch(splitk_reduce_kernel<true>, blocks, 256, 0, s, part, splits, T, N, out, ld_out);
  else pdl_launch(splitk_reduce_kernel<false>, blocks, 256, 0, s, part, splits, T, N, out, ld_out);
  check_launch("splitk_reduce");
}

void embed_gather(const int* ids, const void* table, void* out, int T, int H, int V, int* status,
                  cudaStream_t s, const int* feed_src, const int* feed_tokens) {
  if (T == 0) return;
  if (H % 8) throw std::runtime_error("embed_gather: H % 8");
  pdl_launch(embed_gather_kernel, T, 256, 0, s, ids, (const bf16*)table, (bf16*)out, H, V, status, feed_src,
             feed_tokens);
  check_launch("embed_gather");
}

void rmsnorm(const void* x, const void* res_in, const void* w, void* out, void* res_out, int T, int H,
             float eps, cudaStream_t s, const float* part, int splits) {
  if (T == 0) return;
  const bf16 *X = (const bf16*)x, *R = (const bf16*)res_in, *W = (const bf16*)w;
  bf16 *O = (bf16*)out, *RO = (bf16*)res_out;
  const size_t ss = (size_t)T * H;
  if (H == 2048) pdl_launch(rmsnorm_kernel<256, 1>, T, 256, 0, s, X, R, W, O, RO, H, eps, part, splits, ss);
  else if (H == 4096) pdl_launch(rmsnorm_kernel<256, 2>, T, 256, 0, s, X, R, W, O, RO, H, eps, part, splits, ss);
  else if (H == 256) pdl_launch(rmsnorm_kernel<32, 1>, T, 32, 0, s, X, R, W, O, RO, H, eps, part, splits, ss);
  else if (H == 512) pdl_launch(rmsnorm_kernel<64, 1>, T, 64, 0, s, X, R, W, O, RO, H, eps, part, splits, ss);
  else if (H == 1024) pdl_launch(rmsnorm_kernel<128, 1>, T, 128, 0, s, X, R, W, O, RO, H, eps, part, splits, ss);
  else throw std::runtime_error("rmsnorm: unsupported hidden size " + std::to_string(H));
  check_launch("rmsnorm");
}

void moe_combine_add_rmsnorm(const void* slots, int topk, void* residual, const void* w, void* out, int T,
                             int H, float eps, cudaStream_t s, int* zero_buf, int zero_n, const CombineWait& cw) {
  if (T == 0 && cw.flags == nullptr) return;
  if (cw.flags != nullptr && (cw.world < 1 || cw.world > 32 || cw.epoch == nullptr))
    throw std::runtime_error("moe_combine: bad expert-parallel wait arguments");
  const bf16 *S = (const bf16*)slots, *W = (const bf16*)w;
  bf16 *R = (bf16*)residual, *O = (bf16*)out;
  const int G = T > 0 ? T : 1;
  if (H == 2048) pdl_launch(moe_combine_kernel<256, 1>, G, 256, 0, s, S, topk, R, W, O, H, eps, zero_buf, zero_n, T, cw);
  else if (H == 4096) pdl_launch(moe_combine_kernel<256, 2>, G, 256, 0, s, S, topk, R, W, O, H, eps, zero_buf, zero_n, T, cw);
  else if (H == 256) pdl_launch(moe_combine_kernel<32, 1>, G, 32, 0, s, S, topk, R, W, O, H, eps, zero_buf, zero_n, T, cw);
  else if (H == 512) pdl_launch(moe_combine_kernel<64, 1>, G, 64, 0, s, S, topk, R, W, O, H, eps, zero_buf, zero_n, T, cw);
  else if (H == 1024) pdl_launch(moe_combine_kernel<128, 1>, G, 128, 0, s, S, topk, R, W, O, H, eps, zero_buf, zero_n, T, cw);
  else throw std::runtime_error("moe_combine: unsupported hidden size " + std::to_string(H));
  check_launch("moe_combine_add_rmsnorm");
}

void qknorm_rope_kvstore(const QkvArgs& a, int T, cudaStream_t s) {
  if (T == 0) return;
  const int heads = a.num_q_heads + 2 * a.num_kv_heads;
  const int threads = 32 * std::min(heads, 16);
  if (a.head_dim == 128) pdl_launch(qknorm_rope_kvstore_kernel<128>, T, threads, 0, s, a);
  else if (a.head_dim == 64) pdl_launch(qknorm_rope_kvstore_kernel<64>, T, threads, 0, s, a);
  else throw std::runtime_error("qknorm_rope_kvstore: head_dim must be 64 or 128");
  check_launch("qknorm_rope_kvstore");
}

void router_topk(const float* logits, int ld, int T, int E, int topk, bool renorm, int* ids, float* weights,
                 int* counts, cudaStream_t s) {
  if (T == 0) return;
  if (topk > 8 || topk < 1) throw std::runtime_error("router_topk: topk must be in [1, 8]");
  const int blocks = (T * 32 + 255) / 256;
  if (E <= 32) pdl_launch(router_topk_kernel<1>, blocks, 256, 0, s, logits, ld, T, E, topk, renorm, ids, weights, counts);
  else if (E <= 64) pdl_launch(router_topk_kernel<2>, blocks, 256, 0, s, logits, ld, T, E, topk, renorm, ids, weights, counts);
  else if (E <= 128) pdl_launch(router_topk_kernel<4>, blocks, 256, 0, s, logits, ld, T, E, topk, renorm, ids, weights, counts);
  else if (E <= 256) pdl_launch(router_topk_kernel<8>, blocks, 256, 0, s, logits, ld, T, E, topk, renorm, ids, weights, counts);
  else throw std::runtime_error("router_topk: at most 256 experts");
  check_launch("router_topk");
}

static PFN_cuTensorMapEncodeTiled_v12000 rt_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || p == nullptr)
      throw std::runtime_error("cuTensorMapEncodeTiled entry point not available");
    return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }();
  return fn;
}

// [rows, H] bf16, box 64 x box_rows, 128-byte swizzle; the last few maps are cached
static CUtensorMap rt_map(const void* base, int rows, int H, int box_rows) {
  struct Entry { const void* base; int rows, H, box; CUtensorMap map; };
  static thread_local std::vector<Entry> cache;
  for (auto& e : cache)
    if (e.base == base && e.rows == rows && e.H == H && e.box == box_rows) return e.map;
  CUtensorMap map;
  const cuuint64_t dims[2] = {(cuuint64_t)H, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)H * 2};
  const cuuint32_t box[2] = {(cuuint32_t)kRtK, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = rt_encode_fn()(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box,
                              estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw std::runtime_error("router tensor map: encode failed " + std::to_string((int)r));
  if (cache.size() >= 64) cache.erase(cache.begin());
  cache.push_back({base, rows, H, box_rows, map});
  return map;
}

void router_fused(const void* x, const void* w, int T, int H, int E, int w_rows, int topk, bool renorm, int* ids,
                  float* weights, int* counts, int* status, cudaStream_t s, float* part, int* tile_cnt,
                  int part_tiles, const EpArgs* ep) {
  if (T == 0) {
    // expert parallelism: a rank without tokens still publishes (zero counts) every layer
    if (ep != nullptr) ep_dispatch(*ep, x, ids, weights, 0, topk, s);
    return;
  }
  if (ep != nullptr && ep->hidden != H) throw std::runtime_error("router_fused: expert-parallel hidden mismatch");
  if (E > kRtE || w_rows < kRtE || topk < 1 || topk > 8 || H % kRtK)
    throw std::runtime_error("router_fused: needs <= 128 experts (weight padded to 128 rows), top-k in [1, 8], "
                             "hidden % 64 == 0");
  if ((reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(w) & 15))
    throw std::runtime_error("router_fused: operands must be 16-byte aligned");
  smem_opt_in(router_fused_kernel, kRtSmem);
  const CUtensorMap xm = rt_map(x, T, H, kRtTok);
  const CUtensorMap wm = rt_map(w, kRtE, H, kRtE);
  const int tiles = (T + kRtTok - 1) / kRtTok;
  // K splits: enough CTAs to cover the SMs once, at most 8 chunks' worth per split ... and never
  // more partial tiles than the scratch holds
  int ks = 1;
  if (part != nullptr && tile_cnt != nullptr) {
    const int sms = device_sm_count();
    while (ks < 8 && tiles * ks * 2 <= sms && (H / kRtK) >= ks * 2 * 2 && tiles * ks * 2 <= part_tiles) ks *= 2;
  }
  pdl_launch(router_fused_kernel, dim3(tiles, ks), 256, kRtSmem, s, xm, wm, T, H, E, topk, renorm ? 1 : 0, ids,
             weights, counts, status, part, tile_cnt, static_cast<const bf16*>(x), ep != nullptr ? *ep : EpArgs{},
             ep != nullptr ? 1 : 0);
  check_launch("router_fused");
}

void moe_permute(const void* x, const int* ids, int T, int topk, int E, int H, const int* counts, int* cursor,
                 void* x_perm, int* slot_of_row, int* offsets_out, cudaStream_t s) {
  if (E > kMaxExperts) throw std::runtime_error("moe_permute: too many experts");
  const int rows = T * topk;
  const int blocks = std::max(1, (rows * 32 + 255) / 256);
  pdl_launch(moe_permute_kernel, blocks, 256, 0, s, (const bf16*)x, ids, T, topk, E, H, counts, cursor, (bf16*)x_perm,
                                            slot_of_row, offsets_out);
  check_launch("moe_permute");
}

}  // namespace b200

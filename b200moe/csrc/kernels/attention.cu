// Paged-KV attention for Qwen3 GQA (sm_100a).
//
// KV pool layout per layer: [num_blocks, kv_heads, block_size, D] so that one
// (block, kv head) is a contiguous block_size x D slab; `block_stride` is the
// element distance between consecutive blocks (the pool interleaves layers).
//
// paged_decode_attn   one query per sequence.  Split-KV (flash-decoding): CTA =
//                     (split, kv head, sequence); the GQA group's G query heads
//                     are the MMA rows, so every K/V byte is read once per
//                     group.  64-key tiles are staged through shared memory with
//                     cp.async double buffering; each warp owns 16 keys of a tile
//                     and keeps its own online-softmax state; warps and splits
//                     are merged at the end.  Decode attention is bound by HBM
//                     (bytes of K/V per query head group), so the 16x8x16 bf16
//                     warp MMA is enough compute.
// paged_prefill_attn  varlen causal prefill / chunked prefill over the paged pool
//                     (prefix-cache hits and earlier chunks included).  CTA =
//                     (query block, kv head, sequence); the 64 MMA rows pack
//                     64/G query positions x G heads of one group, so K/V tiles
//                     are shared by the whole group.
//
// int8 KV: tiles are dequantised (per-token-head scale) while they are staged.
//
// Reference: Triton paged decode kernel nanovllm/kernels/paged_attention.py:74-190
// (one program per (batch, q head), no GQA sharing) and the per-sequence SDPA
// prefill loop nanovllm/layers/attention.py:179-213.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>
#include <algorithm>
#include <cstdint>
#include <cstdlib>
#include <mutex>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

#include "sm100.cuh"
#include "pdl.cuh"
#include "attention.h"

namespace b200 {

using bf16 = __nv_bfloat16;
constexpr int kKT = 64;  // keys per tile
constexpr int kKVStages = 3;  // K/V tiles in flight (cp.async groups)

// ------------------------------------------------------------- primitives
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  const int n = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(n) : "memory");
}
template <int N>  // 4 or 8 bytes (.ca: the 16-byte .cg form is cp_async16)
__device__ __forceinline__ void cp_async_small(uint32_t dst, const void* src, bool valid) {
  const int n = valid ? N : 0;
  asm volatile("cp.async.ca.shared.global [%0], [%1], %2, %3;" ::"r"(dst), "l"(src), "n"(N), "r"(n) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__device__ __forceinline__ void ldmatrix_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}
__device__ __forceinline__ void ldmatrix_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}
__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// Row-major [rows][D] bf16 tile with the 16-byte chunk index XOR-swizzled by row % 8.
template <int D>
__device__ __forceinline__ uint32_t tile_off(int row, int chunk) {
  return row * (D * 2) + ((chunk ^ (row & 7)) << 4);
}

// Load kKT keys [k0, k0+kKT) of kv head h into swizzled K and V tiles.  Keys at
// or beyond k_end are zero-filled and never read out of bounds.
template <int D, int NT>
__device__ __forceinline__ void load_kv_tile(uint32_t sk, uint32_t sv, const void* kc_, const void* vc_,
                                             const float* ks, const float* vs, bool int8, const int* btab,
                                             int bs, int64_t block_stride, int64_t sblock_stride, int h,
                                             int k0, int k_end, uint8_t* sk_gen, uint8_t* sv_gen,
                                             bool chan = false, KvChannel ch = KvChannel{}, int nkv = 0) {
  constexpr int CPR = D / 8;  // 16-byte chunks per bf16 row
  if (!int8) {
    const bf16* kc = static_cast<const bf16*>(kc_);
    const bf16* vc = static_cast<const bf16*>(vc_);
    // A thread's chunk column is fixed and its rows step by NT / CPR: gather all
    // its block-table entries first (independent loads), then issue the copies,
    // so no copy waits behind a table lookup.
    static_assert(NT % CPR == 0 && kKT % (NT / CPR) == 0, "tile / thread mapping");
    constexpr int RPI = NT / CPR;          // rows per iteration
    constexpr int ITERS = kKT / RPI;
    const int c = threadIdx.x % CPR, r0 = threadIdx.x / CPR;
    int64_t off[ITERS];
#pragma unroll
    for (int i = 0; i < ITERS; ++i) {
      const int key = k0 + r0 + i * RPI;
      off[i] = key < k_end ? (int64_t)btab[key / bs] * block_stride + ((int64_t)h * bs + key % bs) * D + c * 8
                           : -1;
    }
#pragma unroll
    for (int i = 0; i < ITERS; ++i) {
      const int r = r0 + i * RPI;
      const bool valid = off[i] >= 0;
      const int64_t o = valid ? off[i] : 0;
      cp_async16(sk + tile_off<D>(r, c), kc + o, valid);
      cp_async16(sv + tile_off<D>(r, c), vc + o, valid);
    }
    return;
  }
  // int8: 8 values per thread-iteration, dequantised into the bf16 tile
  const int8_t* kc = static_cast<const int8_t*>(kc_);
  const int8_t* vc = static_cast<const int8_t*>(vc_);
  if (chan) {
    // channel mode: q * per-channel read scale, then the head's exact outlier dims from the side pool
    const float* kds = ch.dscale + (size_t)h * D;
    const float* vds = ch.dscale + (size_t)(nkv + h) * D;
    const int n_out = ch.n_out[h];
    int od[kKvNoutMax];
#pragma unroll
    for (int i = 0; i < kKvNoutMax; ++i) od[i] = i < n_out ? ch.out_idx[h * kKvNoutMax + i] : -1;
    const bf16* sdk = static_cast<const bf16*>(ch.side_k);
    const bf16* sdv = static_cast<const bf16*>(ch.side_v);
    for (int idx = threadIdx.x; idx < kKT * CPR; idx += NT) {
      const int r = idx / CPR, c = idx % CPR;
      const int key = k0 + r;
      uint4 ko = make_uint4(0, 0, 0, 0), vo = make_uint4(0, 0, 0, 0);
      if (key < k_end) {
        const int blk = btab[key / bs];
        const int64_t tok = (int64_t)h * bs + key % bs;
        const int64_t off = (int64_t)blk * block_stride + tok * D + c * 8;
        const uint2 kq = *reinterpret_cast<const uint2*>(kc + off);
        const uint2 vq = *reinterpret_cast<const uint2*>(vc + off);
        const int8_t* kb = reinterpret_cast<const int8_t*>(&kq);
        const int8_t* vb = reinterpret_cast<const int8_t*>(&vq);
        float kf[8], vf[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          kf[j] = (float)kb[j] * kds[c * 8 + j];
          vf[j] = (float)vb[j] * vds[c * 8 + j];
        }
#pragma unroll
        for (int i = 0; i < kKvNoutMax; ++i) {
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            if (od[i] == c * 8 + j) {  // an exact bf16 value replaces the (zero) int8 payload
              const int64_t so = (int64_t)blk * ch.side_block_stride + tok * kKvNoutMax + i;
              kf[j] = __bfloat162float(sdk[so]);
              vf[j] = __bfloat162float(sdv[so]);
            }
          }
        }
        uint32_t kw[4], vw[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          kw[j] = pack_bf16(kf[2 * j], kf[2 * j + 1]);
          vw[j] = pack_bf16(vf[2 * j], vf[2 * j + 1]);
        }
        ko = make_uint4(kw[0], kw[1], kw[2], kw[3]);
        vo = make_uint4(vw[0], vw[1], vw[2], vw[3]);
      }
      *reinterpret_cast<uint4*>(sk_gen + tile_off<D>(r, c)) = ko;
      *reinterpret_cast<uint4*>(sv_gen + tile_off<D>(r, c)) = vo;
    }
    return;
  }
  for (int idx = threadIdx.x; idx < kKT * CPR; idx += NT) {
    const int r = idx / CPR, c = idx % CPR;
    const int key = k0 + r;
    uint4 ko = make_uint4(0, 0, 0, 0), vo = make_uint4(0, 0, 0, 0);
    if (key < k_end) {
      const int blk = btab[key / bs];
      const int64_t tok = (int64_t)h * bs + key % bs;
      const int64_t off = (int64_t)blk * block_stride + tok * D + c * 8;
      const float skl = ks[(int64_t)blk * sblock_stride + tok];
      const float svl = vs[(int64_t)blk * sblock_stride + tok];
      const uint2 kq = *reinterpret_cast<const uint2*>(kc + off);
      const uint2 vq = *reinterpret_cast<const uint2*>(vc + off);
      const int8_t* kb = reinterpret_cast<const int8_t*>(&kq);
      const int8_t* vb = reinterpret_cast<const int8_t*>(&vq);
      uint32_t kw[4], vw[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        kw[j] = pack_bf16(kb[2 * j] * skl, kb[2 * j + 1] * skl);
        vw[j] = pack_bf16(vb[2 * j] * svl, vb[2 * j + 1] * svl);
      }
      ko = make_uint4(kw[0], kw[1], kw[2], kw[3]);
      vo = make_uint4(vw[0], vw[1], vw[2], vw[3]);
    }
    *reinterpret_cast<uint4*>(sk_gen + tile_off<D>(r, c)) = ko;
    *reinterpret_cast<uint4*>(sv_gen + tile_off<D>(r, c)) = vo;
  }
}

// ------------------------------------------------ int8 decode: raw staging
// The int8 decode kernel copies each tile's raw payload (and its per-token scales,
// or the channel mode's outlier side values) with cp.async into a ring of raw
// slots, kKVStages tiles ahead, and dequantises one slot into the bf16 compute
// tile just before its MMAs: the global loads stay asynchronous, as in the bf16
// kernel, and the pool is read at one byte per value.
template <int D>
struct Int8Slots {
  static constexpr int RAW = kKT * D;               // bytes of one raw K (or V) tile
  static constexpr int SC = kKT * 4;                // per-token scales of one tile
  static constexpr int SIDE = kKT * kKvNoutMax * 2; // outlier side values of one tile
  static constexpr int BYTES = kKVStages * (RAW + SC + SIDE);
  static_assert(BYTES <= (kKVStages - 1) * kKT * D * 2, "int8 slots fit in the bf16 stages 1..S-1");
  __device__ static uint8_t* raw(uint8_t* base, int slot) { return base + slot * RAW; }
  __device__ static float* scale(uint8_t* base, int slot) {
    return reinterpret_cast<float*>(base + kKVStages * RAW + slot * SC);
  }
  __device__ static bf16* side(uint8_t* base, int slot) {
    return reinterpret_cast<bf16*>(base + kKVStages * (RAW + SC) + slot * SIDE);
  }
};

template <int D, int NT>
__device__ __forceinline__ void issue_int8_tile(uint8_t* kb, uint8_t* vb, int slot, const DecodeArgs& a,
                                                const int* btab, int64_t sbs, int h, int k0, int k_end) {
  using S = Int8Slots<D>;
  constexpr int CPR = D / 16;  // 16-byte chunks per int8 row
  static_assert(NT % CPR == 0 && kKT % (NT / CPR) == 0, "tile / thread mapping");
  constexpr int RPI = NT / CPR, ITERS = kKT / RPI;
  const int8_t* kc = static_cast<const int8_t*>(a.k_cache);
  const int8_t* vc = static_cast<const int8_t*>(a.v_cache);
  const int bs = a.block_size;
  const int c = threadIdx.x % CPR, r0 = threadIdx.x / CPR;
  int64_t off[ITERS];
#pragma unroll
  for (int i = 0; i < ITERS; ++i) {  // all block-table lookups first, then the copies
    const int key = k0 + r0 + i * RPI;
    off[i] = key < k_end ? (int64_t)btab[key / bs] * a.block_stride + ((int64_t)h * bs + key % bs) * D + c * 16 : -1;
  }
  const uint32_t rk = smem_u32(S::raw(kb, slot)), rv = smem_u32(S::raw(vb, slot));
#pragma unroll
  for (int i = 0; i < ITERS; ++i) {
    const int r = r0 + i * RPI;
    const bool valid = off[i] >= 0;
    const int64_t o = valid ? off[i] : 0;
    cp_async16(rk + r * D + c * 16, kc + o, valid);
    cp_async16(rv + r * D + c * 16, vc + o, valid);
  }
  for (int r = threadIdx.x; r < kKT; r += NT) {  // per-row metadata: one thread per key
    const int key = k0 + r;
    const bool valid = key < k_end;
    const int blk = valid ? btab[key / bs] : 0;
    const int64_t tok = valid ? (int64_t)h * bs + key % bs : 0;
    if (a.kv_int8 == 2) {
      const int64_t so = (int64_t)blk * a.ch.side_block_stride + tok * kKvNoutMax;
      cp_async_small<8>(smem_u32(S::side(kb, slot) + r * kKvNoutMax), static_cast<const bf16*>(a.ch.side_k) + so, valid);
      cp_async_small<8>(smem_u32(S::side(vb, slot) + r * kKvNoutMax), static_cast<const bf16*>(a.ch.side_v) + so, valid);
    } else {
      const int64_t so = (int64_t)blk * sbs + tok;
      cp_async_small<4>(smem_u32(S::scale(kb, slot) + r), a.k_scale + so, valid);
      cp_async_small<4>(smem_u32(S::scale(vb, slot) + r), a.v_scale + so, valid);
    }
  }
}

// Per-thread constants of the channel mode: the thread's 8-value column chunk is
// fixed (NT is a multiple of D / 8), so its read scales and outlier slots are too.
template <int D>
struct Int8Col {
  float kds[8], vds[8];
  int od[kKvNoutMax];  // outlier dim relative to the chunk start, -1 if none / elsewhere
};

template <int D, int NT>
__device__ __forceinline__ void int8_col_init(Int8Col<D>& col, const DecodeArgs& a, int h) {
  const int c = threadIdx.x % (D / 8);
  if (a.kv_int8 != 2) return;
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    col.kds[e] = a.ch.dscale[(size_t)h * D + c * 8 + e];
    col.vds[e] = a.ch.dscale[(size_t)(a.num_kv_heads + h) * D + c * 8 + e];
  }
  const int n_out = a.ch.n_out[h];
#pragma unroll
  for (int i = 0; i < kKvNoutMax; ++i) {
    const int d = i < n_out ? a.ch.out_idx[h * kKvNoutMax + i] - c * 8 : -1;
    col.od[i] = d >= 0 && d < 8 ? d : -1;
  }
}

__device__ __forceinline__ void int8x8_to_float(uint2 q, float (&f)[8]) {
  const uint32_t w[2] = {q.x, q.y};
#pragma unroll
  for (int e = 0; e < 8; ++e) f[e] = (float)(int8_t)((w[e >> 2] >> (8 * (e & 3))) & 0xffu);
}

// raw slot -> bf16 compute tiles (tile_off layout), the values load_kv_tile computes
template <int D, int NT>
__device__ __forceinline__ void dequant_int8_tile(uint8_t* kb, uint8_t* vb, int slot, uint8_t* tk, uint8_t* tv,
                                                  bool chan, const Int8Col<D>& col) {
  using S = Int8Slots<D>;
  constexpr int CPR = D / 8;
  const uint8_t* rk = S::raw(kb, slot);
  const uint8_t* rv = S::raw(vb, slot);
  for (int idx = threadIdx.x; idx < kKT * CPR; idx += NT) {
    const int r = idx / CPR, c = idx % CPR;
    float kf[8], vf[8];
    int8x8_to_float(*reinterpret_cast<const uint2*>(rk + r * D + c * 8), kf);
    int8x8_to_float(*reinterpret_cast<const uint2*>(rv + r * D + c * 8), vf);
    if (chan) {
      const bf16* sk = S::side(kb, slot) + r * kKvNoutMax;
      const bf16* sv = S::side(vb, slot) + r * kKvNoutMax;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        float x = kf[e] * col.kds[e], y = vf[e] * col.vds[e];
#pragma unroll
        for (int i = 0; i < kKvNoutMax; ++i) {
          x = col.od[i] == e ? __bfloat162float(sk[i]) : x;
          y = col.od[i] == e ? __bfloat162float(sv[i]) : y;
        }
        kf[e] = x;
        vf[e] = y;
      }
    } else {
      const float skl = S::scale(kb, slot)[r], svl = S::scale(vb, slot)[r];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        kf[e] *= skl;
        vf[e] *= svl;
      }
    }
    *reinterpret_cast<uint4*>(tk + tile_off<D>(r, c)) =
        make_uint4(pack_bf16(kf[0], kf[1]), pack_bf16(kf[2], kf[3]), pack_bf16(kf[4], kf[5]), pack_bf16(kf[6], kf[7]));
    *reinterpret_cast<uint4*>(tv + tile_off<D>(r, c)) =
        make_uint4(pack_bf16(vf[0], vf[1]), pack_bf16(vf[2], vf[3]), pack_bf16(vf[4], vf[5]), pack_bf16(vf[6], vf[7]));
  }
}

// 128B-swizzled tile as a TMA load with CU_TENSOR_MAP_SWIZZLE_128B writes it:
// [D / 64 halves][kKT rows][128 B], 16-byte unit u of row r stored at u ^ (r & 7).
template <int D>
__device__ __forceinline__ uint32_t swz_off(int row, int chunk) {
  return (chunk >> 3) * (kKT * 128) + row * 128 + (((chunk & 7) ^ (row & 7)) << 4);
}
template <int D, bool TMA>
__device__ __forceinline__ uint32_t kv_off(int row, int chunk) {
  if constexpr (TMA) return swz_off<D>(row, chunk);
  else return tile_off<D>(row, chunk);
}

// S[16 x 8*NB] = Q(frag) * K^T for keys [kbase, kbase + 8*NB) of the smem tile
template <int D, int NB, bool TMA = false>
__device__ __forceinline__ void qk_mma(float (&s)[NB][4], const uint32_t (&qf)[D / 16][4], uint32_t sk,
                                       int kbase, int lane) {
#pragma unroll
  for (int n = 0; n < NB; ++n)
#pragma unroll
    for (int e = 0; e < 4; ++e) s[n][e] = 0.f;
#pragma unroll
  for (int ks = 0; ks < D / 16; ++ks) {
#pragma unroll
    for (int n = 0; n < NB; n += 2) {
      // x4: (keys n*8.., d lo), (same keys, d hi), (keys +8, d lo), (keys +8, d hi)
      const int mi = lane >> 3, rr = lane & 7;
      const int key = kbase + n * 8 + (mi >> 1) * 8 + rr;
      const int chunk = ks * 2 + (mi & 1);
      uint32_t b0, b1, b2, b3;
      ldmatrix_x4(sk + kv_off<D, TMA>(key, chunk), b0, b1, b2, b3);
      mma16816(s[n], qf[ks], b0, b1);
      mma16816(s[n + 1], qf[ks], b2, b3);
    }
  }
}

// O[16 x D] += P(16 x 16 keys, bf16 A fragment) * V[keys kbase.., D]
template <int D, bool TMA = false>
__device__ __forceinline__ void pv_mma(float (&o)[D / 8][4], const uint32_t (&pf)[4], uint32_t sv, int kbase,
                                       int lane) {
#pragma unroll
  for (int n = 0; n < D / 8; n += 2) {
    // trans x4: (keys 0-7, d n*8), (keys 8-15, d n*8), (keys 0-7, d n*8+8), (keys 8-15, d n*8+8)
    const int mi = lane >> 3, rr = lane & 7;
    const int key = kbase + (mi & 1) * 8 + rr;
    const int chunk = n + (mi >> 1);
    uint32_t b0, b1, b2, b3;
    ldmatrix_x4_t(sv + kv_off<D, TMA>(key, chunk), b0, b1, b2, b3);
    mma16816(o[n], pf, b0, b1);
    mma16816(o[n + 1], pf, b2, b3);
  }
}

// online-softmax update of one 16-row fragment set; returns row correction factors
template <int NB>
__device__ __forceinline__ void softmax_update(float (&s)[NB][4], float (&m_r)[2], float (&l_r)[2],
                                               float (&corr)[2]) {
  float mx[2] = {m_r[0], m_r[1]};
#pragma unroll
  for (int n = 0; n < NB; ++n)
#pragma unroll
    for (int e = 0; e < 4; ++e) mx[e >> 1] = fmaxf(mx[e >> 1], s[n][e]);
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
    mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
    corr[r] = mx[r] == -INFINITY ? 1.f : exp2f(m_r[r] - mx[r]);
    m_r[r] = mx[r];
  }
  float rs[2] = {0.f, 0.f};
#pragma unroll
  for (int n = 0; n < NB; ++n)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float mm = m_r[e >> 1];
      const float p = mm == -INFINITY ? 0.f : exp2f(s[n][e] - mm);
      s[n][e] = p;
      rs[e >> 1] += p;
    }
#pragma unroll
  for (int r = 0; r < 2; ++r) l_r[r] = l_r[r] * corr[r] + rs[r];
}

// ================================================================== decode
// Q rows: r < G are heads h*G + r of the sequence's single query.
template <int D, bool INT8>
__global__ void __launch_bounds__(128) decode_attn_kernel(const DecodeArgs a) {
  pdl_enter();
  constexpr int NT = 128;
  extern __shared__ __align__(128) uint8_t smem[];
  const int b = blockIdx.z, h = blockIdx.y, split = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = a.group;
  const int L = a.seq_lens[b];
  const int k_begin = split * a.split_len;
  const int k_end = min(L, k_begin + a.split_len);
  const int nq = a.num_kv_heads * G;
  const int64_t sbs = a.block_stride / a.head_dim;  // int8 scale pool block stride

  uint8_t* sQ = smem;                                   // [16][D]
  uint8_t* sK = sQ + 16 * D * 2;                        // kKVStages x [64][D]
  uint8_t* sV = sK + kKVStages * kKT * D * 2;           // kKVStages x [64][D]
  float* sM = reinterpret_cast<float*>(sV + kKVStages * kKT * D * 2);  // [4][16]
  float* sL = sM + 64;                                  // [4][16]
  float* sO = reinterpret_cast<float*>(sK);             // [16][D], reuses the K tiles after the loop

  const bf16* qsrc = static_cast<const bf16*>(a.q) + ((size_t)b * nq + (size_t)h * G) * D;
  for (int idx = threadIdx.x; idx < 16 * (D / 8); idx += NT) {
    const int r = idx / (D / 8), c = idx % (D / 8);
    uint4 v = make_uint4(0, 0, 0, 0);
    if (r < G) v = *reinterpret_cast<const uint4*>(qsrc + (size_t)r * D + c * 8);
    *reinterpret_cast<uint4*>(sQ + tile_off<D>(r, c)) = v;
  }
  const int* btab = a.block_tables + (size_t)b * a.max_blocks;
  const uint32_t sk0 = smem_u32(sK), sv0 = smem_u32(sV);
  const int ntiles = k_end > k_begin ? (k_end - k_begin + kKT - 1) / kKT : 0;
  constexpr int TB = kKT * D * 2;  // bytes of one K (or V) tile
  // int8: raw slots live in the bf16 stages 1..S-1, stage 0 holds the dequantised compute tile
  uint8_t* const rawK = sK + TB;
  uint8_t* const rawV = sV + TB;
  const bool chan = a.kv_int8 == 2;
  Int8Col<D> col;
  if constexpr (INT8) int8_col_init<D, NT>(col, a, h);
#pragma unroll
  for (int p = 0; p < kKVStages - 1; ++p) {
    if (p < ntiles) {
      if constexpr (INT8)
        issue_int8_tile<D, NT>(rawK, rawV, p, a, btab, sbs, h, k_begin + p * kKT, k_end);
      else
        load_kv_tile<D, NT>(sk0 + p * TB, sv0 + p * TB, a.k_cache, a.v_cache, a.k_scale, a.v_scale, false, btab,
                            a.block_size, a.block_stride, sbs, h, k_begin + p * kKT, k_end, sK + p * TB,
                            sV + p * TB);
    }
    cp_async_commit();
  }
  __syncthreads();

  uint32_t qf[D / 16][4];
#pragma unroll
  for (int ks = 0; ks < D / 16; ++ks) {
    const int mi = lane >> 3, rr = lane & 7;
    // A x4: (rows 0-7, k lo), (rows 8-15, k lo), (rows 0-7, k hi), (rows 8-15, k hi)
    const int row = (mi & 1) * 8 + rr, chunk = ks * 2 + (mi >> 1);
    ldmatrix_x4(smem_u32(sQ) + tile_off<D>(row, chunk), qf[ks][0], qf[ks][1], qf[ks][2], qf[ks][3]);
  }

  const float sl2 = a.scale * 1.4426950408889634f;
  float m_r[2] = {-INFINITY, -INFINITY}, l_r[2] = {0.f, 0.f};
  float o[D / 8][4];
#pragma unroll
  for (int n = 0; n < D / 8; ++n)
#pragma unroll
    for (int e = 0; e < 4; ++e) o[n][e] = 0.f;

  for (int t = 0; t < ntiles; ++t) {
    const int buf = t % kKVStages;
    if (t + kKVStages - 1 < ntiles) {
      const int nb = (t + kKVStages - 1) % kKVStages;
      if constexpr (INT8)
        issue_int8_tile<D, NT>(rawK, rawV, nb, a, btab, sbs, h, k_begin + (t + kKVStages - 1) * kKT, k_end);
      else
        load_kv_tile<D, NT>(sk0 + nb * TB, sv0 + nb * TB, a.k_cache, a.v_cache, a.k_scale, a.v_scale, false, btab,
                            a.block_size, a.block_stride, sbs, h, k_begin + (t + kKVStages - 1) * kKT, k_end,
                            sK + nb * TB, sV + nb * TB);
    }
    cp_async_commit();
    cp_async_wait<kKVStages - 1>();
    __syncthreads();
    uint32_t sk = sk0 + buf * TB, sv = sv0 + buf * TB;
    if constexpr (INT8) {
      // the previous tile's MMAs finished at the loop-end barrier: stage 0 is free
      dequant_int8_tile<D, NT>(rawK, rawV, buf, sK, sV, chan, col);
      __syncthreads();
      sk = sk0;
      sv = sv0;
    }
    float s[2][4];
    qk_mma<D, 2>(s, qf, sk, warp * 16, lane);
    const int key0 = k_begin + t * kKT + warp * 16;
#pragma unroll
    for (int n = 0; n < 2; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int key = key0 + n * 8 + 2 * (lane & 3) + (e & 1);
        s[n][e] = key < k_end ? s[n][e] * sl2 : -INFINITY;
      }
    float corr[2];
    softmax_update<2>(s, m_r, l_r, corr);
#pragma unroll
    for (int n = 0; n < D / 8; ++n) {
      o[n][0] *= corr[0]; o[n][1] *= corr[0];
      o[n][2] *= corr[1]; o[n][3] *= corr[1];
    }
    uint32_t pf[4];
    pf[0] = pack_bf16(s[0][0], s[0][1]);
    pf[1] = pack_bf16(s[0][2], s[0][3]);
    pf[2] = pack_bf16(s[1][0], s[1][1]);
    pf[3] = pack_bf16(s[1][2], s[1][3]);
    pv_mma<D>(o, pf, sv, warp * 16, lane);
    __syncthreads();
  }
  cp_async_wait<0>();

  // ---- merge the 4 warps (each saw different keys)
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    float l = l_r[r];
    l += __shfl_xor_sync(0xffffffffu, l, 1);
    l += __shfl_xor_sync(0xffffffffu, l, 2);
    l_r[r] = l;
  }
  const int r0 = lane >> 2;
  if ((lane & 3) == 0) {
    sM[warp * 16 + r0] = m_r[0];
    sM[warp * 16 + r0 + 8] = m_r[1];
    sL[warp * 16 + r0] = l_r[0];
    sL[warp * 16 + r0 + 8] = l_r[1];
  }
  __syncthreads();  // every warp is done with the K/V tiles that sO reuses
  for (int i = threadIdx.x; i < 16 * D; i += NT) sO[i] = 0.f;
  __syncthreads();
  float wscale[2];
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int row = r0 + 8 * r;
    float m = -INFINITY;
    for (int w = 0; w < 4; ++w) m = fmaxf(m, sM[w * 16 + row]);
    wscale[r] = (m == -INFINITY || m_r[r] == -INFINITY) ? 0.f : exp2f(m_r[r] - m);
  }
  for (int w = 0; w < 4; ++w) {
    if (w == warp) {
#pragma unroll
      for (int n = 0; n < D / 8; ++n) {
        const int col = n * 8 + 2 * (lane & 3);
        sO[r0 * D + col] += o[n][0] * wscale[0];
        sO[r0 * D + col + 1] += o[n][1] * wscale[0];
        sO[(r0 + 8) * D + col] += o[n][2] * wscale[1];
        sO[(r0 + 8) * D + col + 1] += o[n][3] * wscale[1];
      }
    }
    __syncthreads();
  }
  for (int idx = threadIdx.x; idx < G * D; idx += NT) {
    const int row = idx / D, col = idx % D;
    float m = -INFINITY;
    for (int w = 0; w < 4; ++w) m = fmaxf(m, sM[w * 16 + row]);
    float l = 0.f;
    for (int w = 0; w < 4; ++w) {
      const float mw = sM[w * 16 + row];
      if (mw != -INFINITY) l += sL[w * 16 + row] * exp2f(mw - m);
    }
    const int head = h * G + row;
    if (a.num_splits == 1) {
      bf16* out = static_cast<bf16*>(a.out) + ((size_t)b * nq + head) * D;
      out[col] = __float2bfloat16(l > 0.f ? sO[row * D + col] / l : 0.f);
    } else {
      const size_t pidx = ((size_t)b * nq + head) * a.num_splits + split;
      a.part_o[pidx * D + col] = sO[row * D + col];
      if (col == 0) {
        a.part_m[pidx] = m;
        a.part_l[pidx] = l;
      }
    }
  }
  pdl_trigger();
}

template <int D>
__global__ void decode_combine_kernel(const DecodeArgs a) {
  pdl_enter();
  const int b = blockIdx.y, head = blockIdx.x;
  const int nq = a.num_kv_heads * a.group;
  const int L = a.seq_lens[b];
  const int nsplit = min(a.num_splits, (L + a.split_len - 1) / a.split_len);
  const size_t base = ((size_t)b * nq + head) * a.num_splits;
  float m = -INFINITY;
  for (int s = 0; s < nsplit; ++s) m = fmaxf(m, a.part_m[base + s]);
  float l = 0.f;
  for (int s = 0; s < nsplit; ++s) {
    const float ms = a.part_m[base + s];
    if (ms != -INFINITY) l += a.part_l[base + s] * exp2f(ms - m);
  }
  for (int col = threadIdx.x; col < D; col += blockDim.x) {
    float acc = 0.f;
    for (int s = 0; s < nsplit; ++s) {
      const float ms = a.part_m[base + s];
      if (ms != -INFINITY) acc += a.part_o[(base + s) * D + col] * exp2f(ms - m);
    }
    bf16* out = static_cast<bf16*>(a.out) + ((size_t)b * nq + head) * D;
    out[col] = __float2bfloat16(l > 0.f ? acc / l : 0.f);
  }
  pdl_trigger();
}

// ============================================================ decode (TMA)
// Same math and CTA mapping as decode_attn_kernel, restructured for sm_100a:
// a producer warp streams 64-key K/V tiles with TMA (128B-swizzled, one tensor
// map over the layer's pool planes) into a 3-stage ring guarded by full /
// empty mbarriers; four consumer warps (16 keys each) run the MMAs and an
// online softmax whose running max is moved only when a row's max grows by
// more than 2^8 (FlashAttention-3's lazy rescale), so the 64-multiply output
// rescale is skipped on most tiles.  Consumers issue no loads.
constexpr int kTmaStages = 3;
constexpr float kLazyLog2 = 8.f;

__device__ __forceinline__ void tma_load_4d(uint32_t dst, const CUtensorMap* map, uint64_t* bar, int x, int y, int z,
                                            int w) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];"
      ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z), "r"(w)
      : "memory");
}

template <int D>
struct DecTma {
  static constexpr int TILE = kKT * D * 2;                     // bytes of one K (or V) tile
  static constexpr int RING = kTmaStages * 2 * TILE;
  static constexpr int BTAB = 256;  // block-table entries of one split staged in shared memory
  static constexpr int SMEM = 1024 + RING + 16 * D * 2 + 2 * 64 * 4 + 2 * kTmaStages * 8 + 16 + BTAB * 4;
};

template <int D>
__global__ void __launch_bounds__(160) decode_attn_tma_kernel(const __grid_constant__ CUtensorMap kv_map,
                                                             const DecodeArgs a, int sub_rows, int oob_block) {
  pdl_enter();
  constexpr int NC = 128;  // consumer threads
  using C = DecTma<D>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ring = smem;                                   // stage s: K tile at s*2*TILE, V tile after it
  uint8_t* sQ = ring + C::RING;                           // [16][D]
  float* sM = reinterpret_cast<float*>(sQ + 16 * D * 2);  // [4][16]
  float* sL = sM + 64;
  uint64_t* full = reinterpret_cast<uint64_t*>(sL + 64);
  uint64_t* empty = full + kTmaStages;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + kTmaStages);
  int* sBt = reinterpret_cast<int*>(empty + kTmaStages) + 4;  // [BTAB] block ids of this split
  float* sO = reinterpret_cast<float*>(ring);             // [16][D], reuses the ring after the loop

  const int b = blockIdx.z, h = blockIdx.y, split = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = a.group;
  const int L = a.seq_lens[b];
  const int k_begin = split * a.split_len;
  const int k_end = min(L, k_begin + a.split_len);
  const int nq = a.num_kv_heads * G;
  const int ntiles = k_end > k_begin ? (k_end - k_begin + kKT - 1) / kKT : 0;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kTmaStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 4);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  const bf16* qsrc = static_cast<const bf16*>(a.q) + ((size_t)b * nq + (size_t)h * G) * D;
  for (int idx = threadIdx.x; idx < 16 * (D / 8); idx += blockDim.x) {
    const int r = idx / (D / 8), c = idx % (D / 8);
    uint4 v = make_uint4(0, 0, 0, 0);
    if (r < G) v = *reinterpret_cast<const uint4*>(qsrc + (size_t)r * D + c * 8);
    *reinterpret_cast<uint4*>(sQ + tile_off<D>(r, c)) = v;
  }
  __syncthreads();

  float m_r[2] = {-INFINITY, -INFINITY}, l_r[2] = {0.f, 0.f};
  float o[D / 8][4];
#pragma unroll
  for (int n = 0; n < D / 8; ++n)
#pragma unroll
    for (int e = 0; e < 4; ++e) o[n][e] = 0.f;

  if (warp == 4) {
    // ------------------------------------------------------------ producer
    // the split's block ids, gathered by the whole warp up front: no dependent
    // global load sits between two tile issues
    const int* btab = a.block_tables + (size_t)b * a.max_blocks;
    const int blk0 = k_begin / a.block_size;
    const int nblk = ntiles > 0 ? (k_end - 1) / a.block_size - blk0 + 1 : 0;
    const bool staged = nblk <= C::BTAB;
    if (staged)
      for (int i = lane; i < nblk; i += 32) sBt[i] = btab[blk0 + i];
    __syncwarp();
    if (lane == 0 && ntiles > 0) {
      tma_prefetch_desc(&kv_map);
      const int nsub = kKT / sub_rows;
      for (int t = 0; t < ntiles; ++t) {
        const int st = t % kTmaStages;
        const uint32_t ph = (t / kTmaStages) & 1;
        if (!mbar_wait(&empty[st], ph ^ 1, a.status, kStatusTimeoutEmpty, abort_flag)) break;
        mbar_arrive_expect_tx(&full[st], 2 * C::TILE);
        const uint32_t sk = smem_u32(ring + st * 2 * C::TILE), sv = sk + C::TILE;
        const int k0 = k_begin + t * kKT;
        for (int j = 0; j < nsub; ++j) {
          const int key = k0 + j * sub_rows;
          // keys past the sequence read a block coordinate outside the map: TMA zero-fills
          const int blk = key >= k_end ? oob_block
                          : staged ? sBt[key / a.block_size - blk0] : btab[key / a.block_size];
          const int y = key % a.block_size;
#pragma unroll
          for (int hf = 0; hf < D / 64; ++hf) {
            const uint32_t off = hf * (kKT * 128) + j * sub_rows * 128;
            tma_load_4d(sk + off, &kv_map, &full[st], hf * 64, y, h, blk);
            tma_load_4d(sv + off, &kv_map, &full[st], hf * 64, y, a.num_kv_heads + h, blk);
          }
        }
      }
      if (*abort_flag) {
        // a wait gave up: let loads already issued (valid sources) land before the CTA exits
        const uint64_t t0 = globaltimer_ns();
        while (globaltimer_ns() - t0 < 1000000ull) __nanosleep(1000);
      }
    }
  } else {
    // ------------------------------------------------------------ consumers
    uint32_t qf[D / 16][4];
#pragma unroll
    for (int ks = 0; ks < D / 16; ++ks) {
      const int mi = lane >> 3, rr = lane & 7;
      const int row = (mi & 1) * 8 + rr, chunk = ks * 2 + (mi >> 1);
      ldmatrix_x4(smem_u32(sQ) + tile_off<D>(row, chunk), qf[ks][0], qf[ks][1], qf[ks][2], qf[ks][3]);
    }
    const float sl2 = a.scale * 1.4426950408889634f;
    for (int t = 0; t < ntiles; ++t) {
      const int st = t % kTmaStages;
      const uint32_t ph = (t / kTmaStages) & 1;
      const bool ok = mbar_wait(&full[st], ph, a.status, kStatusTimeoutFull, abort_flag);
      if (!__all_sync(0xffffffffu, ok)) break;
      const uint32_t sk = smem_u32(ring + st * 2 * C::TILE), sv = sk + C::TILE;
      float sc[2][4];
      qk_mma<D, 2, true>(sc, qf, sk, warp * 16, lane);
      const int key0 = k_begin + t * kKT + warp * 16;
      float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
      for (int n = 0; n < 2; ++n)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int key = key0 + n * 8 + 2 * (lane & 3) + (e & 1);
          sc[n][e] = key < k_end ? sc[n][e] * sl2 : -INFINITY;
          mx[e >> 1] = fmaxf(mx[e >> 1], sc[n][e]);
        }
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
        mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
      }
      // lazy rescale: move the reference max only when a row grew by > 2^8
      const bool grow0 = mx[0] > m_r[0] + kLazyLog2, grow1 = mx[1] > m_r[1] + kLazyLog2;
      if (__any_sync(0xffffffffu, grow0 || grow1)) {
        float corr[2];
#pragma unroll
        for (int r = 0; r < 2; ++r) {
          const bool g = r ? grow1 : grow0;
          const float mn = g ? mx[r] : m_r[r];
          corr[r] = (m_r[r] == -INFINITY || !g) ? 1.f : exp2f(m_r[r] - mn);
          m_r[r] = mn;
          l_r[r] *= corr[r];
        }
#pragma unroll
        for (int n = 0; n < D / 8; ++n) {
          o[n][0] *= corr[0]; o[n][1] *= corr[0];
          o[n][2] *= corr[1]; o[n][3] *= corr[1];
        }
      }
#pragma unroll
      for (int n = 0; n < 2; ++n)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float mm = m_r[e >> 1];
          const float p = mm == -INFINITY ? 0.f : exp2f(sc[n][e] - mm);
          sc[n][e] = p;
          l_r[e >> 1] += p;
        }
      uint32_t pf[4];
      pf[0] = pack_bf16(sc[0][0], sc[0][1]);
      pf[1] = pack_bf16(sc[0][2], sc[0][3]);
      pf[2] = pack_bf16(sc[1][0], sc[1][1]);
      pf[3] = pack_bf16(sc[1][2], sc[1][3]);
      pv_mma<D, true>(o, pf, sv, warp * 16, lane);
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[st]);  // this warp is done with the stage
    }
  }

  // ---- merge the 4 consumer warps (each saw different keys); the producer warp only syncs
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    float l = l_r[r];
    l += __shfl_xor_sync(0xffffffffu, l, 1);
    l += __shfl_xor_sync(0xffffffffu, l, 2);
    l_r[r] = l;
  }
  const int r0 = lane >> 2;
  if (warp < 4 && (lane & 3) == 0) {
    sM[warp * 16 + r0] = m_r[0];
    sM[warp * 16 + r0 + 8] = m_r[1];
    sL[warp * 16 + r0] = l_r[0];
    sL[warp * 16 + r0 + 8] = l_r[1];
  }
  __syncthreads();  // every TMA write and every consumer read of the ring is complete
  for (int i = threadIdx.x; i < 16 * D; i += blockDim.x) sO[i] = 0.f;
  __syncthreads();
  if (warp < 4) {
    float wscale[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const int row = r0 + 8 * r;
      float m = -INFINITY;
      for (int w = 0; w < 4; ++w) m = fmaxf(m, sM[w * 16 + row]);
      wscale[r] = (m == -INFINITY || m_r[r] == -INFINITY) ? 0.f : exp2f(m_r[r] - m);
    }
    for (int w = 0; w < 4; ++w) {
      if (w == warp) {
#pragma unroll
        for (int n = 0; n < D / 8; ++n) {
          const int col = n * 8 + 2 * (lane & 3);
          sO[r0 * D + col] += o[n][0] * wscale[0];
          sO[r0 * D + col + 1] += o[n][1] * wscale[0];
          sO[(r0 + 8) * D + col] += o[n][2] * wscale[1];
          sO[(r0 + 8) * D + col + 1] += o[n][3] * wscale[1];
        }
      }
      named_barrier_sync(1, NC);
    }
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < G * D; idx += blockDim.x) {
    const int row = idx / D, col = idx % D;
    float m = -INFINITY;
    for (int w = 0; w < 4; ++w) m = fmaxf(m, sM[w * 16 + row]);
    float l = 0.f;
    for (int w = 0; w < 4; ++w) {
      const float mw = sM[w * 16 + row];
      if (mw != -INFINITY) l += sL[w * 16 + row] * exp2f(mw - m);
    }
    const int head = h * G + row;
    if (a.num_splits == 1) {
      bf16* out = static_cast<bf16*>(a.out) + ((size_t)b * nq + head) * D;
      out[col] = __float2bfloat16(l > 0.f ? sO[row * D + col] / l : 0.f);
    } else {
      const size_t pidx = ((size_t)b * nq + head) * a.num_splits + split;
      a.part_o[pidx * D + col] = sO[row * D + col];
      if (col == 0) {
        a.part_m[pidx] = m;
        a.part_l[pidx] = l;
      }
    }
  }
  pdl_trigger();
}

// ------------------------------------------------- persistent TMA decode
// Same tile pipeline as decode_attn_tma_kernel, but a CTA (two per SM) walks a
// strided list of (sequence, kv head, split) items and its producer warp streams
// the next item's tiles while the consumer warps finish the current one: the
// per-item set-up (Q staging, block-table gather, pipeline fill) and the
// cross-warp merge no longer leave the ring idle, and there is no wave tail.
template <int D>
struct DecPersist {
  static constexpr int TILE = kKT * D * 2;
  static constexpr int RING = kTmaStages * 2 * TILE;
  static constexpr int BTAB = 256;
  static constexpr int SMEM = 1024 + RING + 16 * D * 2 + 16 * D * 4 + 2 * 64 * 4 + 2 * kTmaStages * 8 + 16 + BTAB * 4 + 16;
};

template <int D>
__global__ void __launch_bounds__(160) decode_attn_persist_kernel(const __grid_constant__ CUtensorMap kv_map,
                                                                 const DecodeArgs a, int sub_rows, int oob_block,
                                                                 int n_items) {
  pdl_enter();
  constexpr int NC = 128;  // consumer threads
  using C = DecPersist<D>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ring = smem;                                      // stage s: K tile at s*2*TILE, V tile after it
  uint8_t* sQ = ring + C::RING;                              // [16][D] bf16
  float* sO = reinterpret_cast<float*>(sQ + 16 * D * 2);     // [16][D] merged output of the current item
  float* sM = sO + 16 * D;                                   // [4][16]
  float* sL = sM + 64;
  uint64_t* full = reinterpret_cast<uint64_t*>(sL + 64);
  uint64_t* empty = full + kTmaStages;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + kTmaStages);
  int* sBt = reinterpret_cast<int*>(empty + kTmaStages) + 4;  // [BTAB] block ids of the producer's item
  volatile int* sStop = sBt + C::BTAB;  // consumers' copy of the abort flag (read between their barriers)

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = a.group;
  const int nq = a.num_kv_heads * G;
  const int S = a.num_splits;
  if (threadIdx.x == 0) {
    for (int i = 0; i < kTmaStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 4);
    }
    *abort_flag = 0;
    *sStop = 0;
    fence_barrier_init();
  }
  for (int i = threadIdx.x; i < 16 * D; i += blockDim.x) sO[i] = 0.f;
  __syncthreads();

  // item w -> (sequence b, kv head h, split), keys [k_begin, k_end)
  struct Item { int b, h, split, k_begin, k_end, ntiles; };
  auto item = [&](int w) {
    Item it;
    it.split = w % S;
    w /= S;
    it.h = w % a.num_kv_heads;
    it.b = w / a.num_kv_heads;
    const int L = a.seq_lens[it.b];
    it.k_begin = it.split * a.split_len;
    it.k_end = min(L, it.k_begin + a.split_len);
    it.ntiles = it.k_end > it.k_begin ? (it.k_end - it.k_begin + kKT - 1) / kKT : 0;
    return it;
  };

  if (warp == 4) {
    // ------------------------------------------------------------ producer
    int tc = 0;  // tiles issued by this CTA (ring position)
    for (int w = blockIdx.x; w < n_items && !*abort_flag; w += gridDim.x) {
      const Item it = item(w);
      if (it.ntiles == 0) continue;
      const int* btab = a.block_tables + (size_t)it.b * a.max_blocks;
      const int blk0 = it.k_begin / a.block_size;
      const int nblk = (it.k_end - 1) / a.block_size - blk0 + 1;
      const bool staged = nblk <= C::BTAB;
      if (staged)
        for (int i = lane; i < nblk; i += 32) sBt[i] = btab[blk0 + i];
      __syncwarp();
      if (lane == 0) {
        if (w == (int)blockIdx.x) tma_prefetch_desc(&kv_map);
        const int nsub = kKT / sub_rows;
        for (int t = 0; t < it.ntiles; ++t, ++tc) {
          const int st = tc % kTmaStages;
          const uint32_t ph = (tc / kTmaStages) & 1;
          if (!mbar_wait(&empty[st], ph ^ 1, a.status, kStatusTimeoutEmpty, abort_flag)) break;
          mbar_arrive_expect_tx(&full[st], 2 * C::TILE);
          const uint32_t sk = smem_u32(ring + st * 2 * C::TILE), sv = sk + C::TILE;
          const int k0 = it.k_begin + t * kKT;
          for (int j = 0; j < nsub; ++j) {
            const int key = k0 + j * sub_rows;
            // keys past the sequence read a block coordinate outside the map: TMA zero-fills
            const int blk = key >= it.k_end ? oob_block
                            : staged ? sBt[key / a.block_size - blk0] : btab[key / a.block_size];
            const int y = key % a.block_size;
#pragma unroll
            for (int hf = 0; hf < D / 64; ++hf) {
              const uint32_t off = hf * (kKT * 128) + j * sub_rows * 128;
              tma_load_4d(sk + off, &kv_map, &full[st], hf * 64, y, it.h, blk);
              tma_load_4d(sv + off, &kv_map, &full[st], hf * 64, y, a.num_kv_heads + it.h, blk);
            }
          }
        }
      }
      tc = __shfl_sync(0xffffffffu, tc, 0);
      __syncwarp();  // lane 0 has issued every tile of the item before sBt is overwritten
    }
    if (lane == 0 && *abort_flag) {
      // a wait gave up: let loads already issued (valid sources) land before the CTA exits
      const uint64_t t0 = globaltimer_ns();
      while (globaltimer_ns() - t0 < 1000000ull) __nanosleep(1000);
    }
  } else {
    // ------------------------------------------------------------ consumers
    const float sl2 = a.scale * 1.4426950408889634f;
    const int r0 = lane >> 2;
    int tc = 0;
    bool ok = true;
    for (int w = blockIdx.x; w < n_items; w += gridDim.x) {
      const Item it = item(w);
      if (it.ntiles == 0) continue;
      named_barrier_sync(1, NC);  // the previous item's readers of sQ / sM / sL are done
      // every consumer warp takes the same exit (a divergent one would strand the
      // others at a named barrier): the flag copy was written before the last barrier
      if (*sStop) break;
      const bf16* qsrc = static_cast<const bf16*>(a.q) + ((size_t)it.b * nq + (size_t)it.h * G) * D;
      for (int idx = threadIdx.x; idx < 16 * (D / 8); idx += NC) {
        const int r = idx / (D / 8), c = idx % (D / 8);
        uint4 v = make_uint4(0, 0, 0, 0);
        if (r < G) v = *reinterpret_cast<const uint4*>(qsrc + (size_t)r * D + c * 8);
        *reinterpret_cast<uint4*>(sQ + tile_off<D>(r, c)) = v;
      }
      named_barrier_sync(1, NC);
      uint32_t qf[D / 16][4];
#pragma unroll
      for (int ks = 0; ks < D / 16; ++ks) {
        const int mi = lane >> 3, rr = lane & 7;
        const int row = (mi & 1) * 8 + rr, chunk = ks * 2 + (mi >> 1);
        ldmatrix_x4(smem_u32(sQ) + tile_off<D>(row, chunk), qf[ks][0], qf[ks][1], qf[ks][2], qf[ks][3]);
      }
      float m_r[2] = {-INFINITY, -INFINITY}, l_r[2] = {0.f, 0.f};
      float o[D / 8][4];
#pragma unroll
      for (int n = 0; n < D / 8; ++n)
#pragma unroll
        for (int e = 0; e < 4; ++e) o[n][e] = 0.f;
      for (int t = 0; t < it.ntiles; ++t, ++tc) {
        const int st = tc % kTmaStages;
        const uint32_t ph = (tc / kTmaStages) & 1;
        ok = mbar_wait(&full[st], ph, a.status, kStatusTimeoutFull, abort_flag);
        if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
        const uint32_t sk = smem_u32(ring + st * 2 * C::TILE), sv = sk + C::TILE;
        float sc[2][4];
        qk_mma<D, 2, true>(sc, qf, sk, warp * 16, lane);
        const int key0 = it.k_begin + t * kKT + warp * 16;
        float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
        for (int n = 0; n < 2; ++n)
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int key = key0 + n * 8 + 2 * (lane & 3) + (e & 1);
            sc[n][e] = key < it.k_end ? sc[n][e] * sl2 : -INFINITY;
            mx[e >> 1] = fmaxf(mx[e >> 1], sc[n][e]);
          }
#pragma unroll
        for (int r = 0; r < 2; ++r) {
          mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
          mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
        }
        // lazy rescale: move the reference max only when a row grew by > 2^8
        const bool grow0 = mx[0] > m_r[0] + kLazyLog2, grow1 = mx[1] > m_r[1] + kLazyLog2;
        if (__any_sync(0xffffffffu, grow0 || grow1)) {
          float corr[2];
#pragma unroll
          for (int r = 0; r < 2; ++r) {
            const bool g = r ? grow1 : grow0;
            const float mn = g ? mx[r] : m_r[r];
            corr[r] = (m_r[r] == -INFINITY || !g) ? 1.f : exp2f(m_r[r] - mn);
            m_r[r] = mn;
            l_r[r] *= corr[r];
          }
#pragma unroll
          for (int n = 0; n < D / 8; ++n) {
            o[n][0] *= corr[0]; o[n][1] *= corr[0];
            o[n][2] *= corr[1]; o[n][3] *= corr[1];
          }
        }
#pragma unroll
        for (int n = 0; n < 2; ++n)
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float mm = m_r[e >> 1];
            const float p = mm == -INFINITY ? 0.f : exp2f(sc[n][e] - mm);
            sc[n][e] = p;
            l_r[e >> 1] += p;
          }
        uint32_t pf[4];
        pf[0] = pack_bf16(sc[0][0], sc[0][1]);
        pf[1] = pack_bf16(sc[0][2], sc[0][3]);
        pf[2] = pack_bf16(sc[1][0], sc[1][1]);
        pf[3] = pack_bf16(sc[1][2], sc[1][3]);
        pv_mma<D, true>(o, pf, sv, warp * 16, lane);
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[st]);  // this warp is done with the stage
      }
      if (!__all_sync(0xffffffffu, ok)) { ok = false; }
      // ---- merge the 4 warps (each saw a quarter of every tile's keys) into sO
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        float l = l_r[r];
        l += __shfl_xor_sync(0xffffffffu, l, 1);
        l += __shfl_xor_sync(0xffffffffu, l, 2);
        l_r[r] = l;
      }
      if ((lane & 3) == 0) {
        sM[warp * 16 + r0] = m_r[0];
        sM[warp * 16 + r0 + 8] = m_r[1];
        sL[warp * 16 + r0] = l_r[0];
        sL[warp * 16 + r0 + 8] = l_r[1];
      }
      named_barrier_sync(1, NC);
      float wscale[2];
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        const int row = r0 + 8 * r;
        float m = -INFINITY;
        for (int q = 0; q < 4; ++q) m = fmaxf(m, sM[q * 16 + row]);
        wscale[r] = (m == -INFINITY || m_r[r] == -INFINITY) ? 0.f : exp2f(m_r[r] - m);
      }
      if (r0 < G) {
#pragma unroll
        for (int n = 0; n < D / 8; ++n) {
          const int col = n * 8 + 2 * (lane & 3);
          atomicAdd(&sO[r0 * D + col], o[n][0] * wscale[0]);
          atomicAdd(&sO[r0 * D + col + 1], o[n][1] * wscale[0]);
        }
      }
      if (r0 + 8 < G) {
#pragma unroll
        for (int n = 0; n < D / 8; ++n) {
          const int col = n * 8 + 2 * (lane & 3);
          atomicAdd(&sO[(r0 + 8) * D + col], o[n][2] * wscale[1]);
          atomicAdd(&sO[(r0 + 8) * D + col + 1], o[n][3] * wscale[1]);
        }
      }
      if (threadIdx.x == 0) *sStop = *abort_flag;
      named_barrier_sync(1, NC);
      for (int idx = threadIdx.x; idx < G * D; idx += NC) {
        const int row = idx / D, col = idx % D;
        float m = -INFINITY;
        for (int q = 0; q < 4; ++q) m = fmaxf(m, sM[q * 16 + row]);
        float l = 0.f;
        for (int q = 0; q < 4; ++q) {
          const float mw = sM[q * 16 + row];
          if (mw != -INFINITY) l += sL[q * 16 + row] * exp2f(mw - m);
        }
        const float v = sO[idx];
        sO[idx] = 0.f;  // ready for the next item (only this thread touches idx here)
        const int head = it.h * G + row;
        if (S == 1) {
          bf16* out = static_cast<bf16*>(a.out) + ((size_t)it.b * nq + head) * D;
          out[col] = __float2bfloat16(l > 0.f ? v / l : 0.f);
        } else {
          const size_t pidx = ((size_t)it.b * nq + head) * S + it.split;
          a.part_o[pidx * D + col] = v;
          if (col == 0) {
            a.part_m[pidx] = m;
            a.part_l[pidx] = l;
          }
        }
      }
    }
  }
  __syncthreads();
  pdl_trigger();
}

// ================================================================= prefill
// Packed rows: r -> query position qb*QPB + r / G, head h*G + r % G.
template <int D>
__global__ void __launch_bounds__(128) prefill_attn_kernel(const PrefillArgs a) {
  pdl_enter();
  constexpr int NT = 128;
  extern __shared__ __align__(128) uint8_t smem[];
  const int b = blockIdx.z, h = blockIdx.y, qb = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = a.group;
  const int QPB = 64 / G;
  const int q0 = a.cu_seqlens_q[b];
  const int q_len = a.cu_seqlens_q[b + 1] - q0;
  if (qb * QPB >= q_len) return;
  const int kv_len = a.seq_lens[b];
  const int pos0 = kv_len - q_len;  // position of query 0
  const int nq = a.num_kv_heads * G;
  const bool int8 = a.kv_int8 != 0;
  const int64_t sbs = a.block_stride / a.head_dim;

  uint8_t* sQ = smem;                     // [64][D]
  uint8_t* sK = sQ + 64 * D * 2;          // kKVStages x [64][D]
  uint8_t* sV = sK + kKVStages * kKT * D * 2;

  const bf16* q = static_cast<const bf16*>(a.q);
  for (int idx = threadIdx.x; idx < 64 * (D / 8); idx += NT) {
    const int r = idx / (D / 8), c = idx % (D / 8);
    const int qi = qb * QPB + r / G, head = h * G + r % G;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (qi < q_len) v = *reinterpret_cast<const uint4*>(q + ((size_t)(q0 + qi) * nq + head) * D + c * 8);
    *reinterpret_cast<uint4*>(sQ + tile_off<D>(r, c)) = v;
  }
  const int* btab = a.block_tables + (size_t)b * a.max_blocks;
  const int last_q = min(q_len, (qb + 1) * QPB) - 1;
  const int k_end = min(kv_len, pos0 + last_q + 1);  // causal bound of the block's last query
  const int ntiles = (k_end + kKT - 1) / kKT;
  const uint32_t sk0 = smem_u32(sK), sv0 = smem_u32(sV);
  constexpr int TB = kKT * D * 2;
#pragma unroll
  for (int p = 0; p < kKVStages - 1; ++p) {
    if (p < ntiles)
      load_kv_tile<D, NT>(sk0 + p * TB, sv0 + p * TB, a.k_cache, a.v_cache, a.k_scale, a.v_scale, int8, btab,
                          a.block_size, a.block_stride, sbs, h, p * kKT, k_end, sK + p * TB, sV + p * TB,
                          a.kv_int8 == 2, a.ch, a.num_kv_heads);
    cp_async_commit();
  }
  __syncthreads();

  uint32_t qf[D / 16][4];
#pragma unroll
  for (int ks = 0; ks < D / 16; ++ks) {
    const int mi = lane >> 3, rr = lane & 7;
    const int row = warp * 16 + (mi & 1) * 8 + rr, chunk = ks * 2 + (mi >> 1);
    ldmatrix_x4(smem_u32(sQ) + tile_off<D>(row, chunk), qf[ks][0], qf[ks][1], qf[ks][2], qf[ks][3]);
  }
  int qpos[2];
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int row = warp * 16 + (lane >> 2) + 8 * r;
    const int qi = qb * QPB + row / G;
    qpos[r] = qi < q_len ? pos0 + qi : -1;
  }
  const float sl2 = a.scale * 1.4426950408889634f;
  float m_r[2] = {-INFINITY, -INFINITY}, l_r[2] = {0.f, 0.f};
  float o[D / 8][4];
#pragma unroll
  for (int n = 0; n < D / 8; ++n)
#pragma unroll
    for (int e = 0; e < 4; ++e) o[n][e] = 0.f;

  for (int t = 0; t < ntiles; ++t) {
    const int buf = t % kKVStages;
    if (t + kKVStages - 1 < ntiles) {
      const int nb = (t + kKVStages - 1) % kKVStages;
      load_kv_tile<D, NT>(sk0 + nb * TB, sv0 + nb * TB, a.k_cache, a.v_cache, a.k_scale, a.v_scale, int8, btab,
                          a.block_size, a.block_stride, sbs, h, (t + kKVStages - 1) * kKT, k_end, sK + nb * TB,
                          sV + nb * TB, a.kv_int8 == 2, a.ch, a.num_kv_heads);
    }
    cp_async_commit();
    cp_async_wait<kKVStages - 1>();
    __syncthreads();
    const uint32_t sk = sk0 + buf * TB, sv = sv0 + buf * TB;
    float s[8][4];
    qk_mma<D, 8>(s, qf, sk, 0, lane);
#pragma unroll
    for (int n = 0; n < 8; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int key = t * kKT + n * 8 + 2 * (lane & 3) + (e & 1);
        s[n][e] = (key <= qpos[e >> 1]) ? s[n][e] * sl2 : -INFINITY;
      }
    float corr[2];
    softmax_update<8>(s, m_r, l_r, corr);
#pragma unroll
    for (int n = 0; n < D / 8; ++n) {
      o[n][0] *= corr[0]; o[n][1] *= corr[0];
      o[n][2] *= corr[1]; o[n][3] *= corr[1];
    }
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {  // 16-key chunks of the 64-key tile
      uint32_t pf[4];
      pf[0] = pack_bf16(s[2 * kk][0], s[2 * kk][1]);
      pf[1] = pack_bf16(s[2 * kk][2], s[2 * kk][3]);
      pf[2] = pack_bf16(s[2 * kk + 1][0], s[2 * kk + 1][1]);
      pf[3] = pack_bf16(s[2 * kk + 1][2], s[2 * kk + 1][3]);
      pv_mma<D>(o, pf, sv, kk * 16, lane);
    }
    __syncthreads();
  }
  cp_async_wait<0>();
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    float l = l_r[r];
    l += __shfl_xor_sync(0xffffffffu, l, 1);
    l += __shfl_xor_sync(0xffffffffu, l, 2);
    l_r[r] = l;
  }
  bf16* out = static_cast<bf16*>(a.out);
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int row = warp * 16 + (lane >> 2) + 8 * r;
    const int qi = qb * QPB + row / G, head = h * G + row % G;
    if (qi >= q_len) continue;
    const float inv = l_r[r] > 0.f ? 1.f / l_r[r] : 0.f;
    bf16* dst = out + ((size_t)(q0 + qi) * nq + head) * D;
#pragma unroll
    for (int n = 0; n < D / 8; ++n) {
      const int col = n * 8 + 2 * (lane & 3);
      *reinterpret_cast<uint32_t*>(dst + col) = pack_bf16(o[n][2 * r] * inv, o[n][2 * r + 1] * inv);
    }
  }
  pdl_trigger();
}

// --------------------------------------------------------------- launchers
static void check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

template <int D>
static int decode_smem() { return 16 * D * 2 + 2 * kKVStages * kKT * D * 2 + 2 * 64 * 4; }
template <int D>
static int prefill_smem() { return 64 * D * 2 + 2 * kKVStages * kKT * D * 2; }

// ---- TMA tensor map of one layer's pool planes: dims {D, block_size, 2 * kv_heads
// (K heads then V heads), blocks}, box {64, rows, 1, 1}, 128-byte swizzle.
static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (fn == nullptr) {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || p == nullptr)
      throw std::runtime_error("cuTensorMapEncodeTiled entry point not available");
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

struct KvMapKey {
  const void* base;
  int dev, D, bs, kvh, nblocks, sub_rows;
  int64_t block_stride;
  bool operator==(const KvMapKey& o) const {
    return base == o.base && dev == o.dev && D == o.D && bs == o.bs && kvh == o.kvh && nblocks == o.nblocks &&
           sub_rows == o.sub_rows && block_stride == o.block_stride;
  }
};

// Returned by value: the cache may be cleared by another thread's call.
static CUtensorMap kv_tensor_map(const DecodeArgs& a, int sub_rows) {
  static std::mutex mu;
  static std::vector<std::pair<KvMapKey, CUtensorMap>> cache;  // one entry per layer of a pool
  const KvMapKey key{a.k_cache, current_device(), a.head_dim, a.block_size, a.num_kv_heads, a.num_blocks,
                     sub_rows, a.block_stride};
  std::lock_guard<std::mutex> lock(mu);
  for (auto& e : cache)
    if (e.first == key) return e.second;
  CUtensorMap map;
  const cuuint64_t dims[4] = {(cuuint64_t)a.head_dim, (cuuint64_t)a.block_size, (cuuint64_t)(2 * a.num_kv_heads),
                              (cuuint64_t)a.num_blocks};
  const cuuint64_t strides[3] = {(cuuint64_t)a.head_dim * 2, (cuuint64_t)a.block_size * a.head_dim * 2,
                                 (cuuint64_t)a.block_stride * 2};
  const cuuint32_t box[4] = {64, (cuuint32_t)sub_rows, 1, 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = encode_fn()(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(a.k_cache), dims, strides,
                           box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw std::runtime_error("kv tensor map: cuTensorMapEncodeTiled failed " + std::to_string((int)r));
  if (cache.size() > 512) cache.clear();
  cache.emplace_back(key, map);
  return cache.back().second;
}

// The TMA kernel needs a bf16 pool whose V planes follow the K planes of the same
// layer and block (the pool layout), 64-key tiles that stay inside one block or
// cover whole blocks, and 16-byte aligned planes.
static bool use_tma_decode(const DecodeArgs& a, int* sub_rows) {
  static const bool enabled = [] {
    const char* e = std::getenv("B200MOE_DECODE_TMA");
    return e == nullptr || std::string(e) != "0";
  }();
  if (!enabled || a.kv_int8 || a.num_blocks <= 0) return false;
  if (a.head_dim != 64 && a.head_dim != 128) return false;
  const bf16* k = static_cast<const bf16*>(a.k_cache);
  if (static_cast<const bf16*>(a.v_cache) != k + (int64_t)a.num_kv_heads * a.block_size * a.head_dim) return false;
  if ((reinterpret_cast<uintptr_t>(a.k_cache) & 15) || (a.block_stride * 2) % 16) return false;
  if (a.block_size % kKT == 0) *sub_rows = kKT;
  else if (kKT % a.block_size == 0 && a.block_size % 8 == 0) *sub_rows = a.block_size;
  else return false;
  return true;
}

static int num_sms_attn() { return device_sm_count(); }

template <int D>
static void launch_decode_tma(const DecodeArgs& a, int B, int sub_rows, cudaStream_t s) {
  const CUtensorMap map = kv_tensor_map(a, sub_rows);
  static const bool persist = [] {
    const char* e = std::getenv("B200MOE_DECODE_PERSIST");
    return e == nullptr || std::string(e) != "0";
  }();
  if (persist) {
    smem_opt_in(decode_attn_persist_kernel<D>, DecPersist<D>::SMEM);
    const int n_items = a.num_splits * a.num_kv_heads * B;
    const int grid = std::max(1, std::min(n_items, 2 * num_sms_attn()));
    pdl_launch(decode_attn_persist_kernel<D>, grid, 160, DecPersist<D>::SMEM, s, map, a, sub_rows, a.num_blocks, n_items);
    if (a.num_splits > 1) pdl_launch(decode_combine_kernel<D>, dim3(a.num_kv_heads * a.group, B), D, 0, s, a);
    return;
  }
  smem_opt_in(decode_attn_tma_kernel<D>, DecTma<D>::SMEM);
  dim3 grid(a.num_splits, a.num_kv_heads, B);
  pdl_launch(decode_attn_tma_kernel<D>, grid, 160, DecTma<D>::SMEM, s, map, a, sub_rows, a.num_blocks);
  if (a.num_splits > 1) pdl_launch(decode_combine_kernel<D>, dim3(a.num_kv_heads * a.group, B), D, 0, s, a);
}

template <int D>
static void launch_decode_split(const DecodeArgs& a, int B, dim3 grid, cudaStream_t s) {
  if (a.kv_int8) {
    smem_opt_in(decode_attn_kernel<D, true>, decode_smem<D>());
    pdl_launch(decode_attn_kernel<D, true>, grid, 128, decode_smem<D>(), s, a);
  } else {
    smem_opt_in(decode_attn_kernel<D, false>, decode_smem<D>());
    pdl_launch(decode_attn_kernel<D, false>, grid, 128, decode_smem<D>(), s, a);
  }
  if (a.num_splits > 1) pdl_launch(decode_combine_kernel<D>, dim3(a.num_kv_heads * a.group, B), D, 0, s, a);
}

void paged_decode_attn(const DecodeArgs& a, int B, cudaStream_t s) {
  if (B == 0) return;
  int sub_rows = 0;
  if (a.group <= 16 && 64 % a.group == 0 && a.split_len % kKT == 0 && use_tma_decode(a, &sub_rows)) {
    if (a.head_dim == 128) launch_decode_tma<128>(a, B, sub_rows, s);
    else launch_decode_tma<64>(a, B, sub_rows, s);
    check_launch("paged_decode_attn (tma)");
    return;
  }
  if (a.group > 16 || 64 % a.group) throw std::runtime_error("decode attention: GQA group must divide 64 and be <= 16");
  if (a.split_len % kKT) throw std::runtime_error("decode attention: split_len % 64");
  if (a.kv_int8 == 1 && (!a.k_scale || !a.v_scale)) throw std::runtime_error("decode attention: int8 KV needs scales");
  if (a.kv_int8 == 2 && (!a.ch.dscale || !a.ch.out_idx || !a.ch.n_out || !a.ch.side_k || !a.ch.side_v))
    throw std::runtime_error("decode attention: int8 channel mode needs its scales and side pool");
  dim3 grid(a.num_splits, a.num_kv_heads, B);
  if (a.head_dim == 128) {
    launch_decode_split<128>(a, B, grid, s);
  } else if (a.head_dim == 64) {
    launch_decode_split<64>(a, B, grid, s);
  } else {
    throw std::runtime_error("decode attention: head_dim must be 64 or 128");
  }
  check_launch("paged_decode_attn");
}

// ========================================================= int8 -> bf16 stage
// One CTA per (block of a sequence, k|v plane, kv head).  A thread owns one
// 16-value column chunk (256 threads step whole rows), so its read scales
// (channel mode) and outlier slots are loaded once.
template <int D, bool CHAN>
__global__ void __launch_bounds__(256) kv_int8_stage_kernel(const KvStageArgs a) {
  pdl_enter();
  constexpr int CPR = D / 16;  // 16-value chunks per row
  static_assert(256 % CPR == 0, "thread / chunk mapping");
  const int j = blockIdx.x, b = blockIdx.y;
  const int kv = blockIdx.z / a.num_kv_heads, h = blockIdx.z % a.num_kv_heads;
  const int bs = a.block_size;
  const int L = a.seq_lens[b];
  if ((int64_t)j * bs < L) {
    const int valid = min(bs, L - j * bs);
    const int blk = a.block_tables[(size_t)b * a.max_blocks + j];
    const int8_t* src = static_cast<const int8_t*>(kv ? a.v_cache : a.k_cache) + (int64_t)blk * a.block_stride +
                        (int64_t)h * bs * D;
    bf16* dst = static_cast<bf16*>(a.stage) +
                (((size_t)b * a.max_blocks + j) * 2 * a.num_kv_heads + (size_t)kv * a.num_kv_heads + h) * bs * D;
    const int c = threadIdx.x % CPR;
    float ds[16];
    int od[kKvNoutMax];
    const float* tsc = nullptr;
    const bf16* side = nullptr;
    if constexpr (CHAN) {
      const float* row = a.ch.dscale + ((size_t)kv * a.num_kv_heads + h) * D + c * 16;
#pragma unroll
      for (int e = 0; e < 16; ++e) ds[e] = row[e];
      const int n_out = a.ch.n_out[h];
#pragma unroll
      for (int i = 0; i < kKvNoutMax; ++i) od[i] = i < n_out ? a.ch.out_idx[h * kKvNoutMax + i] - c * 16 : -1;
      side = static_cast<const bf16*>(kv ? a.ch.side_v : a.ch.side_k) + (int64_t)blk * a.ch.side_block_stride +
             (int64_t)h * bs * kKvNoutMax;
    } else {
      tsc = (kv ? a.v_scale : a.k_scale) + (int64_t)blk * (a.block_stride / D) + (int64_t)h * bs;
    }
    for (int tok = threadIdx.x / CPR; tok < bs; tok += 256 / CPR) {
      uint4 w0 = make_uint4(0, 0, 0, 0), w1 = make_uint4(0, 0, 0, 0);
      if (tok < valid) {
        const uint4 raw = *reinterpret_cast<const uint4*>(src + (int64_t)tok * D + c * 16);
        const uint32_t rw[4] = {raw.x, raw.y, raw.z, raw.w};
        float qv[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) qv[e] = (float)(int8_t)((rw[e >> 2] >> (8 * (e & 3))) & 0xff);
        float f[16];
        if constexpr (CHAN) {
#pragma unroll
          for (int e = 0; e < 16; ++e) f[e] = qv[e] * ds[e];
          float sd[kKvNoutMax];  // this token's exact outlier values (replacing a zero payload)
#pragma unroll
          for (int i = 0; i < kKvNoutMax; ++i)
            sd[i] = od[i] >= 0 && od[i] < 16 ? __bfloat162float(side[(int64_t)tok * kKvNoutMax + i]) : 0.f;
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            float x = f[e];
#pragma unroll
            for (int i = 0; i < kKvNoutMax; ++i) x = od[i] == e ? sd[i] : x;
            f[e] = x;
          }
        } else {
          const float sc = tsc[tok];
#pragma unroll
          for (int e = 0; e < 16; ++e) f[e] = qv[e] * sc;
        }
        w0 = make_uint4(pack_bf16(f[0], f[1]), pack_bf16(f[2], f[3]), pack_bf16(f[4], f[5]), pack_bf16(f[6], f[7]));
        w1 = make_uint4(pack_bf16(f[8], f[9]), pack_bf16(f[10], f[11]), pack_bf16(f[12], f[13]),
                        pack_bf16(f[14], f[15]));
      }
      uint4* o = reinterpret_cast<uint4*>(dst + (int64_t)tok * D + c * 16);
      o[0] = w0;
      o[1] = w1;
    }
  }
  pdl_trigger();
}

void kv_int8_stage(const KvStageArgs& a, cudaStream_t s) {
  if (a.batch == 0 || a.max_blocks == 0) return;
  if (a.kv_int8 == 1 && (!a.k_scale || !a.v_scale)) throw std::runtime_error("int8 stage: per-token mode needs scales");
  if (a.kv_int8 == 2 && (!a.ch.dscale || !a.ch.out_idx || !a.ch.n_out || !a.ch.side_k || !a.ch.side_v))
    throw std::runtime_error("int8 stage: channel mode needs its scales and side pool");
  if (a.kv_int8 != 1 && a.kv_int8 != 2) throw std::runtime_error("int8 stage: the pool is not int8");
  if (a.block_stride % 16 || (reinterpret_cast<uintptr_t>(a.k_cache) & 15) || (reinterpret_cast<uintptr_t>(a.v_cache) & 15) ||
      (reinterpret_cast<uintptr_t>(a.stage) & 15))
    throw std::runtime_error("int8 stage: pool and stage must be 16-byte aligned");
  dim3 grid(a.max_blocks, a.batch, 2 * a.num_kv_heads);
  const bool chan = a.kv_int8 == 2;
  if (a.head_dim == 128) {
    if (chan) pdl_launch(kv_int8_stage_kernel<128, true>, grid, 256, 0, s, a);
    else pdl_launch(kv_int8_stage_kernel<128, false>, grid, 256, 0, s, a);
  } else if (a.head_dim == 64) {
    if (chan) pdl_launch(kv_int8_stage_kernel<64, true>, grid, 256, 0, s, a);
    else pdl_launch(kv_int8_stage_kernel<64, false>, grid, 256, 0, s, a);
  } else {
    throw std::runtime_error("int8 stage: head_dim must be 64 or 128");
  }
  check_launch("kv_int8_stage");
}

void paged_prefill_attn(const PrefillArgs& a, int B, int max_q_len, cudaStream_t s) {
  if (B == 0 || max_q_len == 0) return;
  if (a.group > 16 || 64 % a.group) throw std::runtime_error("prefill attention: GQA group must divide 64");
  if (a.kv_int8 == 1 && (!a.k_scale || !a.v_scale)) throw std::runtime_error("prefill attention: int8 KV needs scales");
  if (a.kv_int8 == 2 && (!a.ch.dscale || !a.ch.out_idx || !a.ch.n_out || !a.ch.side_k || !a.ch.side_v))
    throw std::runtime_error("prefill attention: int8 channel mode needs its scales and side pool");
  int sub_rows = 0;
  if (fmha_prefill_supported(a, &sub_rows)) {
    fmha_prefill(a, B, max_q_len, sub_rows, s);
    return;
  }
  const int QPB = 64 / a.group;
  dim3 grid((max_q_len + QPB - 1) / QPB, a.num_kv_heads, B);
  if (a.head_dim == 128) {
    smem_opt_in(prefill_attn_kernel<128>, prefill_smem<128>());
    pdl_launch(prefill_attn_kernel<128>, grid, 128, prefill_smem<128>(), s, a);
  } else if (a.head_dim == 64) {
    smem_opt_in(prefill_attn_kernel<64>, prefill_smem<64>());
    pdl_launch(prefill_attn_kernel<64>, grid, 128, prefill_smem<64>(), s, a);
  } else {
    throw std::runtime_error("prefill attention: head_dim must be 64 or 128");
  }
  check_launch("paged_prefill_attn");
}

}  // namespace b200

// ====================================================== no-allocation entry
// Split-KV decode attention whose partial results live in a file-scope device
// array instead of a caller-provided workspace; the contract (limits, set-up,
// races) is in include/noalloc.h.  It goes through paged_decode_attn with the
// pool's block count left at 0, which selects the cp.async split kernel
// (decode_attn_kernel) and its combine: the TMA kernels need the block count for
// their tensor map.  It allocates no device memory.
#include <cstdio>
#include <mutex>
#include "noalloc.h"

namespace {

constexpr int kNoAllocRows = B200MOE_NOALLOC_MAX_ROWS;
constexpr int kNoAllocMaxD = 128;
// [rows][128] part_o, then [rows] part_m, then [rows] part_l.
static __device__ __align__(256) float g_noalloc_scratch[kNoAllocRows * (kNoAllocMaxD + 2)];

constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
float* g_noalloc_ptr[kMaxDevices] = {};

int noalloc_fail(char* err, int err_len, int code, const char* msg) {
  if (err != nullptr && err_len > 0) std::snprintf(err, (size_t)err_len, "%s", msg);
  return code;
}

// Address of this device's scratch array, resolved once per device (with it current).
int noalloc_scratch(float** out, char* err, int err_len) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return noalloc_fail(err, err_len, 3, cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return noalloc_fail(err, err_len, 3, "device ordinal out of range");
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (g_noalloc_ptr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) {
      char msg[256];
      std::snprintf(msg, sizeof(msg), "cudaGetSymbolAddress(scratch) failed: %s", cudaGetErrorString(e));
      return noalloc_fail(err, err_len, 3, msg);
    }
    g_noalloc_ptr[dev] = static_cast<float*>(p);
  }
  *out = g_noalloc_ptr[dev];
  return 0;
}

}  // namespace

extern "C" int b200moe_decode_attn_noalloc_max_rows(void) { return kNoAllocRows; }

extern "C" int b200moe_decode_attn_noalloc(const void* q, const void* k_cache, const void* v_cache,
                                           const float* k_scale, const float* v_scale, int kv_int8,
                                           const int* block_tables, const int* seq_lens, int batch,
                                           int max_blocks, int block_size, long long block_stride,
                                           int num_q_heads, int num_kv_heads, int head_dim, float scale,
                                           int num_splits, int split_len, void* out, void* stream, char* err,
                                           int err_len) {
  if (batch < 0 || num_splits < 1 || num_kv_heads < 1 || num_q_heads < 1 || num_q_heads % num_kv_heads != 0)
    return noalloc_fail(err, err_len, 1, "decode_attn_noalloc: bad batch / splits / head counts");
  const int group = num_q_heads / num_kv_heads;
  if (group > 16 || 64 % group != 0)
    return noalloc_fail(err, err_len, 1, "decode_attn_noalloc: q_heads / kv_heads must divide 64 and be <= 16");
  if (block_size < 1 || max_blocks < 1 || block_stride <= 0)
    return noalloc_fail(err, err_len, 1, "decode_attn_noalloc: block_size, max_blocks and block_stride must be > 0");
  if (split_len < 1 || split_len % 64 != 0)
    return noalloc_fail(err, err_len, 1, "decode_attn_noalloc: split_len must be a positive multiple of 64");
  if (head_dim != 64 && head_dim != kNoAllocMaxD)
    return noalloc_fail(err, err_len, 1, "decode_attn_noalloc: head_dim must be 64 or 128");
  if (kv_int8 && (k_scale == nullptr || v_scale == nullptr))
    return noalloc_fail(err, err_len, 1, "decode_attn_noalloc: int8 KV needs k_scale and v_scale");
  if (batch > 0 && (q == nullptr || k_cache == nullptr || v_cache == nullptr || block_tables == nullptr ||
                    seq_lens == nullptr || out == nullptr))
    return noalloc_fail(err, err_len, 1, "decode_attn_noalloc: null tensor pointer");
  const long long rows = (long long)batch * num_q_heads * num_splits;
  if (num_splits > 1 && rows > kNoAllocRows) {
    char msg[256];
    std::snprintf(msg, sizeof(msg),
                  "decode_attn_noalloc: batch*q_heads*num_splits = %lld exceeds the scratch limit of %d rows",
                  rows, kNoAllocRows);
    return noalloc_fail(err, err_len, 2, msg);
  }
  float* scratch = nullptr;
  const int rc = noalloc_scratch(&scratch, err, err_len);
  if (rc != 0) return rc;
  b200::DecodeArgs a{};
  a.q = q;
  a.k_cache = k_cache;
  a.v_cache = v_cache;
  a.k_scale = k_scale;
  a.v_scale = v_scale;
  a.kv_int8 = kv_int8;
  a.block_tables = block_tables;
  a.seq_lens = seq_lens;
  a.max_blocks = max_blocks;
  a.block_size = block_size;
  a.block_stride = block_stride;
  a.num_kv_heads = num_kv_heads;
  a.group = group;
  a.head_dim = head_dim;
  a.scale = scale;
  a.num_splits = num_splits;
  a.split_len = split_len;
  a.part_o = scratch;
  a.part_m = scratch + (size_t)kNoAllocRows * kNoAllocMaxD;
  a.part_l = a.part_m + kNoAllocRows;
  a.out = out;
  a.num_blocks = 0;  // no pool size: the cp.async kernel, not the TMA one
  try {
    b200::paged_decode_attn(a, batch, static_cast<cudaStream_t>(stream));
  } catch (const std::exception& ex) {
    const bool launch = std::string(ex.what()).find("paged_decode_attn:") == 0;
    return noalloc_fail(err, err_len, launch ? 3 : 1, ex.what());
  }
  return 0;
}

// Causal prefill attention on the 5th-generation tensor cores (sm_100a):
// paged bf16 KV, head_dim 128, grouped-query heads packed into the M dimension.
//
// One CTA owns 128 packed rows -- 128 / G query positions x the G query heads
// that share one KV head -- and walks the keys up to its causal bound in tiles
// of 128:
//
//   warp 0      TMA producer: K and V tiles (two 64-column halves, 128-byte
//               swizzle) from the paged pool through a 4-D tensor map
//               {D, block_size, 2*kv_heads, blocks}; blocks past the sequence
//               read an out-of-range block coordinate and come back zero-filled.
//   warp 1      one thread issues tcgen05.mma: S_j = Q K_j^T into one of two TMEM
//               S buffers, O += P_j V_j into a TMEM O accumulator (V is read
//               MN-major straight from its [key][d] tile).  Issue order
//               S0 S1 PV0 S2 PV1 ... keeps the next S product running while the
//               softmax works on the current one.
//   warps 2..5  softmax: one thread per row (TMEM lane = row), so the row max and
//               sum need no shuffles.  P is rounded to bf16 and written to shared
//               memory in the UMMA K-major layout.  The O rescale is lazy: the
//               running max moves only when a row's max grows by more than 2^8,
//               and only then is the O row read from TMEM, scaled and written back.
//
// Every wait is bounded (sm100.cuh); on expiry the roles unwind, drain their
// in-flight copies and MMAs, free TMEM and return with a status code.
//
// Reference behaviour: nanovllm/layers/attention.py:179-213 (causal prefill over
// the paged cache, GQA).  Numerics: fp32 scores and accumulators, bf16 P, as in
// the mma.sync kernel of attention.cu that remains for other head sizes and int8 KV.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdint>
#include <cstdlib>
#include <mutex>
#include <stdexcept>
#include <string>
#include <vector>

#include "attention.h"
#include "sm100.cuh"
#include "pdl.cuh"

namespace b200 {
namespace {

using bf16 = __nv_bfloat16;

constexpr int kD = 128;                        // head dim
constexpr int kRows = 128;                     // packed (query, head) rows per CTA
constexpr int kKeys = 128;                     // keys per tile
constexpr int kSlots = 4;                      // K / V tiles in flight
constexpr int kTile = kKeys * kD * 2;          // 32 KB: one K (or V, Q, P) tile
constexpr int kHalf = kTile / 2;               // [128 rows][64 cols] bf16 half, 16 KB
constexpr float kLazyLog2 = 8.f;
constexpr int kThreads = 192;
constexpr uint32_t kTmemCols = 512;            // S0 | S1 | O (| unused)

struct Layout {
  static constexpr int Q = 0;                          // two Q buffers (items alternate)
  static constexpr int P = Q + 2 * kTile;
  static constexpr int RING = P + kTile;
  static constexpr int BARS = RING + kSlots * kTile;
  // kv full/empty, s_full[2], p_full, p_empty, q_full[2], q_empty[2], fin
  static constexpr int NBARS = 2 * kSlots + 2 + 2 + 4 + 1;
  static constexpr int SMEM = BARS + NBARS * 8 + 16 + 1024;
};
static_assert(Layout::SMEM <= 232448, "shared memory budget");

// 16-byte chunk u (0..7) of row r in a [rows][64] bf16 half with 128-byte swizzle
__device__ __forceinline__ uint32_t sw_off(int r, int u) { return r * 128 + ((u ^ (r & 7)) << 4); }

__device__ __forceinline__ void tma_load_4d(uint32_t dst, const CUtensorMap* map, uint64_t* bar, int x, int y,
                                            int z, int w) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];"
      ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z), "r"(w)
      : "memory");
}

__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, uint64_t* bar, int x, int y,
                                            int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];"
      ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}

// Shared-memory descriptor of an MN-major operand in 128-byte swizzle: 64
// contiguous elements per 128-byte row, rows = K; `lbo` = bytes between 64-wide
// MN chunks, SBO = 1024 bytes between groups of 8 K rows.
__device__ __forceinline__ uint64_t sdesc_sw128_mn(uint32_t addr, uint32_t lbo) {
  uint64_t d = 0;
  d |= uint64_t((addr >> 4) & 0x3FFFu);
  d |= uint64_t((lbo >> 4) & 0x3FFFu) << 16;
  d |= uint64_t(1024 >> 4) << 32;
  d |= uint64_t(1) << 46;
  d |= uint64_t(2) << 61;
  return d;
}

// 32 lanes x 32 columns per thread
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* v) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float* v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};"
      ::"r"(taddr), "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
        "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
        "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
        "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
        "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
        "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])),
        "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])),
        "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
        "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])),
        "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])),
        "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
      : "memory");
}

__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// One work item = (kv head h, sequence b, query tile qt): 128 packed rows.
struct FmItem {
  int h, b, qt, q0, q_len, pos0, ntiles;
};

__device__ __forceinline__ bool fm_item(const PrefillArgs& a, int qtiles, int w, FmItem& it) {
  // heaviest query tiles (largest causal extent) first, then sequence, then kv head
  const int B = a.batch;
  it.h = w % a.num_kv_heads;
  w /= a.num_kv_heads;
  it.b = w % B;
  it.qt = qtiles - 1 - w / B;
  const int QPB = kRows / a.group;
  it.q0 = a.cu_seqlens_q[it.b];
  it.q_len = a.cu_seqlens_q[it.b + 1] - it.q0;
  if (it.qt * QPB >= it.q_len) return false;
  const int kv_len = a.seq_lens[it.b];
  it.pos0 = kv_len - it.q_len;
  const int last_q = min(it.q_len, (it.qt + 1) * QPB) - 1;
  const int k_end = min(kv_len, it.pos0 + last_q + 1);
  it.ntiles = (k_end + kKeys - 1) / kKeys;
  return true;
}

__global__ void __launch_bounds__(kThreads, 1)
fmha_prefill_kernel(const __grid_constant__ CUtensorMap kv_map, const __grid_constant__ CUtensorMap q_map,
                    const PrefillArgs a, int sub_rows, int oob_block, int qtiles, int n_items) {
  pdl_enter();
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem + Layout::Q;
  uint8_t* sP = smem + Layout::P;
  uint8_t* ring = smem + Layout::RING;
  uint64_t* kv_full = reinterpret_cast<uint64_t*>(smem + Layout::BARS);
  uint64_t* kv_empty = kv_full + kSlots;
  uint64_t* s_full = kv_empty + kSlots;
  uint64_t* p_full = s_full + 2;
  uint64_t* p_empty = p_full + 1;
  uint64_t* q_full = p_empty + 1;     // [2]
  uint64_t* q_empty = q_full + 2;     // [2]
  uint64_t* fin = q_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(fin + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int G = a.group;
  const int nq = a.num_kv_heads * G;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int* status = a.status;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kSlots; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
    }
    mbar_init(&s_full[0], 1);
    mbar_init(&s_full[1], 1);
    mbar_init(p_full, 4);
    mbar_init(p_empty, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
    }
    mbar_init(fin, 1);
    fence_barrier_init();
    *abort_flag = 0;
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tO = tmem + 256;

  if (warp == 0) {
    // ================================================================ TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&kv_map);
      tma_prefetch_desc(&q_map);
      const int nsub = kKeys / sub_rows;
      const int QPB = kRows / G;
      int p = 0, li = 0;  // K/V tiles issued; items begun by this CTA
      bool ok = true;
      for (int w = blockIdx.x; w < n_items && ok; w += gridDim.x) {
        FmItem it;
        if (!fm_item(a, qtiles, w, it)) continue;
        // Q tile: {64 d, G heads, QPB tokens} boxes land as [pos * G + g][64] rows, 128-byte swizzled
        const int qb = li & 1;
        if (!mbar_wait(&q_empty[qb], ((li >> 1) & 1) ^ 1, status, kStatusTimeoutEmpty, abort_flag)) { ok = false; break; }
        mbar_arrive_expect_tx(&q_full[qb], kTile);
#pragma unroll
        for (int hf = 0; hf < 2; ++hf)
          tma_load_3d(smem_u32(sQ + qb * kTile + hf * kHalf), &q_map, &q_full[qb], hf * 64, it.h * G,
                      it.q0 + it.qt * QPB);
        ++li;
        const int* btab = a.block_tables + (size_t)it.b * a.max_blocks;
        const int kv_len = it.pos0 + it.q_len;
        const int k_end = min(kv_len, it.pos0 + min(it.q_len, (it.qt + 1) * QPB));
        for (int e = 0; e < 2 * it.ntiles; ++e, ++p) {
          const int j = e >> 1, slot = p % kSlots;
          const uint32_t ph = (p / kSlots) & 1;
          if (!mbar_wait(&kv_empty[slot], ph ^ 1, status, kStatusTimeoutEmpty, abort_flag)) { ok = false; break; }
          mbar_arrive_expect_tx(&kv_full[slot], kTile);
          const uint32_t dst = smem_u32(ring + slot * kTile);
          const int plane = (e & 1) ? a.num_kv_heads + it.h : it.h;  // V planes follow the K planes
          for (int sub = 0; sub < nsub; ++sub) {
            const int key = j * kKeys + sub * sub_rows;
            const int blk = key >= k_end ? oob_block : btab[key / a.block_size];
            const int y = key % a.block_size;
#pragma unroll
            for (int hf = 0; hf < 2; ++hf)
              tma_load_4d(dst + hf * kHalf + sub * sub_rows * 128, &kv_map, &kv_full[slot], hf * 64, y, plane, blk);
          }
        }
      }
      if (*abort_flag) {
        // a wait gave up: let loads already issued land before the CTA exits
        const uint64_t t0 = globaltimer_ns();
        while (globaltimer_ns() - t0 < 1000000ull) __nanosleep(1000);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ================================================================ MMA issuer
    // One stream of (item, key tile) across the CTA's items: S of tile g + 2 is
    // issued right after PV of tile g, so the next item's first S products run
    // while the softmax finishes the current item.
    if (lane == 0) {
      const uint32_t idesc_s = umma_idesc_bf16(kRows, kKeys);
      const uint32_t idesc_pv = umma_idesc_bf16(kRows, kD) | (1u << 16);  // B (V) is MN-major
      const uint32_t pb = smem_u32(sP);
      struct Cursor {
        int w, li, t, n;  // item index, local item number, tile in item, tiles in item
      };
      auto first = [&](Cursor& c, int w0) {
        FmItem it;
        for (c.w = w0; c.w < n_items; c.w += gridDim.x)
          if (fm_item(a, qtiles, c.w, it)) { c.t = 0; c.n = it.ntiles; return; }
        c.n = 0;
      };
      auto next = [&](Cursor& c) {
        if (++c.t < c.n) return;
        ++c.li;
        first(c, c.w + gridDim.x);
      };
      Cursor cs{0, 0, 0, 0}, cp{0, 0, 0, 0};
      first(cs, blockIdx.x);
      first(cp, blockIdx.x);
      int gs = 0, gp = 0;  // global tile counters of the S and PV streams
      bool ok = true;
      auto issue_s = [&]() -> bool {
        const int qb = cs.li & 1;
        if (cs.t == 0) {
          if (!mbar_wait(&q_full[qb], (cs.li >> 1) & 1, status, kStatusTimeoutFull, abort_flag)) return false;
        }
        const int pk = 2 * gs, slot = pk % kSlots;
        if (!mbar_wait(&kv_full[slot], (pk / kSlots) & 1, status, kStatusTimeoutFull, abort_flag)) return false;
        tc_fence_after();
        const uint32_t qa = smem_u32(sQ + qb * kTile), kb = smem_u32(ring + slot * kTile);
#pragma unroll
        for (int k = 0; k < kD / 16; ++k) {
          const uint32_t off = (k >> 2) * kHalf + (k & 3) * 32;
          umma_f16_ss(tmem + (gs & 1) * kKeys, umma_sdesc_sw128(qa + off), umma_sdesc_sw128(kb + off), idesc_s,
                      k > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[gs & 1]);
        umma_commit(&kv_empty[slot]);
        if (cs.t + 1 == cs.n) umma_commit(&q_empty[qb]);  // the item's Q is no longer read
        ++gs;
        next(cs);
        return true;
      };
      auto issue_pv = [&]() -> bool {
        if (!mbar_wait(p_full, gp & 1, status, kStatusTimeoutConv, abort_flag)) return false;
        const int pk = 2 * gp + 1, slot = pk % kSlots;
        if (!mbar_wait(&kv_full[slot], (pk / kSlots) & 1, status, kStatusTimeoutFull, abort_flag)) return false;
        tc_fence_after();
        const uint32_t vb = smem_u32(ring + slot * kTile);
#pragma unroll
        for (int k = 0; k < kKeys / 16; ++k) {
          const uint64_t adesc = umma_sdesc_sw128(pb + (k >> 2) * kHalf + (k & 3) * 32);
          const uint64_t bdesc = sdesc_sw128_mn(vb + k * 16 * 128, kHalf);
          umma_f16_ss(tO, adesc, bdesc, idesc_pv, (cp.t > 0 || k > 0) ? 1u : 0u);
        }
        umma_commit(p_empty);
        umma_commit(&kv_empty[slot]);
        ++gp;
        next(cp);
        return true;
      };
      for (int i = 0; i < 2 && ok && cs.n > 0; ++i) ok = issue_s();
      while (ok && cp.n > 0) {
        ok = issue_pv();
        if (ok && cs.n > 0) ok = issue_s();
      }
      // every MMA issued so far completes before TMEM is released
      umma_commit(fin);
      mbar_wait(fin, 0, status, kStatusTimeoutAccEmpty, nullptr);
    }
    __syncwarp();
  } else {
    // ================================================================ softmax
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
    const float sl2 = a.scale * 1.4426950408889634f;
    const int QPB = kRows / G;
    int g = 0;  // global tile counter (S / P stream)
    bool ok = true;
    for (int w = blockIdx.x; w < n_items && ok; w += gridDim.x) {
      FmItem it;
      if (!fm_item(a, qtiles, w, it)) continue;
      const int qi = it.qt * QPB + r / G, head = it.h * G + r % G;
      const bool valid = qi < it.q_len;
      const int qpos = valid ? it.pos0 + qi : -1;
      float m_run = -INFINITY, l_run = 0.f;
      for (int j = 0; j < it.ntiles; ++j, ++g) {
        ok = mbar_wait(&s_full[g & 1], (g >> 1) & 1, status, kStatusTimeoutAccFull, abort_flag);
        if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
        tc_fence_after();
        float s[kKeys];
#pragma unroll
        for (int c = 0; c < kKeys / 32; ++c) tmem_ld32(tmem + lane_base + (g & 1) * kKeys + c * 32, s + c * 32);
        tmem_ld_wait();
        const int kbase = j * kKeys;
        if (kbase + kKeys - 1 > qpos) {
#pragma unroll
          for (int c = 0; c < kKeys; ++c)
            if (kbase + c > qpos) s[c] = -INFINITY;
        }
        float mx = -INFINITY;
#pragma unroll
        for (int c = 0; c < kKeys; ++c) mx = fmaxf(mx, s[c]);
        mx *= sl2;
        const bool grow = mx > m_run + kLazyLog2;
        // PV of the previous tile (of any item) must be done before P is rewritten,
        // and before O is rescaled (same item)
        if (g > 0) {
          ok = mbar_wait(p_empty, (g - 1) & 1, status, kStatusTimeoutAccEmpty, abort_flag);
          if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
          tc_fence_after();
        }
        if (__any_sync(0xffffffffu, grow)) {
          float alpha = 1.f;
          if (grow) {
            alpha = m_run == -INFINITY ? 1.f : exp2f(m_run - mx);
            m_run = mx;
            l_run *= alpha;
          }
          if (j > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll 1
            for (int c = 0; c < kD / 32; ++c) {
              float o[32];
              tmem_ld32(tO + lane_base + c * 32, o);
              tmem_ld_wait();
#pragma unroll
              for (int i = 0; i < 32; ++i) o[i] *= alpha;
              tmem_st32(tO + lane_base + c * 32, o);
            }
            tmem_st_wait();
          }
        }
        const float mu = m_run == -INFINITY ? 0.f : m_run;
        float sum = 0.f;
#pragma unroll
        for (int cc = 0; cc < kKeys / 8; ++cc) {  // 8 keys = one 16-byte chunk of P
          uint32_t wv[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float p0 = exp2f(fmaf(s[cc * 8 + 2 * e], sl2, -mu));
            const float p1 = exp2f(fmaf(s[cc * 8 + 2 * e + 1], sl2, -mu));
            sum += p0 + p1;
            wv[e] = pack2(p0, p1);
          }
          *reinterpret_cast<uint4*>(sP + (cc >> 3) * kHalf + sw_off(r, cc & 7)) =
              make_uint4(wv[0], wv[1], wv[2], wv[3]);
        }
        l_run += sum;
        fence_proxy_async_smem();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(p_full);
      }
      if (!ok) break;
      // ---- item epilogue: O / l once the item's last PV has landed
      ok = mbar_wait(p_empty, (g - 1) & 1, status, kStatusTimeoutAccEmpty, abort_flag);
      if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
      tc_fence_after();
      const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
      uint4* dst = reinterpret_cast<uint4*>(static_cast<bf16*>(a.out) +
                                            ((size_t)(it.q0 + (valid ? qi : 0)) * nq + head) * kD);
#pragma unroll 1
      for (int c = 0; c < kD / 32; ++c) {
        float o[32];
        tmem_ld32(tO + lane_base + c * 32, o);
        tmem_ld_wait();
        if (valid) {
#pragma unroll
          for (int v = 0; v < 4; ++v)
            dst[c * 4 + v] = make_uint4(pack2(o[8 * v] * inv, o[8 * v + 1] * inv),
                                        pack2(o[8 * v + 2] * inv, o[8 * v + 3] * inv),
                                        pack2(o[8 * v + 4] * inv, o[8 * v + 5] * inv),
                                        pack2(o[8 * v + 6] * inv, o[8 * v + 7] * inv));
        }
      }
      tc_fence_before();  // O reads complete before the next item's first PV overwrites it
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
  pdl_trigger();
}

// ------------------------------------------------------------------ host side
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
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

struct MapKey {
  const void* base;
  int dev, bs, kvh, nblocks, rows;
  int64_t block_stride;
  bool operator==(const MapKey& o) const {
    return base == o.base && dev == o.dev && bs == o.bs && kvh == o.kvh && nblocks == o.nblocks &&
           rows == o.rows && block_stride == o.block_stride;
  }
};

// Returned by value: another thread's call may clear the cache.
CUtensorMap kv_map(const PrefillArgs& a, int sub_rows) {
  static std::mutex mu;
  static std::vector<std::pair<MapKey, CUtensorMap>> cache;  // one entry per layer of a pool
  const MapKey key{a.k_cache, current_device(), a.block_size, a.num_kv_heads, a.num_blocks, sub_rows,
                   a.block_stride};
  std::lock_guard<std::mutex> lock(mu);
  for (auto& e : cache)
    if (e.first == key) return e.second;
  CUtensorMap map;
  const cuuint64_t dims[4] = {(cuuint64_t)kD, (cuuint64_t)a.block_size, (cuuint64_t)(2 * a.num_kv_heads),
                              (cuuint64_t)a.num_blocks};
  const cuuint64_t strides[3] = {(cuuint64_t)kD * 2, (cuuint64_t)a.block_size * kD * 2,
                                 (cuuint64_t)a.block_stride * 2};
  const cuuint32_t box[4] = {64, (cuuint32_t)sub_rows, 1, 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = encode_fn()(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(a.k_cache), dims, strides,
                           box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw std::runtime_error("prefill kv tensor map: encode failed " + std::to_string((int)r));
  if (cache.size() > 512) cache.clear();
  cache.emplace_back(key, map);
  return cache.back().second;
}

}  // namespace

// Shapes the tensor-core kernel takes: bf16 pool with V planes after the K planes
// of each block, head_dim 128, a GQA group dividing 128, 16-byte aligned planes,
// and 128-key tiles that either sit inside one block or cover whole blocks.
bool fmha_prefill_supported(const PrefillArgs& a, int* sub_rows) {
  const char* e = std::getenv("B200MOE_PREFILL_TC");
  if (e != nullptr && std::string(e) == "0") return false;
  if (a.kv_int8 || a.head_dim != kD || a.num_blocks <= 0 || a.group <= 0 || kRows % a.group) return false;
  const bf16* k = static_cast<const bf16*>(a.k_cache);
  if (static_cast<const bf16*>(a.v_cache) != k + (int64_t)a.num_kv_heads * a.block_size * kD) return false;
  if ((reinterpret_cast<uintptr_t>(a.k_cache) & 15) || (a.block_stride * 2) % 16) return false;
  if (a.block_size % kKeys == 0) *sub_rows = kKeys;
  else if (kKeys % a.block_size == 0 && a.block_size % 8 == 0) *sub_rows = a.block_size;
  else return false;
  return true;
}

// Q as a 3-D tensor {head_dim, q heads, rows}: a box {64, G, 128 / G} is one half of
// a 128-row packed tile (row = position * G + group head).
static CUtensorMap q_map(const PrefillArgs& a) {
  struct Entry { const void* base; int rows, nq, G; CUtensorMap map; };
  static std::mutex mu;
  static std::vector<Entry> cache;
  std::lock_guard<std::mutex> lock(mu);
  const int nq = a.num_kv_heads * a.group;
  for (auto& e : cache)
    if (e.base == a.q && e.rows == a.q_rows && e.nq == nq && e.G == a.group) return e.map;
  CUtensorMap map;
  const cuuint64_t dims[3] = {(cuuint64_t)kD, (cuuint64_t)nq, (cuuint64_t)a.q_rows};
  const cuuint64_t strides[2] = {(cuuint64_t)kD * 2, (cuuint64_t)nq * kD * 2};
  const cuuint32_t box[3] = {64, (cuuint32_t)a.group, (cuuint32_t)(kRows / a.group)};
  const cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = encode_fn()(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(a.q), dims, strides, box,
                           estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw std::runtime_error("prefill q tensor map: encode failed " + std::to_string((int)r));
  if (cache.size() >= 64) cache.erase(cache.begin());
  cache.push_back({a.q, a.q_rows, nq, a.group, map});
  return map;
}

static int num_sms_fmha() { return device_sm_count(); }

void fmha_prefill(const PrefillArgs& a_in, int B, int max_q_len, int sub_rows, cudaStream_t s) {
  PrefillArgs a = a_in;
  a.batch = B;
  if (a.q_rows <= 0 || (reinterpret_cast<uintptr_t>(a.q) & 15))
    throw std::runtime_error("prefill attention: q rows / alignment");
  const CUtensorMap kvm = kv_map(a, sub_rows);
  const CUtensorMap qm = q_map(a);
  smem_opt_in(fmha_prefill_kernel, Layout::SMEM);
  const int QPB = kRows / a.group;
  const int qtiles = (max_q_len + QPB - 1) / QPB;
  const int64_t n_items = (int64_t)a.num_kv_heads * B * qtiles;
  if (n_items > (1 << 30)) throw std::runtime_error("prefill attention: too many query tiles for one launch");
  const int grid = (int)std::min<int64_t>(n_items, num_sms_fmha());
  pdl_launch(fmha_prefill_kernel, grid, kThreads, Layout::SMEM, s, kvm, qm, a, sub_rows, a.num_blocks, qtiles, (int)n_items);
  cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) throw std::runtime_error(std::string("fmha_prefill launch: ") + cudaGetErrorString(err));
}

}  // namespace b200

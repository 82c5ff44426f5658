// Grouped weight x activation GEMM on tcgen05 (sm_100a).
//
//   D_g^T[m, n] = sum_k  W_g[m, k] * X[row_off[g] + n, k]      for every group g
//
// W (the "A" operand, M = output features) is either a 128x128 block-scaled
// e4m3 weight (the checkpoint format: w = q * scale_inv[m/128, k/128]) or a
// plain bf16 weight.  X (the "B" operand, N = tokens) is bf16.  One CTA per SM
// runs a persistent loop over (group, n-tile, m-tile) work items computed on
// the device from per-group token counts, so the launch needs no host sync and
// is CUDA-graph safe.  Roles (fp8: 704 threads, bf16: 192):
//
//   warp 0      TMA producer: fp8 (or bf16) weight tile + bf16 activation tile
//               per stage into a deep ring that holds only the loaded bytes
//   warp 1      TMEM allocator + single-thread tcgen05.mma issuer
//   warps 2-17  (fp8 only) 16 independent dequantiser warps: e4m3 * scale ->
//               bf16 into a separate ring in the 128B-swizzled UMMA layout
//               (exactly bf16(float(q) * scale), the reference's load-time
//               dequant, done per tile in shared memory).  Each warp converts
//               one 16-byte chunk per lane of every weight tile and arrives on
//               the stage barriers itself: no CTA-level barrier on the path,
//               and 4 warps per scheduler hide the conversion latency.
//               Keeping the bf16 copies out of the load ring is what lets
//               several loads per SM stay in flight.
//   last 4      epilogue: tcgen05.ld of the double-buffered TMEM accumulator,
//               fused op, global store; per-tile row metadata (scatter slots and
//               routing weights) is staged in shared memory once per tile
//
// Epilogues: bf16 store, fp32 store (router / LM-head logits), SiLU(gate)*up of
// a gate/up tile pair (two MMAs into adjacent TMEM columns), and the MoE "down"
// epilogue that scales by the routing weight and scatters each row to its
// (token, k) slot so the combine is a fixed-order sum.
//
// Reference ops replaced: torch._grouped_mm / torch.bmm expert GEMMs and
// F.linear (nanovllm/models/qwen3_moe.py:216-340, nanovllm/layers/linear.py:73),
// fused_silu_and_mul (nanovllm/kernels/moe_fusion.py:19-28) and the weighted
// slot scatter (qwen3_moe.py:270-279).
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <algorithm>
#include <cstdint>
#include <stdexcept>
#include <string>

#include "sm100.cuh"
#include "pdl.cuh"
#include "ep_sync.cuh"
#include "gemm_tc.h"

namespace b200 {

constexpr int kMaxGroups = 512;
constexpr int kBK = 64;            // K elements per pipeline stage (128 B of bf16)
constexpr int kSmemBudget = 225 * 1024;

template <int BN, bool PAIR, bool AFP8>
struct GemmCfg {
  static constexpr int NA = PAIR ? 2 : 1;
  static constexpr int CONV_WARPS = AFP8 ? 16 : 0;    // one 16-byte chunk per lane of a 128x64 e4m3 tile
  static constexpr int EPI_WARP0 = 2 + CONV_WARPS;
  // token tiles of 64+ (prefill): eight epilogue warps (two per TMEM lane quarter)
  // that transpose each 16-column chunk through shared memory and write 16-byte
  // pieces of output rows; decode-size tiles keep four warps and direct stores,
  // whose shared memory goes to load stages instead
  static constexpr bool EPI_STAGED = BN >= 64;
  static constexpr int EPI_WARPS = EPI_STAGED ? 8 : 4;
  static constexpr int THREADS = (EPI_WARP0 + EPI_WARPS) * 32;
  static constexpr int EPI_STAGE = EPI_STAGED ? EPI_WARPS * 16 * 32 * 4 : 0;  // per warp: 16 cols x 32 rows x 4 B
  // Single-tile TMEM-ring GEMMs (decode down / QKV / O) take 128 K per stage: the
  // producer and MMA threads pay their per-stage cost (barrier probes, commits,
  // descriptors) once per 8 MMAs instead of 4, which bounded them at decode size.
  // (The gate/up pair already issues 8 MMAs per 64-wide stage; 128-wide stages
  // leave it 3 TMEM slots and measured no faster: 97 vs 99 us at 256 tokens.)
  static constexpr bool WIDE_K = AFP8 && !PAIR && BN <= 128;
  static constexpr int KS = WIDE_K ? 128 : kBK;       // K elements per pipeline stage
  static constexpr int KSUB = KS / kBK;               // 64-wide sub-blocks per stage
  static constexpr int A16_BYTES = 128 * kBK * 2;     // 16 KB bf16 tile
  static constexpr int A8_BYTES = 128 * KS;           // e4m3 tile of one stage (8 or 16 KB)
  static constexpr int B_BYTES = BN * KS * 2;         // KSUB 128-byte-swizzled [BN][64] atoms
  // load ring: what TMA writes (fp8 weights or, in bf16 mode, the UMMA-ready A tile)
  static constexpr int ALOAD_BYTES = AFP8 ? A8_BYTES : A16_BYTES;
  static constexpr int STAGE_BYTES = NA * ALOAD_BYTES + B_BYTES;
  static constexpr int ACC_COLS = NA * BN;
  // Decode-size tiles (BN <= 64, or 128 without the gate/up pair) keep the dequantised bf16 A tiles in TMEM
  // (tcgen05.st by the dequantisers, MMA with A from TMEM): TMEM left over by the
  // two accumulators holds the bf16 ring, and the shared memory it used to take
  // goes to e4m3 load stages -- these GEMMs are bound by the bytes in flight per SM.
  static constexpr bool A_TMEM = AFP8 && (PAIR ? BN <= 64 : BN <= 128);
  static constexpr int SLOT_COLS = NA * KS / 2;       // TMEM columns of one bf16 ring slot
  static constexpr int TSLOTS_RAW = A_TMEM ? (512 - 2 * ACC_COLS) / SLOT_COLS : 0;
  // bf16 slots: TMEM ring (up to 8) for decode-size tiles, else a shared-memory ring
  // of 2 for BN >= 128 (MMA-bound: the shared memory goes to deeper load stages for
  // the large B tiles)
  static constexpr int CONV_SLOTS = !AFP8 ? 0 : A_TMEM ? (TSLOTS_RAW > 8 ? 8 : TSLOTS_RAW)
                                    : BN >= 128 ? 2 : PAIR ? 3 : 4;
  static constexpr int CONV_BYTES = A_TMEM ? 0 : CONV_SLOTS * NA * A16_BYTES;
  static constexpr int EXTRA = 4096 + 2 * (kMaxGroups + 1) * 4 + 2 * 256 * 8 + 128 * 4;
  // TMEM-ring tiles split the load ring: e4m3 stages (freed by the dequantisers as
  // soon as they have read them) and a separate, deeper ring of activation tiles
  // (freed by the MMA), so weight bytes never wait for the MMA to release a slot
  static constexpr int SB = !A_TMEM ? 0 : PAIR ? (BN <= 32 ? 12 : 8) : BN <= 32 ? 8 : BN == 64 ? 6 : 3;
  static constexpr int A_STAGE_BYTES = NA * ALOAD_BYTES;
  static constexpr int STAGES_RAW = A_TMEM
      ? (kSmemBudget - EXTRA - 1024 - EPI_STAGE - SB * B_BYTES) / A_STAGE_BYTES
      : (kSmemBudget - EXTRA - 1024 - CONV_BYTES - EPI_STAGE) / STAGE_BYTES;
  static constexpr int MAX_STAGES = A_TMEM ? 16 : 12;
  static constexpr int STAGES = STAGES_RAW > MAX_STAGES ? MAX_STAGES : STAGES_RAW;
  static constexpr int RING_BYTES = A_TMEM ? STAGES * A_STAGE_BYTES + SB * B_BYTES : STAGES * STAGE_BYTES;
  static constexpr int SMEM = RING_BYTES + CONV_BYTES + EPI_STAGE + EXTRA + 1024;
  // dequantiser warp groups taking stages round robin: never more groups than
  // load stages or bf16 slots (a group waits on its own stage and slot)
  static constexpr int DEQ_GROUPS = !AFP8 ? 1 : (STAGES >= 4 && CONV_SLOTS >= 4) ? 4 : 2;
  static_assert(!AFP8 || (CONV_WARPS % DEQ_GROUPS == 0 && DEQ_GROUPS <= CONV_SLOTS && DEQ_GROUPS <= STAGES),
                "dequant groups must fit the load ring and the bf16 ring");
  static_assert(!A_TMEM || CONV_SLOTS >= 2, "TMEM bf16 ring needs two slots");
  static constexpr int TMEM_COLS_RAW = A_TMEM ? 512 : 2 * ACC_COLS;
  static constexpr int TMEM_COLS = TMEM_COLS_RAW <= 32 ? 32 : TMEM_COLS_RAW <= 64 ? 64
                                   : TMEM_COLS_RAW <= 128 ? 128 : TMEM_COLS_RAW <= 256 ? 256 : 512;
  static constexpr int TSLOT_COL0 = 2 * ACC_COLS;       // first TMEM column of the bf16 ring
  static_assert(STAGES >= 2, "not enough shared memory for two stages");
  static_assert(STAGES <= 16 && SB <= 16, "barrier arrays hold 16 stages");
  static_assert(TMEM_COLS_RAW <= 512, "accumulators exceed TMEM");
  static_assert(BN % 16 == 0 && BN >= 16 && BN <= 256, "UMMA N must be a multiple of 16 in [16,256]");
  static constexpr uint32_t TX_BYTES = NA * ALOAD_BYTES + B_BYTES;
};

struct TileCoord {
  int g, j, i;   // group, token tile, weight tile
  int ks0, ks1;  // K stages [ks0, ks1) of this work item (split-K)
  int sp;        // split index
};

// tile_prefix[g] = first work item of group g (exclusive prefix, ngroups+1
// entries); the owner of item t is the last g with tile_prefix[g] <= t.  Items
// of a group are ordered (token tile, weight tile, split).
__device__ __forceinline__ TileCoord decode_tile(int t, const int* tile_prefix, int ngroups, int m_tiles,
                                                 int k_stages, int k_splits) {
  int lo = 0, hi = ngroups;
  while (hi - lo > 1) {
    int mid = (lo + hi) >> 1;
    if (tile_prefix[mid] <= t) lo = mid; else hi = mid;
  }
  int local = t - tile_prefix[lo];
  TileCoord c;
  c.g = lo;
  c.sp = local % k_splits;
  local /= k_splits;
  c.j = local / m_tiles;
  c.i = local % m_tiles;
  const int per = (k_stages + k_splits - 1) / k_splits;
  c.ks0 = c.sp * per;
  c.ks1 = min(k_stages, c.ks0 + per);
  return c;
}

// Pipeline trace (debug/profiling) of CTA 0: trace[1 + role * cap + index] =
// %globaltimer for role 0 TMA issued, 1 dequant start, 2 dequant done, 3 MMA
// issue, 4 accumulator ready (epilogue start), 5 epilogue done, 6 e4m3 tile
// landed (seen by the dequantiser), 7 producer reaches a stage, 8 its e4m3 slot
// is free, 9 MMA thread reaches a stage; cap = (entries - 1) / 10.
__device__ __forceinline__ void trace_ev(const GemmArgs& a, int role, int idx) {
  // plain stores at [role][idx] (no atomics: a returned value would stall the recording role)
  if (a.trace == nullptr || blockIdx.x != 0 || idx < 0 || idx >= a.trace_cap) return;
  a.trace[1 + (size_t)role * a.trace_cap + idx] = globaltimer_ns();
}

// Two fp32 products in one instruction (sm_100 packed f32x2 multiply, IEEE
// round-to-nearest per lane, denormals kept).
__device__ __forceinline__ float2 fmul2(float2 a, float2 b) {
  float2 r;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\t"
      "mov.b64 rb, {%4, %5};\n\t"
      "mul.rn.f32x2 rd, ra, rb;\n\t"
      "mov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(r.x), "=f"(r.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return r;
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 b = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&b);
}

// 16 e4m3 -> 16 bf16 = bf16(float(q) * scale): e4m3 -> f16 and f16 -> f32 are
// exact, the fp32 product is rounded once, then rounded to bf16 (the
// reference's load-time dequantisation, bit for bit).
__device__ __forceinline__ void dequant16(const uint4 q, float sc, uint32_t (&o)[8]) {
  const uint32_t w[4] = {q.x, q.y, q.z, q.w};
  const float2 s2 = make_float2(sc, sc);
#pragma unroll
  for (int h = 0; h < 4; ++h) {
    __half2_raw lo = __nv_cvt_fp8x2_to_halfraw2(static_cast<__nv_fp8x2_storage_t>(w[h] & 0xFFFFu), __NV_E4M3);
    __half2_raw hi = __nv_cvt_fp8x2_to_halfraw2(static_cast<__nv_fp8x2_storage_t>(w[h] >> 16), __NV_E4M3);
    const float2 flo = fmul2(__half22float2(*reinterpret_cast<__half2*>(&lo)), s2);
    const float2 fhi = fmul2(__half22float2(*reinterpret_cast<__half2*>(&hi)), s2);
    o[2 * h] = pack_bf16x2(flo.x, flo.y);
    o[2 * h + 1] = pack_bf16x2(fhi.x, fhi.y);
  }
}

template <int BN, bool PAIR, bool AFP8, int EPI>
__global__ void __launch_bounds__(GemmCfg<BN, PAIR, AFP8>::THREADS, 1)
gemm_tc_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
               const GemmArgs args) {
  pdl_enter();
  using C = GemmCfg<BN, PAIR, AFP8>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));

  // ---- shared-memory carve-up
  uint8_t* stage_base = smem;
  uint8_t* conv_base = smem + C::RING_BYTES;
  uint8_t* epi_stage = conv_base + C::CONV_BYTES;            // [EPI_WARPS][16][32] 4-byte transpose buffers
  uint8_t* extra = epi_stage + C::EPI_STAGE;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(extra);   // [16] TMA landed
  uint64_t* empty_bar = full_bar + 16;                       // [16] load slot free
  uint64_t* cfull_bar = empty_bar + 16;                      // [8] bf16 slot written
  uint64_t* cempty_bar = cfull_bar + 8;                      // [8] bf16 slot consumed
  uint64_t* bfull_bar = cempty_bar + 8;                      // [16] activation tile landed (TMEM-ring mode)
  uint64_t* bempty_bar = bfull_bar + 16;                     // [16] activation slot free
  uint64_t* accf_bar = bempty_bar + 16;
  uint64_t* acce_bar = accf_bar + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acce_bar + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* epi_ok = reinterpret_cast<volatile int*>(tmem_slot + 3);
  int* tile_prefix = reinterpret_cast<int*>(extra + 4096);
  int* row_off = tile_prefix + (kMaxGroups + 1);
  int* meta_slot = row_off + (kMaxGroups + 1);                 // [2][256] scatter slot per column
  float* meta_w = reinterpret_cast<float*>(meta_slot + 512);   // [2][256] routing weight per column

  auto ALd = [&](int s, int a) {
    return C::A_TMEM ? stage_base + s * C::A_STAGE_BYTES + a * C::ALOAD_BYTES
                     : stage_base + s * C::STAGE_BYTES + a * C::ALOAD_BYTES;
  };
  // activation tile of load stage s (shared ring) or of B-ring slot s (TMEM-ring mode)
  auto Bt = [&](int s) {
    return C::A_TMEM ? stage_base + C::STAGES * C::A_STAGE_BYTES + s * C::B_BYTES
                     : stage_base + s * C::STAGE_BYTES + C::NA * C::ALOAD_BYTES;
  };
  auto A16 = [&](int j, int a) { return conv_base + (j * C::NA + a) * C::A16_BYTES; };

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int ngroups = args.num_groups;
  const int m_tiles = args.m_tiles;
  const int k_splits = args.k_splits > 0 ? args.k_splits : 1;

  // ---- per-CTA schedule: prefix sums of tiles and rows over groups (one warp)
  if (warp == 0) {
    const int per = (ngroups + 31) / 32;
    int g0 = lane * per, g1 = min(ngroups, g0 + per);
    int tiles = 0, rows = 0;
    for (int g = g0; g < g1; ++g) {
      int c = args.group_count[g];
      tiles += (c + BN - 1) / BN * m_tiles * k_splits;
      rows += c;
    }
    int tincl = tiles, rincl = rows;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      int tv = __shfl_up_sync(0xffffffffu, tincl, o);
      int rv = __shfl_up_sync(0xffffffffu, rincl, o);
      if (lane >= o) { tincl += tv; rincl += rv; }
    }
    int tpre = tincl - tiles, rpre = rincl - rows;
    for (int g = g0; g < g1; ++g) {
      int c = args.group_count[g];
      tile_prefix[g] = tpre;
      row_off[g] = args.group_offset ? args.group_offset[g] : rpre;
      tpre += (c + BN - 1) / BN * m_tiles * k_splits;
      rpre += c;
    }
    if (lane == 31) tile_prefix[ngroups] = tincl;
  }
  if (threadIdx.x == 32) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      // fp8: the stage's dequant group (+ the MMA when the stage also holds the activation tile)
      mbar_init(&empty_bar[s], AFP8 ? C::CONV_WARPS / C::DEQ_GROUPS + (C::A_TMEM ? 0 : 1) : 1);
    }
    for (int s = 0; s < C::SB; ++s) {
      mbar_init(&bfull_bar[s], 1);
      mbar_init(&bempty_bar[s], 1);
    }
    for (int j = 0; j < 8; ++j) {
      mbar_init(&cfull_bar[j], AFP8 ? C::CONV_WARPS / C::DEQ_GROUPS : 1);
      mbar_init(&cempty_bar[j], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&accf_bar[b], 1);
      mbar_init(&acce_bar[b], C::EPI_WARPS);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  __syncwarp();
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmap_a);
    tma_prefetch_desc(&tmap_b);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int total_tiles = tile_prefix[ngroups];
  const int k_stages = args.k_stages / C::KSUB;  // pipeline stages of K (the host counts 64-wide blocks)
  auto tile_of = [&](int t) { return decode_tile(t, tile_prefix, ngroups, m_tiles, k_stages, k_splits); };
  int* status = args.status;

  if (warp == 0) {
    // ===================================================== TMA producer
    if (elect_one()) {
      int s = 0, sb = 0;
      uint32_t phase = 0, bphase = 0;
      int pi = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < total_tiles && ok; t += gridDim.x) {
        TileCoord tc = tile_of(t);
        const int a_row = tc.g * args.a_rows_per_group + tc.i * 128;
        const int b_row = row_off[tc.g] + tc.j * BN;
        for (int ks = tc.ks0; ks < tc.ks1; ++ks) {
          trace_ev(args, 7, pi);  // producer reaches the stage (before its slot waits)
          if (!mbar_wait(&empty_bar[s], phase ^ 1, status, kStatusTimeoutEmpty, abort_flag)) { ok = false; break; }
          trace_ev(args, 8, pi);  // A slot free
          mbar_arrive_expect_tx(&full_bar[s], C::A_TMEM ? C::A_STAGE_BYTES : C::TX_BYTES);
          const int x = ks * C::KS;
          if (AFP8 && args.a_tiled) {
            // tile-major weights: 64-K block b of row tile r is the 8 KB block r * (K / 64) + b,
            // so a stage (KSUB blocks) is one contiguous run
            const uint8_t* wb = static_cast<const uint8_t*>(args.a_base);
            bulk_load(ALd(s, 0), wb + ((size_t)((a_row >> 7) * args.k_stages + ks * C::KSUB) << 13), C::A8_BYTES,
                      &full_bar[s]);
            if constexpr (PAIR)
              bulk_load(ALd(s, 1),
                        wb + ((size_t)(((a_row + args.pair_row_offset) >> 7) * args.k_stages + ks * C::KSUB) << 13),
                        C::A8_BYTES, &full_bar[s]);
          } else {
#pragma unroll
            for (int sub = 0; sub < C::KSUB; ++sub) {
              tma_load_2d(ALd(s, 0) + sub * 8192, &tmap_a, &full_bar[s], x + sub * kBK, a_row);
              if constexpr (PAIR)
                tma_load_2d(ALd(s, 1) + sub * 8192, &tmap_a, &full_bar[s], x + sub * kBK, a_row + args.pair_row_offset);
            }
          }
          if constexpr (C::A_TMEM) {
            if (!mbar_wait(&bempty_bar[sb], bphase ^ 1, status, kStatusTimeoutEmpty, abort_flag)) { ok = false; break; }
            mbar_arrive_expect_tx(&bfull_bar[sb], C::B_BYTES);
#pragma unroll
            for (int sub = 0; sub < C::KSUB; ++sub)
              tma_load_2d(Bt(sb) + sub * (BN * 128), &tmap_b, &bfull_bar[sb], x + sub * kBK, b_row);
            if (++sb == C::SB) { sb = 0; bphase ^= 1; }
          } else {
            tma_load_2d(Bt(s), &tmap_b, &full_bar[s], x, b_row);
          }
          trace_ev(args, 0, pi++);
          if (++s == C::STAGES) { s = 0; phase ^= 1; }
        }
      }
      if (!ok) {
        // aborted: give loads already issued (valid global sources, so they
        // finish in microseconds) 1 ms to land before the CTA can exit
        const uint64_t t0 = globaltimer_ns();
        while (globaltimer_ns() - t0 < 1000000ull) __nanosleep(1000);
      }
    }
  } else if (warp == 1) {
    // ====================================================== MMA issuer
    if (elect_one()) {
      constexpr uint32_t idesc = umma_idesc_bf16(128, BN);
      int s = 0;       // load stage (shared ring) or activation slot (TMEM-ring mode)
      uint32_t phase = 0;
      int lt = 0;
      int gi = 0;  // global stage counter (bf16 ring index)
      bool ok = true;
      for (int t = blockIdx.x; t < total_tiles && ok; t += gridDim.x, ++lt) {
        const TileCoord tc = tile_of(t);
        const int abuf = lt & 1;
        const uint32_t aphase = (lt >> 1) & 1;
        if (!mbar_wait(&acce_bar[abuf], aphase ^ 1, status, kStatusTimeoutAccEmpty, abort_flag)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d_base = tmem_base + abuf * C::ACC_COLS;
        for (int ks = tc.ks0; ks < tc.ks1; ++ks, ++gi) {
          trace_ev(args, 9, gi);  // MMA thread reaches the stage (before its waits)
          if (!mbar_wait(C::A_TMEM ? &bfull_bar[s] : &full_bar[s], phase, status, kStatusTimeoutFull, abort_flag)) {
            ok = false;
            break;
          }
          const int cj = AFP8 ? gi % C::CONV_SLOTS : 0;
          const uint32_t cph = AFP8 ? (gi / C::CONV_SLOTS) & 1 : 0;
          if constexpr (AFP8) {
            if (!mbar_wait(&cfull_bar[cj], cph, status, kStatusTimeoutConv, abort_flag)) { ok = false; break; }
          }
          tc_fence_after();
          trace_ev(args, 3, gi);
          const uint32_t b_addr = smem_u32(Bt(s));
#pragma unroll
          for (int k = 0; k < C::KS / 16; ++k) {
            const uint64_t bdesc = umma_sdesc_sw128(b_addr + (k >> 2) * (BN * 128) + (k & 3) * 32);
#pragma unroll
            for (int a = 0; a < C::NA; ++a) {
              const uint32_t acc = (ks != tc.ks0 || k != 0) ? 1u : 0u;
              if constexpr (C::A_TMEM) {
                // bf16 A of slot cj: NA tiles x KS/2 columns, K = 16 per 8 columns
                umma_f16_ts(d_base + a * BN,
                            tmem_base + C::TSLOT_COL0 + cj * C::SLOT_COLS + a * (C::KS / 2) + k * 8, bdesc, idesc,
                            acc);
              } else {
                const uint8_t* abuf_ptr = AFP8 ? A16(cj, a) : ALd(s, a);
                const uint64_t adesc = umma_sdesc_sw128(smem_u32(abuf_ptr) + k * 32);
                umma_f16_ss(d_base + a * BN, adesc, bdesc, idesc, acc);
              }
            }
          }
          umma_commit(C::A_TMEM ? &bempty_bar[s] : &empty_bar[s]);
          if constexpr (AFP8) umma_commit(&cempty_bar[cj]);
          if (++s == (C::A_TMEM ? C::SB : C::STAGES)) { s = 0; phase ^= 1; }
        }
        if (!ok) break;
        umma_commit(&accf_bar[abuf]);
      }
    }
  } else if (warp >= 2 && warp < C::EPI_WARP0) {
    // ================================================= dequantisers
    // DEQ_GROUPS groups of warps take stages round robin; a lane converts
    // 16 / (warps per group) chunks of every weight tile of its group's stages,
    // so the per-stage wait / fence / arrive overhead is amortised over more
    // values (2 groups: 32 values per lane per tile, 4 groups: 64).
    if constexpr (AFP8 && C::A_TMEM) {
      // bf16 ring in TMEM: a lane converts chunks of its own row (TMEM lane = row;
      // warp w may only address lane quarter w & 3) and stores them with tcgen05.st.
      // The e4m3 tile arrives as 64-byte-swizzled [128][64] sub-blocks (8 KB each),
      // so the 32 lanes' row reads are bank-conflict-free.
      constexpr int kGroups = C::DEQ_GROUPS;
      constexpr int GW = C::CONV_WARPS / kGroups;          // warps per group
      constexpr int WPQ = GW / 4;                          // warps per lane quarter in a group
      constexpr int CPT = C::KS / 16;                      // 16-byte chunks of a row per tile per stage
      constexpr int CH = C::NA * CPT / WPQ;                // chunks of its row a lane converts per stage
      constexpr int BATCH = CH < 4 ? CH : 4;               // chunks in registers at a time
      static_assert(CH % BATCH == 0, "chunk batches");
      const int dw = warp - 2;
      const int group = dw / GW;
      const int quarter = warp & 3;
      const int wq = (dw % GW) / 4;
      const int row = quarter * 32 + lane;
      const bool tracer = (dw % GW) == 0 && lane == 0;  // one recorder per dequant group
      const int nkb = args.scale_k_blocks;
      const int pair_mb = C::NA > 1 ? args.pair_row_offset / 128 : 0;
      const uint32_t lane_addr = tmem_base + (uint32_t(quarter * 32) << 16) + C::TSLOT_COL0;
      const int swz = (row >> 1) & 3;
      int t = blockIdx.x, ks = -1, ks1 = 0;
      TileCoord tc{};
      auto advance = [&]() -> bool {
        if (++ks < ks1) return true;
        if (ks1 != 0) t += gridDim.x;
        if (t >= total_tiles) return false;
        tc = tile_of(t);
        ks = tc.ks0;
        ks1 = tc.ks1;
        return true;
      };
      auto load_scales = [&](float (&out)[C::NA]) {
        const float* sc = args.a_scale + (size_t)tc.g * args.scale_m_blocks * nkb + (ks * C::KS) / 128;
        out[0] = __ldg(sc + tc.i * nkb);
        if constexpr (C::NA > 1) out[1] = __ldg(sc + (tc.i + pair_mb) * nkb);
      };
      bool have = advance();
      for (int i = 0; i < group && have; ++i) have = advance();
      float next_scale[C::NA];
      if (have) load_scales(next_scale);
      int gi = group, s = group % C::STAGES, cj = group % C::CONV_SLOTS;
      uint32_t phase = (group / C::STAGES) & 1, cph = (group / C::CONV_SLOTS) & 1;
      while (have) {
        float scale[C::NA];
#pragma unroll
        for (int a = 0; a < C::NA; ++a) scale[a] = next_scale[a];
        for (int i = 0; i < kGroups && have; ++i) have = advance();
        if (have) load_scales(next_scale);
        bool w_ok = mbar_wait(&full_bar[s], phase, status, kStatusTimeoutFull, abort_flag);
        if (tracer) trace_ev(args, 6, gi);
        w_ok = w_ok && mbar_wait(&cempty_bar[cj], cph ^ 1, status, kStatusTimeoutConv, abort_flag);
        if (!__all_sync(0xffffffffu, w_ok)) break;
        if (tracer) trace_ev(args, 1, gi);
        tc_fence_after();  // the MMAs that read this TMEM slot have completed (cempty)
        const uint32_t slot_addr = lane_addr + cj * C::SLOT_COLS;
#pragma unroll
        for (int j0 = 0; j0 < CH; j0 += BATCH) {
          uint4 q[BATCH];
#pragma unroll
          for (int j = 0; j < BATCH; ++j) {
            const int c = wq * CH + j0 + j, a = c / CPT, kc = c % CPT;
            q[j] = *reinterpret_cast<const uint4*>(ALd(s, a) + (kc >> 2) * 8192 + row * 64 + (((kc & 3) ^ swz) << 4));
          }
          uint32_t o[BATCH][8];
#pragma unroll
          for (int j = 0; j < BATCH; ++j) {
            const int c = wq * CH + j0 + j;
            dequant16(q[j], scale[c / CPT], o[j]);
          }
          if (j0 + BATCH == CH) {
            // every lane's e4m3 reads have been consumed: the load slot is free for TMA
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty_bar[s]);
          }
#pragma unroll
          for (int j = 0; j < BATCH; ++j) {
            const int c = wq * CH + j0 + j, a = c / CPT, kc = c % CPT;
            tmem_st8(slot_addr + a * (C::KS / 2) + kc * 8, o[j]);
          }
        }
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&cfull_bar[cj]);  // this warp's rows of the bf16 tile are in TMEM
        if (tracer) trace_ev(args, 2, gi);
        gi += kGroups;
        s += kGroups;
        while (s >= C::STAGES) { s -= C::STAGES; phase ^= 1; }
        cj += kGroups;
        while (cj >= C::CONV_SLOTS) { cj -= C::CONV_SLOTS; cph ^= 1; }
      }
    } else if constexpr (AFP8) {
      constexpr int kGroups = C::DEQ_GROUPS;
      constexpr int GW = C::CONV_WARPS / kGroups;          // warps per group
      constexpr int CPL = 128 * kBK / 16 / (GW * 32);      // 16-byte chunks per lane per tile
      const int dw = warp - 2;
      const int group = dw / GW;
      int src_off[CPL], dst0[CPL], dst1[CPL];
#pragma unroll
      for (int j = 0; j < CPL; ++j) {
        const int chunk = (dw % GW) * 32 + lane + j * GW * 32;
        const int row = chunk >> 2, c16 = chunk & 3;
        src_off[j] = row * 64 + ((c16 ^ ((row >> 1) & 3)) << 4);  // e4m3 tiles arrive 64-byte swizzled
        // 128B-swizzled K-major row: 16-byte unit u of row r lives at u ^ (r & 7)
        dst0[j] = row * 128 + (((2 * c16) ^ (row & 7)) << 4);
        dst1[j] = row * 128 + (((2 * c16 + 1) ^ (row & 7)) << 4);
      }
      const bool tracer = dw == 0 && lane == 0;
      const int nkb = args.scale_k_blocks;
      const int pair_mb = C::NA > 1 ? args.pair_row_offset / 128 : 0;
      // (tile, stage) cursor over this CTA's stages; the group takes every kGroups-th
      int t = blockIdx.x, ks = -1, ks1 = 0;
      TileCoord tc{};
      auto advance = [&]() -> bool {
        if (++ks < ks1) return true;
        if (ks1 != 0) t += gridDim.x;
        if (t >= total_tiles) return false;
        tc = tile_of(t);
        ks = tc.ks0;
        ks1 = tc.ks1;
        return true;
      };
      auto load_scales = [&](float (&out)[C::NA]) {
        const float* sc = args.a_scale + (size_t)tc.g * args.scale_m_blocks * nkb + (ks * kBK) / 128;
        out[0] = __ldg(sc + tc.i * nkb);
        if constexpr (C::NA > 1) out[1] = __ldg(sc + (tc.i + pair_mb) * nkb);
      };
      bool have = advance();
      for (int i = 0; i < group && have; ++i) have = advance();
      float next_scale[C::NA];
      if (have) load_scales(next_scale);
      int gi = group, s = group % C::STAGES, cj = group % C::CONV_SLOTS;
      uint32_t phase = (group / C::STAGES) & 1, cph = (group / C::CONV_SLOTS) & 1;
      while (have) {
        float scale[C::NA];
#pragma unroll
        for (int a = 0; a < C::NA; ++a) scale[a] = next_scale[a];
        for (int i = 0; i < kGroups && have; ++i) have = advance();
        if (have) load_scales(next_scale);  // the group's next stage, fetched during this one
        bool w_ok = mbar_wait(&full_bar[s], phase, status, kStatusTimeoutFull, abort_flag);
        if (tracer) trace_ev(args, 6, gi);  // the e4m3 tile has landed
        w_ok = w_ok && mbar_wait(&cempty_bar[cj], cph ^ 1, status, kStatusTimeoutConv, abort_flag);
        if (!__all_sync(0xffffffffu, w_ok)) break;
        if (tracer) trace_ev(args, 1, gi);
        uint4 q[C::NA][CPL];
#pragma unroll
        for (int a = 0; a < C::NA; ++a)
#pragma unroll
          for (int j = 0; j < CPL; ++j) q[a][j] = *reinterpret_cast<const uint4*>(ALd(s, a) + src_off[j]);
#pragma unroll
        for (int a = 0; a < C::NA; ++a) {
          uint8_t* dst = A16(cj, a);
#pragma unroll
          for (int j = 0; j < CPL; ++j) {
            uint32_t o[8];
            dequant16(q[a][j], scale[a], o);
            *reinterpret_cast<uint4*>(dst + dst0[j]) = make_uint4(o[0], o[1], o[2], o[3]);
            *reinterpret_cast<uint4*>(dst + dst1[j]) = make_uint4(o[4], o[5], o[6], o[7]);
          }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&empty_bar[s]);   // this warp is done with the e4m3 tile
          mbar_arrive(&cfull_bar[cj]);  // and its slice of the bf16 tile is written
        }
        if (tracer) trace_ev(args, 2, gi);
        // the group's next stage is kGroups stages further on
        gi += kGroups;
        s += kGroups;
        while (s >= C::STAGES) { s -= C::STAGES; phase ^= 1; }
        cj += kGroups;
        while (cj >= C::CONV_SLOTS) { cj -= C::CONV_SLOTS; cph ^= 1; }
      }
    }
  } else {
    // ====================================================== epilogue
    // EPI_WARPS warps; warp w reads TMEM lane quarter (w & 3) and the two warps of
    // a quarter take alternate 16-column chunks.  A chunk (32 output features x 16
    // tokens) is transposed through a per-warp shared buffer so every lane writes
    // 16 contiguous bytes of one output row instead of one 2-byte value per column.
    constexpr int ET = C::EPI_WARPS * 32;
    const int q = warp & 3;              // TMEM lane quarter this warp may access
    const int ew = warp - C::EPI_WARP0;
    constexpr int CSTEP = C::EPI_WARPS / 4;
    const int chunk0 = ew >> 2;          // first 16-column chunk of this warp
    const int et = threadIdx.x - C::EPI_WARP0 * 32;
    uint8_t* stg = epi_stage + ew * (16 * 32 * 4);
    int lt = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < total_tiles && ok; t += gridDim.x, ++lt) {
      TileCoord tc = tile_of(t);
      const int abuf = lt & 1;
      const uint32_t aphase = (lt >> 1) & 1;
      const int count = args.group_count[tc.g];
      const int ncols = min(BN, count - tc.j * BN);
      const int row0 = row_off[tc.g] + tc.j * BN;
      int* mslot = meta_slot + abuf * 256;
      float* mw = meta_w + abuf * 256;
      if constexpr (EPI == kEpiScatter) {
        // stage the tile's scatter slots and routing weights once (while the MMAs run)
        for (int col = et; col < ncols; col += ET) {
          const int slot = args.slot_of_row[row0 + col];
          mslot[col] = slot;
          mw[col] = args.peer_scatter ? args.slot_weight[row0 + col] : args.slot_weight[slot];
        }
      }
      // one thread waits for the accumulator, the verdict is broadcast so the
      // epilogue warps always leave (or continue) together
      if (et == 0) {
        epi_ok[0] = mbar_wait(&accf_bar[abuf], aphase, status, kStatusTimeoutAccFull, abort_flag) ? 1 : 0;
        trace_ev(args, 4, lt);
      }
      named_barrier_sync(2, ET);
      if (!epi_ok[0]) { ok = false; break; }
      tc_fence_after();
      const uint32_t t_base = tmem_base + (uint32_t(q * 32) << 16) + abuf * C::ACC_COLS;
      const int m0 = tc.i * 128 + q * 32;  // first output feature of this warp's rows
#pragma unroll 1
      for (int c16 = chunk0; c16 < BN / 16; c16 += CSTEP) {
        if (c16 * 16 >= ncols) break;
        float v[16];
        tmem_ld16(t_base + c16 * 16, v);
        if constexpr (EPI == kEpiSiluPair) {
          float u[16];
          tmem_ld16(t_base + BN + c16 * 16, u);
          tmem_ld_wait();
#pragma unroll
          for (int n = 0; n < 16; ++n) v[n] = silu(v[n]) * u[n];
        } else {
          tmem_ld_wait();
        }
        if constexpr (EPI == kEpiScatter) {
#pragma unroll
          for (int n = 0; n < 16; ++n) v[n] *= mw[c16 * 16 + n];
        }
        // first element of output row `col` (this tile's features start at m0)
        auto row_ptr = [&](int col) -> void* {
          if constexpr (EPI == kEpiF32) {
            return reinterpret_cast<float*>(args.out) + (size_t)tc.sp * args.split_stride +
                   (size_t)(row0 + col) * args.ld_out + (size_t)tc.g * args.out_group_stride + m0;
          } else if constexpr (EPI == kEpiScatter) {
            const int code = mslot[col];
            if (args.peer_scatter)  // the row goes to its source rank's slots (peer memory)
              return reinterpret_cast<__nv_bfloat16*>(args.peer_out[code / args.slot_cap]) +
                     (size_t)(code % args.slot_cap) * args.ld_out + m0;
            return reinterpret_cast<__nv_bfloat16*>(args.out) + (size_t)code * args.ld_out + m0;
          } else if constexpr (EPI == kEpiSiluPair) {
            return reinterpret_cast<__nv_bfloat16*>(args.out) + (size_t)(row0 + col) * args.ld_out + m0;
          } else {
            return reinterpret_cast<__nv_bfloat16*>(args.out) + (size_t)(row0 + col) * args.ld_out +
                   (size_t)tc.g * args.out_group_stride + m0;
          }
        };
        if constexpr (!C::EPI_STAGED) {
#pragma unroll
          for (int n = 0; n < 16; ++n) {
            const int col = c16 * 16 + n;
            if (col < ncols) {
              if constexpr (EPI == kEpiF32) reinterpret_cast<float*>(row_ptr(col))[lane] = v[n];
              else reinterpret_cast<__nv_bfloat16*>(row_ptr(col))[lane] = __float2bfloat16(v[n]);
            }
          }
        } else if constexpr (EPI == kEpiF32) {
          float* s32 = reinterpret_cast<float*>(stg);
#pragma unroll
          for (int n = 0; n < 16; ++n) s32[n * 32 + lane] = v[n];
          __syncwarp();
#pragma unroll
          for (int rd = 0; rd < 4; ++rd) {  // 16 columns x 8 four-float pieces
            const int idx = rd * 32 + lane, n = idx >> 3, piece = idx & 7;
            const int col = c16 * 16 + n;
            if (col < ncols)
              *reinterpret_cast<float4*>(reinterpret_cast<float*>(row_ptr(col)) + piece * 4) =
                  *reinterpret_cast<const float4*>(s32 + n * 32 + piece * 4);
          }
        } else {
          __nv_bfloat16* s16 = reinterpret_cast<__nv_bfloat16*>(stg);
#pragma unroll
          for (int n = 0; n < 16; ++n) s16[n * 32 + lane] = __float2bfloat16(v[n]);
          __syncwarp();
#pragma unroll
          for (int rd = 0; rd < 2; ++rd) {  // 16 columns x 4 eight-value pieces
            const int idx = rd * 32 + lane, n = idx >> 2, piece = idx & 3;
            const int col = c16 * 16 + n;
            if (col < ncols)
              *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(row_ptr(col)) + piece * 8) =
                  *reinterpret_cast<const uint4*>(s16 + n * 32 + piece * 8);
          }
        }
        __syncwarp();  // the buffer is rewritten by the next chunk
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acce_bar[abuf]);
      if (et == 0) trace_ev(args, 5, lt);
    }
  }

  tc_fence_before();
  // the epilogue's peer stores are ordered before thread 0's system-scope fence below by
  // this barrier (the fence is cumulative), so no thread fences on its own
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
  if (args.ep_epoch != nullptr && threadIdx.x == 0) {
    fence_acq_rel_sys();
    if (atomicAdd(args.ep_cta_done, 1) == (int)gridDim.x - 1) {  // every CTA's rows are out
      *args.ep_cta_done = 0;
      fence_acq_rel_sys();
      const uint32_t epoch = *args.ep_epoch + (uint32_t)args.ep_epoch_add;
      for (int r = 0; r < args.ep_world; ++r)
        st_release_sys(reinterpret_cast<uint32_t*>(args.ep_done[r]) + args.ep_rank, epoch);
    }
  }
  pdl_trigger();
}

// ------------------------------------------------------------------ host side

static PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (fn == nullptr) {
    cudaDriverEntryPointQueryResult qres;
    void* p = nullptr;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &qres);
    if (e != cudaSuccess || qres != cudaDriverEntryPointSuccess || p == nullptr)
      throw std::runtime_error("cuTensorMapEncodeTiled entry point not available");
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

CUtensorMap make_tmap_2d(const void* base, bool is_bf16, int64_t rows, int64_t cols,
                         int64_t row_stride_bytes, int box_cols, int box_rows, int swizzle_bytes) {
  CUtensorMap map;
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)row_stride_bytes};
  const cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = get_encode_fn()(
      &map, is_bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8, 2,
      const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
      swizzle_bytes == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
      : swizzle_bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_NONE,
      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    throw std::runtime_error("cuTensorMapEncodeTiled failed: " + std::to_string((int)r));
  return map;
}

static int num_sms() { return device_sm_count(); }

template <int BN, bool PAIR, bool AFP8, int EPI>
static void launch_impl(const GemmLaunch& L, cudaStream_t stream) {
  using C = GemmCfg<BN, PAIR, AFP8>;
  auto kern = gemm_tc_kernel<BN, PAIR, AFP8, EPI>;
  smem_opt_in(kern, C::SMEM);
  // A: [groups * rows_per_group, K] row-major, box 64 x 128 rows; tile-major e4m3
  // weights are addressed as [groups * rows_per_group * K / 64, 64]
  const int64_t a_rows = (int64_t)L.args.num_groups * L.args.a_rows_per_group;
  // e4m3 tiles land 64-byte swizzled (the TMEM-ring dequantisers read one row per
  // lane: conflict-free); tile-major weights carry the same order in memory
  const int a_swz = !AFP8 ? 128 : 64;
  // (tile-major e4m3 weights are fetched with bulk copies; the map is then unused)
  CUtensorMap ta = make_tmap_2d(L.a, !AFP8, a_rows, L.K, L.a_row_stride_bytes, kBK, 128, a_swz);
  CUtensorMap tb = make_tmap_2d(L.b, true, L.b_rows, L.K, L.b_row_stride_bytes, kBK, BN, 128);
  // upper bound of work items without reading device counts
  int64_t max_tiles = ((int64_t)L.b_rows / BN + L.args.num_groups) * L.args.m_tiles * std::max(1, L.args.k_splits);
  int grid = (int)std::min<int64_t>(num_sms(), std::max<int64_t>(1, max_tiles));
  pdl_launch(kern, grid, C::THREADS, C::SMEM, stream, ta, tb, L.args);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) throw std::runtime_error(std::string("gemm_tc launch: ") + cudaGetErrorString(e));
}

template <bool PAIR, bool AFP8, int EPI>
static void dispatch_bn(int bn, const GemmLaunch& L, cudaStream_t s) {
  switch (bn) {
    case 16: launch_impl<16, PAIR, AFP8, EPI>(L, s); return;
    case 32: launch_impl<32, PAIR, AFP8, EPI>(L, s); return;
    case 64: launch_impl<64, PAIR, AFP8, EPI>(L, s); return;
    case 128: launch_impl<128, PAIR, AFP8, EPI>(L, s); return;
    case 256:
      if constexpr (!PAIR) { launch_impl<256, PAIR, AFP8, EPI>(L, s); return; }
      break;
    default: break;
  }
  throw std::runtime_error("unsupported BN " + std::to_string(bn));
}

void gemm_tc_launch(const GemmLaunch& L, cudaStream_t stream) {
  if (L.args.num_groups < 1 || L.args.num_groups > kMaxGroups) throw std::runtime_error("bad group count");
  if (L.args.a_tiled && (!L.a_fp8 || L.a_row_stride_bytes != L.K || (reinterpret_cast<uintptr_t>(L.args.a_base) & 15)))
    throw std::runtime_error("tile-major weights must be dense, 16-byte aligned e4m3 [rows, K]");
  if (L.K % 128 != 0) throw std::runtime_error("K must be a multiple of 128");
  if (L.args.a_rows_per_group % 128 != 0) throw std::runtime_error("weight rows must be a multiple of 128");
  if ((reinterpret_cast<uintptr_t>(L.a) & 15) || (reinterpret_cast<uintptr_t>(L.b) & 15))
    throw std::runtime_error("operands must be 16-byte aligned");
  if (L.b_row_stride_bytes % 16 != 0) throw std::runtime_error("activation row stride must be a multiple of 16 bytes");
  {
    // the epilogue writes 16-byte pieces of output rows
    const int vec = L.epi == kEpiF32 ? 4 : 8;
    if (L.args.ld_out % vec || L.args.out_group_stride % vec || L.args.split_stride % vec ||
        (reinterpret_cast<uintptr_t>(L.args.out) & 15))
      throw std::runtime_error("output rows must be 16-byte aligned (row stride, group stride, split stride)");
    if (L.args.peer_scatter)
      for (int r = 0; r < 8; ++r)
        if (reinterpret_cast<uintptr_t>(L.args.peer_out[r]) & 15)
          throw std::runtime_error("peer scatter outputs must be 16-byte aligned");
  }
  const int bn = L.bn;
  if (L.args.k_splits > 1) {
    if (L.epi != kEpiF32 || L.pair) throw std::runtime_error("split-K needs the fp32 epilogue");
    // e4m3 single-tile GEMMs with token tiles up to 128 run 128-wide K stages
    const int stages = (L.a_fp8 && bn <= 128) ? L.args.k_stages / 2 : L.args.k_stages;
    const int per = (stages + L.args.k_splits - 1) / L.args.k_splits;
    if ((L.args.k_splits - 1) * per >= stages) throw std::runtime_error("split-K leaves a split empty");
  }
  if (L.pair) {
    if (L.epi != kEpiSiluPair) throw std::runtime_error("pair mode is the silu epilogue only");
    if (L.a_fp8) dispatch_bn<true, true, kEpiSiluPair>(bn, L, stream);
    else dispatch_bn<true, false, kEpiSiluPair>(bn, L, stream);
    return;
  }
  if (L.a_fp8) {
    if (L.epi == kEpiBf16) dispatch_bn<false, true, kEpiBf16>(bn, L, stream);
    else if (L.epi == kEpiF32) dispatch_bn<false, true, kEpiF32>(bn, L, stream);
    else if (L.epi == kEpiScatter) dispatch_bn<false, true, kEpiScatter>(bn, L, stream);
    else throw std::runtime_error("unsupported fp8 epilogue");
  } else {
    if (L.epi == kEpiF32) dispatch_bn<false, false, kEpiF32>(bn, L, stream);
    else if (L.epi == kEpiBf16) dispatch_bn<false, false, kEpiBf16>(bn, L, stream);
    else if (L.epi == kEpiScatter) dispatch_bn<false, false, kEpiScatter>(bn, L, stream);
    else throw std::runtime_error("unsupported bf16 epilogue");
  }
}

}  // namespace b200

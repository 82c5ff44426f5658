// Host/device interface of the tcgen05 grouped GEMM (kernels/gemm_tc.cu).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <cstdint>

namespace b200 {

enum GemmEpilogue : int {
  kEpiBf16 = 0,      // out[row, g*out_group_stride + m] = bf16(acc)
  kEpiF32 = 1,       // same, fp32
  kEpiSiluPair = 2,  // out[row, m] = bf16(silu(acc_gate) * acc_up)
  kEpiScatter = 3,   // out[slot_of_row[row], m] = bf16(acc * slot_weight[slot])
};

// Kernel arguments (passed by value; device pointers only).
struct GemmArgs {
  const float* a_scale;        // fp8 mode: [groups, scale_m_blocks, scale_k_blocks]
  int a_rows_per_group;        // weight rows per group (row stride between groups)
  int m_tiles;                 // 128-row tiles computed per group (pair: gate tiles)
  int k_stages;                // K / 64
  int scale_m_blocks;
  int scale_k_blocks;
  int num_groups;
  const int* group_count;      // [groups] activation rows per group (device)
  const int* group_offset;     // [groups] first activation row, or null = prefix of counts
  int pair_row_offset;         // pair mode: row offset of the "up" half inside a group
  void* out;
  int ld_out;                  // output row stride (elements)
  int out_group_stride;        // column offset per group for kEpiBf16/kEpiF32
  // split-K (kEpiF32 only): work item (tile, split) sums K stages
  // [split * ceil(k_stages / k_splits), ...) and stores its fp32 partial at
  // out + split * split_stride; the caller reduces the partials
  int k_splits;
  long long split_stride;
  const int* slot_of_row;      // kEpiScatter
  const float* slot_weight;    // kEpiScatter: routing weight per output row (indexed by row)
  int* status;                 // device status word (0 = ok)
  // kEpiScatter into peers' memory (expert parallel): slot code = rank * slot_cap + slot
  int peer_scatter;
  int slot_cap;
  void* peer_out[8];
  // optional pipeline trace of CTA 0: pairs (role << 32 | index, %globaltimer); entry 0 = count
  unsigned long long* trace;
  int trace_cap;
  // e4m3 weights stored tile-major: [row tile][K / 64][128 rows][64 B] with the
  // 16-byte chunks of each row in 64-byte-swizzle order, so one pipeline stage is
  // one contiguous 8 KB block fetched by a single bulk copy
  int a_tiled;
  const void* a_base;
  // cross-GPU release (expert-parallel peer scatter, tensor-parallel partials): the
  // CTA that finishes last writes *ep_epoch + ep_epoch_add into ep_done[r] + ep_rank
  // for every rank r, after every CTA has fenced its stores; null ep_epoch = none
  const uint32_t* ep_epoch;
  int ep_epoch_add;
  int* ep_cta_done;            // local counter, zero between launches
  void* ep_done[8];
  int ep_rank;
  int ep_world;
};

struct GemmLaunch {
  GemmArgs args;
  const void* a;               // weight base
  int64_t a_row_stride_bytes;
  const void* b;               // activation base (bf16)
  int64_t b_rows;              // rows addressable through the activation tensor map
  int64_t b_row_stride_bytes;
  int K;
  int bn;                      // token tile: 16, 32, 64, 128 (256 when not pair)
  bool a_fp8;
  bool pair;
  int epi;
};

void gemm_tc_launch(const GemmLaunch& launch, cudaStream_t stream);
CUtensorMap make_tmap_2d(const void* base, bool is_bf16, int64_t rows, int64_t cols,
                         int64_t row_stride_bytes, int box_cols, int box_rows, int swizzle_bytes);

}  // namespace b200

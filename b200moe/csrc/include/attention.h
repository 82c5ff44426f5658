// Host interface of the paged attention kernels (kernels/attention.cu).
#pragma once
#include <cuda_runtime.h>
#include <cstdint>

namespace b200 {

constexpr int kKvNoutMax = 4;  // exact bf16 outlier dims per (layer, kv head), int8 channel mode

// int8 KV "channel" mode (kv_int8 == 2): per-channel read scales and up to
// kKvNoutMax exact bf16 outlier dims per kv head, kept in a side pool.
struct KvChannel {
  const float* dscale;         // layer: [2, kv_heads, D] (k then v), 0 at outlier dims
  const int* out_idx;          // layer: [kv_heads, kKvNoutMax]
  const int* n_out;            // layer: [kv_heads]
  const void* side_k;          // layer base of the side pool [blocks, kv_heads, block_size, kKvNoutMax] bf16
  const void* side_v;
  int64_t side_block_stride;   // elements between consecutive blocks
};

struct DecodeArgs {
  const void* q;             // [B, q_heads, D] bf16
  const void* k_cache;       // layer base of the pool, [blocks, kv_heads, block_size, D]
  const void* v_cache;
  const float* k_scale;      // int8 KV scales (unused for bf16)
  const float* v_scale;
  int kv_int8;               // 0 bf16, 1 int8 per-token scales, 2 int8 channel mode (ch)
  KvChannel ch;
  const int* block_tables;   // [B, max_blocks]
  const int* seq_lens;       // [B] keys per sequence (including the current token)
  int max_blocks;
  int block_size;
  int64_t block_stride;      // elements between consecutive blocks of one layer
  int num_kv_heads;
  int group;                 // q heads per kv head
  int head_dim;
  float scale;
  int num_splits;
  int split_len;             // keys per split (multiple of 64)
  float* part_o;             // [B, q_heads, num_splits, D]
  float* part_m;             // [B, q_heads, num_splits]
  float* part_l;
  void* out;                 // [B, q_heads, D] bf16
  int num_blocks;            // blocks in the pool (TMA path: out-of-range block = zero fill)
  int* status;               // device status word (bounded waits), may be null
};

struct PrefillArgs {
  const void* q;             // [T, q_heads, D] bf16 (rows of all prefill sequences)
  const void* k_cache;
  const void* v_cache;
  const float* k_scale;
  const float* v_scale;
  int kv_int8;               // 0 bf16, 1 int8 per-token scales, 2 int8 channel mode (ch)
  KvChannel ch;
  const int* cu_seqlens_q;   // [B + 1]
  const int* seq_lens;       // [B] total keys (cached + new)
  const int* block_tables;   // [B, max_blocks]
  int max_blocks;
  int block_size;
  int64_t block_stride;
  int num_kv_heads;
  int group;
  int head_dim;
  float scale;
  void* out;                 // [T, q_heads, D] bf16
  int num_blocks;            // blocks in the pool (tensor-core path: out-of-range block = zero fill)
  int* status;               // device status word (bounded waits), may be null
  int q_rows;                // rows of q (tensor-core path: Q tensor map extent)
  int batch;                 // sequences (set by the launcher)
};

// int8 KV -> bf16 staging pool for the tensor-core prefill.  Block j of sequence b
// (j < ceil(seq_lens[b] / block_size)) is dequantised to staging block b * max_blocks + j,
// laid out as the bf16 pool's blocks are ([k|v][kv_heads][block_size][head_dim]); slots
// at or past seq_lens[b] are written as zeros.  Values are the ones the int8 attention
// kernels compute while staging (fp32 product, rounded to bf16 once).
struct KvStageArgs {
  const void* k_cache;       // int8 layer bases
  const void* v_cache;
  const float* k_scale;      // kv_int8 == 1
  const float* v_scale;
  int kv_int8;               // 1 per-token scales, 2 channel mode (ch)
  KvChannel ch;
  const int* block_tables;   // [batch, max_blocks]
  const int* seq_lens;       // [batch]
  int batch;
  int max_blocks;
  int block_size;
  int64_t block_stride;      // int8 elements between consecutive blocks of the layer
  int num_kv_heads;
  int head_dim;
  void* stage;               // bf16 [batch * max_blocks][2][kv_heads][block_size][head_dim]
};
void kv_int8_stage(const KvStageArgs& a, cudaStream_t s);

void paged_decode_attn(const DecodeArgs& a, int B, cudaStream_t s);
void paged_prefill_attn(const PrefillArgs& a, int B, int max_q_len, cudaStream_t s);

// tcgen05 causal prefill (kernels/fmha_tc.cu): bf16 pool, head_dim 128.
bool fmha_prefill_supported(const PrefillArgs& a, int* sub_rows);
void fmha_prefill(const PrefillArgs& a, int B, int max_q_len, int sub_rows, cudaStream_t s);

}  // namespace b200

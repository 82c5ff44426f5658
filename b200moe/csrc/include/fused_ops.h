// Host interface of the memory-bound fused ops (kernels/fused_ops.cu).
#pragma once
#include <cuda_runtime.h>
#include <cstdint>

#include "ep_p2p.h"

namespace b200 {

constexpr int kMaxExperts = 512;

struct QkvArgs {
  const void* qkv;          // [T, qkv_stride] bf16: q heads | k heads | v heads
  int qkv_stride;           // elements
  const int* positions;     // [T]
  const int* slot_mapping;  // [T] flat KV slot (block * block_size + offset), -1 = no store
  const void* q_norm_w;     // [D] bf16
  const void* k_norm_w;     // [D] bf16
  const float* cos_sin;     // [max_pos, D]: cos[0:D/2] | sin[0:D/2]
  void* k_cache;            // layer base, [blocks, kv_heads, block_size, D] bf16 or int8
  void* v_cache;
  float* k_scale;           // int8 KV: layer base, [blocks, kv_heads, block_size]
  float* v_scale;
  int kv_int8;
  int block_size;
  int64_t block_stride;     // elements between consecutive blocks of the KV pool
  int64_t scale_block_stride;
  void* q_out;              // [T, q_heads, D] bf16
  int num_q_heads;
  int num_kv_heads;
  int head_dim;
  float eps;
  // optional: q/k/v given as `splits` fp32 split-K partials of the QKV GEMM at
  // part + s * part_stride + t * qkv_stride, summed in split order and rounded to
  // bf16 here (the same bits as a separate split-K reduction); qkv is then unused
  const float* part;
  int splits;
  int64_t part_stride;
  // int8 channel mode (kv_int8 == 2): per-channel store scales, exact outlier dims
  // in the side pool, and (while calibrating) running max / sum of |x| per channel
  const float* ch_scale;    // layer: [2, kv_heads, D]
  const int* out_idx;       // layer: [kv_heads, 4]
  const int* n_out;         // layer: [kv_heads]
  void* side_k;             // layer base of the side pool [blocks, kv_heads, block_size, 4] bf16
  void* side_v;
  int64_t side_block_stride;
  float* calib_amax;        // layer: [2, kv_heads, D], or null when not calibrating
  float* calib_sum;
};

void embed_gather(const int* ids, const void* table, void* out, int T, int H, int V, int* status,
                  cudaStream_t s,
                  const int* feed_src = nullptr, const int* feed_tokens = nullptr);
// part != null: x is given as `splits` fp32 partial sums [splits, T, H] (split-K GEMM
// output), reduced and rounded to bf16 before the residual add.
void rmsnorm(const void* x, const void* res_in, const void* w, void* out, void* res_out, int T, int H,
             float eps, cudaStream_t s, const float* part = nullptr, int splits = 0);
// Expert parallel: before combining, wait for every owner's done epoch, flags[r] >= *epoch
// for r < world (bounded; the time waited on owner r is added to wait_ns[world + r]).
struct CombineWait {
  const uint32_t* flags = nullptr;   // this rank's done array [world]; null = no wait
  const uint32_t* epoch = nullptr;
  int world = 0;
  int* status = nullptr;
  unsigned long long* wait_ns = nullptr;
};
// T == 0 with a wait still launches one block, which only waits.
void moe_combine_add_rmsnorm(const void* slots, int topk, void* residual, const void* w, void* out, int T,
                             int H, float eps, cudaStream_t s,
                             int* zero_buf = nullptr, int zero_n = 0, const CombineWait& cw = CombineWait{});
void qknorm_rope_kvstore(const QkvArgs& a, int T, cudaStream_t s);
void router_topk(const float* logits, int ld, int T, int E, int topk, bool renorm, int* ids, float* weights,
                 int* counts, cudaStream_t s);
// out[t, n] = sum_s part[s, t, n] (fp32 partials of a split-K GEMM, rows of N
// floats, split stride T*N) stored as bf16 (out_bf16) or fp32 with row stride ld_out.
void splitk_reduce(const float* part, int splits, int T, int N, void* out, int ld_out, bool out_bf16,
                   cudaStream_t s);
// Whole KV-block copy: dst_base + dst_ids[i] * block_bytes <- src_base + src_ids[i] * block_bytes
// (16-byte plain loads / stores; dst may be a peer GPU's pool mapped over NVLink).
void kv_blocks_copy(const void* src_base, const int* src_ids, void* dst_base, const int* dst_ids, int n,
                    int64_t block_bytes, cudaStream_t s);
// Router GEMM (x [T, H] bf16 . w[:E]^T, fp32 accumulate, bf16-rounded logits) +
// softmax + top-k in one launch; E <= 128.
// e4m3 [G, N, K] (row-major or tile-major) + 128x128 block scales -> bf16 row-major
void dequant_weights(const void* q, const float* scale, void* out, int G, int N, int K, bool tiled, cudaStream_t s);
// part / tile_cnt (optional): fp32 scratch for part_tiles partial tiles of 16 x 128 logits and a
// zeroed int per token tile; with them, batches too small to fill the SMs also split K.
// ep (optional): expert parallelism -- the top-k warps also send each routed row to its
// expert's owner and the grid publishes this rank's counts and epoch, which is what
// ep_dispatch does as a separate launch.
void router_fused(const void* x, const void* w, int T, int H, int E, int w_rows, int topk, bool renorm, int* ids,
                  float* weights, int* counts, int* status, cudaStream_t s, float* part = nullptr,
                  int* tile_cnt = nullptr, int part_tiles = 0, const EpArgs* ep = nullptr);
void moe_permute(const void* x, const int* ids, int T, int topk, int E, int H, const int* counts, int* cursor,
                 void* x_perm, int* slot_of_row, int* offsets_out, cudaStream_t s);

}  // namespace b200

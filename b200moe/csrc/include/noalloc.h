// C entry point of split-KV paged decode attention that allocates nothing.
//
// This entry point has no counterpart in the reference: there, every attention call
// gets its workspace from the PyTorch caching allocator.  It exists for callers
// that must not allocate device memory while they run:
//   * a host runtime that is not PyTorch (a C/C++ server, a ctypes or FFI caller)
//     and so has no caching allocator to take a workspace from;
//   * code that runs while an allocator is unusable or forbidden, such as a
//     watchdog or teardown path, or a process with a memory budget that is fixed
//     once the model is loaded.
// The split-KV partial results (part_o / part_m / part_l) live in a file-scope
// `__device__` array of kNoAllocMaxRows rows (kNoAllocMaxRows * (128 + 2) floats,
// 8.1 MiB per device, which the module reserves when it loads).  A call whose
// batch * q_heads * num_splits is above kNoAllocMaxRows is rejected with an error
// message and launches nothing.
//
// Set-up: the first call on each device resolves the array's address with
// cudaGetSymbolAddress while that device is current.  Make that first call
// before any stream capture on the device.
// Nothing in the array has to start at zero: the combine step reads only the
// partials that the split step of the same call writes.
// Calls that overlap in time on one device (different streams, different host
// threads without stream order) share the array and race; serialise them.
#pragma once
#include <cstdint>

#ifdef __cplusplus
extern "C" {
#endif

// Most split rows (batch * q_heads * num_splits) one call may use.
#define B200MOE_NOALLOC_MAX_ROWS 16384

// Returns 0 on success.  On failure returns a non-zero code and writes a
// NUL-terminated message into err[0..err_len) (when err is not null):
//   1  invalid argument: a count below 1 (q / kv heads, num_splits, block_size,
//      max_blocks, block_stride, split_len), q_heads not a multiple of kv_heads,
//      a GQA group above 16 or not dividing 64, split_len not a multiple of 64,
//      head_dim other than 64 / 128, int8 KV without scales, a null pointer
//   2  size above B200MOE_NOALLOC_MAX_ROWS
//   3  CUDA error (device query, symbol lookup or launch)
// Nothing is launched when the code is non-zero.
// Two preconditions live in device memory, so they cannot be checked here and
// are the caller's to keep:
//   * num_splits * split_len >= the longest seq_lens[b]: keys past that are not
//     attended to (the split count is capped, not grown);
//   * block_tables row b holds ceil(seq_lens[b] / block_size) <= max_blocks valid
//     block ids: the kernel reads those entries without a bounds check.
// The kernel is the cp.async split-KV decode kernel (bf16 or int8 KV), not the
// TMA kernel the PyTorch binding uses for bf16 pools: the TMA kernel needs the
// pool's block count, which this signature does not carry.
// q [batch, num_q_heads, head_dim] bf16; k_cache / v_cache the layer base of
// the paged pool [blocks, kv_heads, block_size, head_dim] (bf16, or int8 with
// per-token-head fp32 scales k_scale / v_scale); block_tables [batch,
// max_blocks] int32; seq_lens [batch] int32; out [batch, num_q_heads,
// head_dim] bf16.  `stream` is a cudaStream_t (null = the legacy stream).
int b200moe_decode_attn_noalloc(const void* q, const void* k_cache, const void* v_cache,
                                const float* k_scale, const float* v_scale, int kv_int8,
                                const int* block_tables, const int* seq_lens, int batch, int max_blocks,
                                int block_size, long long block_stride, int num_q_heads, int num_kv_heads,
                                int head_dim, float scale, int num_splits, int split_len, void* out,
                                void* stream, char* err, int err_len);

// B200MOE_NOALLOC_MAX_ROWS, for callers that load the library dynamically.
int b200moe_decode_attn_noalloc_max_rows(void);

#ifdef __cplusplus
}
#endif

// Host interface of the expert-parallel P2P dispatch/combine kernels (kernels/ep_p2p.cu).
#pragma once
#include <cuda_runtime.h>
#include <cstdint>

namespace b200 {

constexpr int kEpMaxWorld = 8;
constexpr int kEpMaxLocalExperts = 256;

// Passed by value.  Pointer arrays hold every rank's copy of a symmetric buffer.
struct EpArgs {
  int world;
  int rank;
  int hidden;
  int cap;                       // rows per source segment of recv_x
  int slot_cap;                  // (token, k) slots per rank
  int num_local;                 // experts per rank (El)
  int num_experts;               // E
  const int* owner;              // [E] owning rank of each global expert
  const int* g2l;                // [E] local index on this rank, -1 if not local
  const int* ge_local;           // [E] local index of each expert on its owner
  int* send_cursor;              // [world] local scratch, zero between layers
  int* ecur;                     // [E] local scratch: rows this rank routed to each expert, zero between layers
  int* done_blocks;              // local scratch counter, zero between layers
  uint32_t* epoch;               // local epoch counter
  int* status;
  // [2 * world] ns spent waiting, accumulated on the device: [0, world) for each
  // source's dispatch flag (ep_count), [world, 2 * world) for each owner's done
  // epoch (ep_wait_done).  A large entry names the rank the others wait for.
  unsigned long long* wait_ns;
  void* recv_x[kEpMaxWorld];
  void* recv_meta[kEpMaxWorld];
  void* counts[kEpMaxWorld];     // [world * num_local] per rank: rows from source s for local expert e at s * El + e
  void* flags[kEpMaxWorld];
  void* done[kEpMaxWorld];
};

void ep_dispatch(const EpArgs& a, const void* x, const int* ids, const float* w, int T, int topk, cudaStream_t s);
void ep_scatter(const EpArgs& a, int* local_counts, void* x_perm, int* slot_code, float* slot_w, int* offsets_out,
                int max_rows, cudaStream_t s);
void ep_signal(const EpArgs& a, cudaStream_t s);
void ep_wait_done(const EpArgs& a, cudaStream_t s);

}  // namespace b200

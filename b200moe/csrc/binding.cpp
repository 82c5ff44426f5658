// PyTorch bindings of the sm_100a kernels.  Every entry point checks device,
// dtype, contiguity and shapes on the host before launching on the current
// CUDA stream, so a bad call raises a Python exception instead of faulting.
#include <torch/extension.h>
#include <cuda.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <cstring>
#include <tuple>
#include <vector>

#include "attention.h"
#include "ep_p2p.h"
#include "tp_comm.h"
#include "fused_ops.h"
#include "gemm_tc.h"
#include "sampler.h"

namespace {

using torch::Tensor;

#define CHECK_CUDA(t) TORCH_CHECK((t).is_cuda(), #t " must be a CUDA tensor")
#define CHECK_CONTIG(t) TORCH_CHECK((t).is_contiguous(), #t " must be contiguous")
#define CHECK_DT(t, dt) TORCH_CHECK((t).scalar_type() == (dt), #t " has dtype ", (t).scalar_type(), ", expected ", dt)

cudaStream_t stream() { return at::cuda::getCurrentCUDAStream().stream(); }

template <typename T>
T* ptr_or_null(const c10::optional<Tensor>& t) {
  return t.has_value() ? static_cast<T*>(t->data_ptr()) : nullptr;
}

// out = grouped GEMM of weight groups x activation rows (see gemm_tc.cu).
void gemm(Tensor weight, c10::optional<Tensor> weight_scale, Tensor x, Tensor group_count,
          c10::optional<Tensor> group_offset, Tensor out, int64_t bn, int64_t epi, int64_t m_tiles,
          int64_t pair_row_offset, int64_t out_group_stride, c10::optional<Tensor> slot_of_row,
          c10::optional<Tensor> slot_weight, Tensor status, c10::optional<Tensor> trace, int64_t k_splits,
          int64_t split_stride, bool a_tiled, std::vector<int64_t> release) {
  CHECK_CUDA(weight); CHECK_CUDA(x); CHECK_CUDA(out); CHECK_CUDA(group_count); CHECK_CUDA(status);
  CHECK_CONTIG(weight); CHECK_CONTIG(group_count);
  TORCH_CHECK(out.stride(-1) == 1, "out must have unit inner stride");
  TORCH_CHECK(x.dim() == 2 && x.stride(1) == 1, "x must be [rows, K] with unit inner stride");
  TORCH_CHECK(weight.dim() == 2 || weight.dim() == 3, "weight must be [N, K] or [groups, N, K]");
  CHECK_DT(x, torch::kBFloat16);
  CHECK_DT(group_count, torch::kInt32);
  CHECK_DT(status, torch::kInt32);
  const bool fp8 = weight.scalar_type() == torch::kFloat8_e4m3fn;
  TORCH_CHECK(fp8 || weight.scalar_type() == torch::kBFloat16, "weight must be e4m3 or bf16");
  const int64_t groups = weight.dim() == 3 ? weight.size(0) : 1;
  const int64_t rows_per_group = weight.size(-2);
  const int64_t K = weight.size(-1);
  TORCH_CHECK(x.size(1) == K, "K mismatch: weight ", K, " vs x ", x.size(1));
  TORCH_CHECK(group_count.numel() == groups, "group_count must have one entry per weight group");
  if (fp8) {
    TORCH_CHECK(weight_scale.has_value(), "fp8 weight needs weight_scale");
    CHECK_DT((*weight_scale), torch::kFloat32);
    CHECK_CONTIG((*weight_scale));
    TORCH_CHECK(weight_scale->numel() == groups * (rows_per_group / 128) * (K / 128),
                "weight_scale must be [groups, N/128, K/128]");
    TORCH_CHECK(K <= 8192, "K must be at most 8192 (64 scale blocks per tile)");
  }
  if (group_offset.has_value()) {
    CHECK_DT((*group_offset), torch::kInt32);
    TORCH_CHECK(group_offset->numel() >= groups, "group_offset too short");
  }
  const bool pair = epi == b200::kEpiSiluPair;
  if (epi == b200::kEpiScatter) {
    TORCH_CHECK(slot_of_row.has_value() && slot_weight.has_value(), "scatter epilogue needs slots");
    CHECK_DT((*slot_of_row), torch::kInt32);
    CHECK_DT((*slot_weight), torch::kFloat32);
  }
  if (epi == b200::kEpiF32) {
    CHECK_DT(out, torch::kFloat32);
  } else {
    CHECK_DT(out, torch::kBFloat16);
  }
  TORCH_CHECK(m_tiles * 128 <= rows_per_group, "m_tiles exceeds weight rows");
  TORCH_CHECK(k_splits >= 1 && k_splits <= K / 64, "k_splits must be in [1, K/64]");
  if (k_splits > 1) {
    TORCH_CHECK(epi == b200::kEpiF32 && groups == 1, "split-K: single group, fp32 partials only");
    TORCH_CHECK(out.is_contiguous() && out.numel() >= k_splits * split_stride &&
                split_stride >= x.size(0) * out.stride(0), "split-K partial buffer too small");
  }
  if (pair) TORCH_CHECK(pair_row_offset + m_tiles * 128 <= rows_per_group, "pair rows out of range");
  if (x.size(0) == 0) return;

  c10::cuda::CUDAGuard guard(x.device());
  b200::GemmLaunch L{};
  L.args.a_scale = fp8 ? weight_scale->data_ptr<float>() : nullptr;
  L.args.a_rows_per_group = (int)rows_per_group;
  L.args.m_tiles = (int)m_tiles;
  L.args.k_stages = (int)(K / 64);
  L.args.scale_m_blocks = (int)(rows_per_group / 128);
  L.args.scale_k_blocks = (int)(K / 128);
  L.args.num_groups = (int)groups;
  L.args.group_count = group_count.data_ptr<int>();
  L.args.group_offset = group_offset.has_value() ? group_offset->data_ptr<int>() : nullptr;
  L.args.pair_row_offset = (int)pair_row_offset;
  L.args.out = out.data_ptr();
  L.args.ld_out = (int)out.stride(0);
  L.args.out_group_stride = (int)out_group_stride;
  L.args.slot_of_row = ptr_or_null<int>(slot_of_row);
  L.args.slot_weight = ptr_or_null<float>(slot_weight);
  L.args.status = status.data_ptr<int>();
  L.args.k_splits = (int)k_splits;
  L.args.split_stride = split_stride;
  L.args.a_tiled = a_tiled ? 1 : 0;
  L.args.a_base = weight.data_ptr();
  if (trace.has_value()) {
    TORCH_CHECK(trace->scalar_type() == torch::kInt64 && trace->is_contiguous(), "trace must be int64");
    L.args.trace = reinterpret_cast<unsigned long long*>(trace->data_ptr());
    L.args.trace_cap = (int)((trace->numel() - 1) / 10);
  }
  if (!release.empty()) {
    // [epoch ptr, CTA counter ptr, rank, epoch add, flag ptr of each rank...]: the last
    // CTA releases *epoch + add into flags[r][rank] for every r (device pointers)
    TORCH_CHECK(release.size() >= 5 && release.size() <= 4 + 8, "release: epoch, counter, rank, add, 1..8 flags");
    L.args.ep_epoch = reinterpret_cast<const uint32_t*>(release[0]);
    L.args.ep_cta_done = reinterpret_cast<int*>(release[1]);
    L.args.ep_rank = (int)release[2];
    L.args.ep_epoch_add = (int)release[3];
    L.args.ep_world = (int)release.size() - 4;
    for (int r = 0; r < L.args.ep_world; ++r) L.args.ep_done[r] = reinterpret_cast<void*>(release[4 + r]);
  }
  L.a = weight.data_ptr();
  L.a_row_stride_bytes = K * weight.element_size();
  L.b = x.data_ptr();
  L.b_rows = x.size(0);
  L.b_row_stride_bytes = x.stride(0) * 2;
  L.K = (int)K;
  L.bn = (int)bn;
  L.a_fp8 = fp8;
  L.pair = pair;
  L.epi = (int)epi;
  b200::gemm_tc_launch(L, stream());
}

// Down GEMM whose epilogue writes each weighted row into its source rank's
// slot buffer (peer memory): slot_code = rank * slot_cap + slot.
void gemm_peer_scatter(Tensor weight, c10::optional<Tensor> weight_scale, Tensor x, Tensor group_count,
                       Tensor group_offset, int64_t bn, Tensor slot_code, Tensor slot_w, std::vector<int64_t> peer_ptrs,
                       int64_t slot_cap, int64_t ld_out, Tensor status, bool a_tiled, c10::optional<Tensor> ep_epoch,
                       c10::optional<Tensor> ep_cta_done, std::vector<int64_t> done_ptrs, int64_t ep_rank) {
  CHECK_CUDA(weight); CHECK_CUDA(x); CHECK_CONTIG(weight);
  // e4m3 + 128x128 scales (dequantised per tile), or bf16 (a resident dequantised copy)
  const bool fp8 = weight.scalar_type() == torch::kFloat8_e4m3fn;
  TORCH_CHECK(weight.dim() == 3 && (fp8 || weight.scalar_type() == torch::kBFloat16),
              "expert weights must be [E, N, K] e4m3 or bf16");
  TORCH_CHECK(fp8 == weight_scale.has_value(), "e4m3 weights need their scales; bf16 weights take none");
  TORCH_CHECK(fp8 || !a_tiled, "bf16 weights are row-major");
  TORCH_CHECK(x.dim() == 2 && x.stride(1) == 1 && x.scalar_type() == torch::kBFloat16, "x must be [rows, K] bf16");
  TORCH_CHECK(peer_ptrs.size() >= 1 && peer_ptrs.size() <= 8, "1..8 peer pointers");
  CHECK_DT(slot_code, torch::kInt32); CHECK_DT(slot_w, torch::kFloat32);
  const int64_t groups = weight.size(0), N = weight.size(1), K = weight.size(2);
  TORCH_CHECK(x.size(1) == K, "K mismatch");
  if (fp8) TORCH_CHECK(weight_scale->numel() == groups * (N / 128) * (K / 128), "weight_scale shape");
  TORCH_CHECK(x.size(0) > 0, "gemm_peer_scatter: x needs at least one row (the grid releases the done epoch)");
  c10::cuda::CUDAGuard guard(x.device());
  b200::GemmLaunch L{};
  L.args.a_scale = fp8 ? weight_scale->data_ptr<float>() : nullptr;
  L.args.a_rows_per_group = (int)N;
  L.args.m_tiles = (int)(N / 128);
  L.args.k_stages = (int)(K / 64);
  L.args.scale_m_blocks = (int)(N / 128);
  L.args.scale_k_blocks = (int)(K / 128);
  L.args.num_groups = (int)groups;
  L.args.group_count = group_count.data_ptr<int>();
  L.args.group_offset = group_offset.data_ptr<int>();
  L.args.out = nullptr;
  L.args.ld_out = (int)ld_out;
  L.args.slot_of_row = slot_code.data_ptr<int>();
  L.args.slot_weight = slot_w.data_ptr<float>();
  L.args.status = status.data_ptr<int>();
  L.args.peer_scatter = 1;
  L.args.a_tiled = a_tiled ? 1 : 0;
  L.args.a_base = weight.data_ptr();
  L.args.slot_cap = (int)slot_cap;
  for (size_t i = 0; i < peer_ptrs.size(); ++i) L.args.peer_out[i] = reinterpret_cast<void*>(peer_ptrs[i]);
  if (ep_epoch.has_value()) {  // the last CTA releases this rank's done epoch to every source
    TORCH_CHECK(ep_cta_done.has_value() && done_ptrs.size() == peer_ptrs.size(), "done release arguments");
    CHECK_DT((*ep_cta_done), torch::kInt32);
    L.args.ep_epoch = reinterpret_cast<const uint32_t*>(ep_epoch->data_ptr());
    L.args.ep_cta_done = ep_cta_done->data_ptr<int>();
    for (size_t i = 0; i < done_ptrs.size(); ++i) L.args.ep_done[i] = reinterpret_cast<void*>(done_ptrs[i]);
    L.args.ep_rank = (int)ep_rank;
    L.args.ep_world = (int)done_ptrs.size();
  }
  L.a = weight.data_ptr();
  L.a_row_stride_bytes = fp8 ? K : K * 2;
  L.b = x.data_ptr();
  L.b_rows = x.size(0);
  L.b_row_stride_bytes = x.stride(0) * 2;
  L.K = (int)K;
  L.bn = (int)bn;
  L.a_fp8 = fp8;
  L.pair = false;
  L.epi = b200::kEpiScatter;
  b200::gemm_tc_launch(L, stream());
}

b200::EpArgs ep_args(std::vector<int64_t> dims, Tensor owner, Tensor g2l, Tensor ge_local, Tensor send_cursor,
                     Tensor ecur, Tensor done_blocks, Tensor epoch, Tensor status, Tensor wait_ns,
                     std::vector<int64_t> recv_x, std::vector<int64_t> recv_meta,
                     std::vector<int64_t> counts, std::vector<int64_t> flags, std::vector<int64_t> done) {
  TORCH_CHECK(dims.size() == 7, "dims = (world, rank, hidden, cap, slot_cap, num_local, num_experts)");
  b200::EpArgs a{};
  a.world = (int)dims[0];
  a.rank = (int)dims[1];
  a.hidden = (int)dims[2];
  a.cap = (int)dims[3];
  a.slot_cap = (int)dims[4];
  a.num_local = (int)dims[5];
  a.num_experts = (int)dims[6];
  TORCH_CHECK(a.num_local >= 1 && a.num_local <= b200::kEpMaxLocalExperts && a.num_experts >= a.num_local,
              "bad expert counts");
  CHECK_DT(ge_local, torch::kInt32); CHECK_DT(ecur, torch::kInt32);
  TORCH_CHECK(owner.numel() >= a.num_experts && g2l.numel() >= a.num_experts && ge_local.numel() >= a.num_experts &&
              ecur.numel() >= a.num_experts, "per-expert tables must hold num_experts entries");
  TORCH_CHECK(a.world >= 1 && a.world <= b200::kEpMaxWorld && a.rank >= 0 && a.rank < a.world, "bad world/rank");
  TORCH_CHECK((int)recv_x.size() == a.world && (int)recv_meta.size() == a.world && (int)counts.size() == a.world &&
              (int)flags.size() == a.world && (int)done.size() == a.world, "one pointer per rank");
  CHECK_DT(owner, torch::kInt32); CHECK_DT(g2l, torch::kInt32); CHECK_DT(send_cursor, torch::kInt32);
  CHECK_DT(done_blocks, torch::kInt32); CHECK_DT(status, torch::kInt32);
  a.owner = owner.data_ptr<int>();
  a.g2l = g2l.data_ptr<int>();
  a.ge_local = ge_local.data_ptr<int>();
  a.send_cursor = send_cursor.data_ptr<int>();
  a.ecur = ecur.data_ptr<int>();
  a.done_blocks = done_blocks.data_ptr<int>();
  a.epoch = reinterpret_cast<uint32_t*>(epoch.data_ptr());
  a.status = status.data_ptr<int>();
  TORCH_CHECK(wait_ns.scalar_type() == torch::kInt64 && wait_ns.numel() >= 2 * a.world && wait_ns.is_contiguous(),
              "wait_ns: int64 [2 * world]");
  a.wait_ns = reinterpret_cast<unsigned long long*>(wait_ns.data_ptr<int64_t>());
  for (int r = 0; r < a.world; ++r) {
    a.recv_x[r] = reinterpret_cast<void*>(recv_x[r]);
    a.recv_meta[r] = reinterpret_cast<void*>(recv_meta[r]);
    a.counts[r] = reinterpret_cast<void*>(counts[r]);
    a.flags[r] = reinterpret_cast<void*>(flags[r]);
    a.done[r] = reinterpret_cast<void*>(done[r]);
  }
  return a;
}

#define EP_ARGS_DECL std::vector<int64_t> dims, Tensor owner, Tensor g2l, Tensor ge_local, Tensor send_cursor, \
  Tensor ecur, Tensor done_blocks, Tensor epoch, Tensor status, Tensor wait_ns, std::vector<int64_t> recv_x, \
  std::vector<int64_t> recv_meta, \
  std::vector<int64_t> counts, std::vector<int64_t> flags, std::vector<int64_t> done
#define EP_ARGS ep_args(dims, owner, g2l, ge_local, send_cursor, ecur, done_blocks, epoch, status, wait_ns, recv_x, \
                        recv_meta, counts, flags, done)

void ep_dispatch(EP_ARGS_DECL, Tensor x, Tensor ids, Tensor w) {
  CHECK_CUDA(x); CHECK_CONTIG(x); CHECK_DT(x, torch::kBFloat16); CHECK_DT(ids, torch::kInt32);
  CHECK_DT(w, torch::kFloat32); CHECK_CONTIG(ids); CHECK_CONTIG(w);
  auto a = EP_ARGS;
  TORCH_CHECK(x.size(1) == a.hidden, "hidden mismatch");
  b200::ep_dispatch(a, x.data_ptr(), ids.data_ptr<int>(), w.data_ptr<float>(), (int)x.size(0), (int)ids.size(1),
                    stream());
}

void ep_scatter(EP_ARGS_DECL, Tensor local_counts, Tensor x_perm, Tensor slot_code, Tensor slot_w,
                Tensor offsets_out) {
  CHECK_CONTIG(x_perm); CHECK_DT(slot_code, torch::kInt32); CHECK_DT(slot_w, torch::kFloat32);
  CHECK_DT(local_counts, torch::kInt32); CHECK_DT(offsets_out, torch::kInt32);
  auto a = EP_ARGS;
  TORCH_CHECK(x_perm.size(0) >= (int64_t)a.world * a.cap, "x_perm must hold world * cap rows");
  TORCH_CHECK(slot_code.numel() >= (int64_t)a.world * a.cap && slot_w.numel() >= (int64_t)a.world * a.cap,
              "slot_code / slot_w must hold world * cap rows");
  TORCH_CHECK(local_counts.numel() >= a.num_local && offsets_out.numel() >= a.num_local + 1,
              "local_counts [El], offsets_out [El + 1]");
  b200::ep_scatter(a, local_counts.data_ptr<int>(), x_perm.data_ptr(), slot_code.data_ptr<int>(),
                   slot_w.data_ptr<float>(), offsets_out.data_ptr<int>(), a.world * a.cap, stream());
}

void ep_signal(EP_ARGS_DECL) { b200::ep_signal(EP_ARGS, stream()); }
void ep_wait_done(EP_ARGS_DECL) { b200::ep_wait_done(EP_ARGS, stream()); }

// Tensor-parallel all-reduce over peer memory.  dims = (world, rank, splits, split_stride);
// part_ptrs / flag_ptrs hold every rank's partial buffer and flag array (device pointers).
b200::TpArgs tp_args(std::vector<int64_t> dims, std::vector<int64_t> part_ptrs, std::vector<int64_t> flag_ptrs,
                     Tensor epoch, Tensor counter, Tensor status, c10::optional<Tensor> wait_ns) {
  TORCH_CHECK(dims.size() == 4, "dims = (world, rank, splits, split_stride)");
  b200::TpArgs a{};
  a.world = (int)dims[0];
  a.rank = (int)dims[1];
  a.splits = (int)dims[2];
  a.split_stride = dims[3];
  TORCH_CHECK(a.world >= 1 && a.world <= b200::kTpMaxWorld && (int)part_ptrs.size() == a.world &&
              (int)flag_ptrs.size() == a.world, "one partial buffer and one flag array per rank");
  for (int r = 0; r < a.world; ++r) {
    a.part[r] = reinterpret_cast<const float*>(part_ptrs[r]);
    a.flags[r] = reinterpret_cast<uint32_t*>(flag_ptrs[r]);
  }
  CHECK_DT(counter, torch::kInt32); CHECK_DT(status, torch::kInt32);
  a.epoch = reinterpret_cast<uint32_t*>(epoch.data_ptr());
  a.counter = counter.data_ptr<int>();
  a.status = status.data_ptr<int>();
  if (wait_ns.has_value()) {
    TORCH_CHECK(wait_ns->scalar_type() == torch::kInt64 && wait_ns->numel() >= a.world, "wait_ns [world] int64");
    a.wait_ns = reinterpret_cast<unsigned long long*>(wait_ns->data_ptr<int64_t>());
  }
  return a;
}

void tp_slots_partial(std::vector<int64_t> dims, std::vector<int64_t> part_ptrs, std::vector<int64_t> flag_ptrs,
                      Tensor epoch, Tensor counter, Tensor status, c10::optional<Tensor> wait_ns, Tensor slots,
                      int64_t topk, int64_t T, int64_t H, int64_t part_rows) {
  CHECK_CUDA(slots); CHECK_CONTIG(slots); CHECK_DT(slots, torch::kBFloat16);
  TORCH_CHECK(slots.numel() >= T * topk * H, "slots too small");
  TORCH_CHECK(T <= part_rows, "partial buffer holds fewer rows than the batch");
  auto a = tp_args(dims, part_ptrs, flag_ptrs, epoch, counter, status, wait_ns);
  TORCH_CHECK(a.splits == 1, "slot partials are a single split");
  b200::tp_slots_partial(a, slots.data_ptr(), (int)topk, (int)T, (int)H, stream());
}

void tp_allreduce_rmsnorm(std::vector<int64_t> dims, std::vector<int64_t> part_ptrs, std::vector<int64_t> flag_ptrs,
                          Tensor epoch, Tensor counter, Tensor status, c10::optional<Tensor> wait_ns, Tensor residual,
                          Tensor weight, Tensor out, double eps, int64_t part_rows) {
  CHECK_CUDA(residual); CHECK_CONTIG(residual); CHECK_CONTIG(out);
  CHECK_DT(residual, torch::kBFloat16); CHECK_DT(weight, torch::kBFloat16); CHECK_DT(out, torch::kBFloat16);
  const int T = (int)residual.size(0), H = (int)residual.size(1);
  TORCH_CHECK(T <= part_rows, "partial buffer holds fewer rows than the batch");
  auto a = tp_args(dims, part_ptrs, flag_ptrs, epoch, counter, status, wait_ns);
  TORCH_CHECK(a.split_stride >= (int64_t)T * H, "split stride below one partial");
  b200::tp_allreduce_rmsnorm(a, residual.data_ptr(), weight.data_ptr(), out.data_ptr(), T, H, (float)eps, stream());
}

void embed(Tensor ids, Tensor table, Tensor out, Tensor status, c10::optional<Tensor> feed_src,
           c10::optional<Tensor> feed_tokens) {
  CHECK_CUDA(ids); CHECK_CUDA(table); CHECK_CUDA(out);
  CHECK_DT(ids, torch::kInt32); CHECK_DT(table, torch::kBFloat16); CHECK_DT(out, torch::kBFloat16);
  CHECK_CONTIG(table); CHECK_CONTIG(out); CHECK_CONTIG(ids);
  TORCH_CHECK(out.size(0) == ids.numel() && out.size(1) == table.size(1), "embed shape mismatch");
  TORCH_CHECK(feed_src.has_value() == feed_tokens.has_value(), "feed needs both the source rows and the tokens");
  if (feed_src.has_value()) {
    CHECK_DT((*feed_src), torch::kInt32); CHECK_DT((*feed_tokens), torch::kInt32);
    TORCH_CHECK(feed_src->numel() >= ids.numel(), "feed_src too short");
  }
  b200::embed_gather(ids.data_ptr<int>(), table.data_ptr(), out.data_ptr(), (int)ids.numel(), (int)table.size(1),
                     (int)table.size(0), status.data_ptr<int>(), stream(), ptr_or_null<int>(feed_src),
                     ptr_or_null<int>(feed_tokens));
}

void rmsnorm(Tensor x, c10::optional<Tensor> residual_in, Tensor weight, Tensor out,
             c10::optional<Tensor> residual_out, double eps) {
  CHECK_CUDA(x); CHECK_CONTIG(x); CHECK_CONTIG(out); CHECK_DT(x, torch::kBFloat16);
  CHECK_DT(weight, torch::kBFloat16); CHECK_DT(out, torch::kBFloat16);
  TORCH_CHECK(residual_in.has_value() == residual_out.has_value(), "residual in/out go together");
  const int H = (int)x.size(-1);
  const int T = (int)(x.numel() / H);
  TORCH_CHECK(out.numel() == x.numel() && weight.numel() == H, "rmsnorm shape mismatch");
  if (residual_in.has_value()) {
    CHECK_CONTIG((*residual_in));
    TORCH_CHECK(residual_in->numel() == x.numel(), "residual shape mismatch");
  }
  b200::rmsnorm(x.data_ptr(), residual_in.has_value() ? residual_in->data_ptr() : nullptr, weight.data_ptr(),
                out.data_ptr(), residual_out.has_value() ? residual_out->data_ptr() : nullptr, T, H, (float)eps,
                stream());
}

void moe_combine(Tensor slots, int64_t topk, Tensor residual, Tensor weight, Tensor out, double eps,
                 c10::optional<Tensor> zero, c10::optional<Tensor> wait_flags, c10::optional<Tensor> wait_epoch,
                 c10::optional<Tensor> wait_status, c10::optional<Tensor> wait_ns) {
  CHECK_CUDA(slots); CHECK_CONTIG(slots); CHECK_CONTIG(residual); CHECK_CONTIG(out);
  CHECK_DT(slots, torch::kBFloat16); CHECK_DT(residual, torch::kBFloat16);
  const int H = (int)residual.size(-1);
  const int T = (int)residual.size(0);
  TORCH_CHECK(slots.numel() >= (int64_t)T * topk * H, "slots too small");
  int* zp = nullptr;
  int zn = 0;
  if (zero.has_value()) {
    CHECK_DT((*zero), torch::kInt32); CHECK_CONTIG((*zero));
    zp = zero->data_ptr<int>();
    zn = (int)zero->numel();
  }
  b200::CombineWait cw;
  if (wait_flags.has_value()) {  // expert parallel: wait for every owner's done epoch first
    TORCH_CHECK(wait_epoch.has_value() && wait_status.has_value(), "wait needs epoch and status");
    CHECK_DT((*wait_flags), torch::kInt32); CHECK_DT((*wait_status), torch::kInt32);
    cw.flags = reinterpret_cast<const uint32_t*>(wait_flags->data_ptr<int>());
    cw.epoch = reinterpret_cast<const uint32_t*>(wait_epoch->data_ptr());
    cw.world = (int)wait_flags->numel();
    cw.status = wait_status->data_ptr<int>();
    if (wait_ns.has_value()) {
      TORCH_CHECK(wait_ns->scalar_type() == torch::kInt64 && wait_ns->numel() >= 2 * cw.world, "wait_ns [2 * world]");
      cw.wait_ns = reinterpret_cast<unsigned long long*>(wait_ns->data_ptr<int64_t>());
    }
  }
  b200::moe_combine_add_rmsnorm(slots.data_ptr(), (int)topk, residual.data_ptr(), weight.data_ptr(),
                                out.data_ptr(), T, H, (float)eps, stream(), zp, zn, cw);
}

void qknorm_rope_kvstore(Tensor qkv, Tensor positions, Tensor slot_mapping, Tensor q_norm_w, Tensor k_norm_w,
                         Tensor cos_sin, Tensor k_cache, Tensor v_cache, c10::optional<Tensor> k_scale,
                         c10::optional<Tensor> v_scale, Tensor q_out, int64_t num_q_heads, int64_t num_kv_heads,
                         int64_t head_dim, int64_t block_size, int64_t block_stride, int64_t scale_block_stride,
                         double eps, c10::optional<Tensor> part, int64_t splits, std::vector<int64_t> chan) {
  CHECK_CUDA(qkv); CHECK_DT(qkv, torch::kBFloat16); CHECK_DT(positions, torch::kInt32);
  CHECK_DT(slot_mapping, torch::kInt32); CHECK_DT(cos_sin, torch::kFloat32); CHECK_CONTIG(q_out);
  TORCH_CHECK(qkv.stride(1) == 1, "qkv inner stride must be 1");
  const int T = (int)qkv.size(0);
  TORCH_CHECK(positions.numel() >= T && slot_mapping.numel() >= T, "positions/slot_mapping too short");
  TORCH_CHECK(qkv.size(1) == (num_q_heads + 2 * num_kv_heads) * head_dim, "qkv width mismatch");
  b200::QkvArgs a{};
  a.qkv = qkv.data_ptr();
  a.qkv_stride = (int)qkv.stride(0);
  a.positions = positions.data_ptr<int>();
  a.slot_mapping = slot_mapping.data_ptr<int>();
  a.q_norm_w = q_norm_w.data_ptr();
  a.k_norm_w = k_norm_w.data_ptr();
  a.cos_sin = cos_sin.data_ptr<float>();
  a.k_cache = k_cache.data_ptr();
  a.v_cache = v_cache.data_ptr();
  a.kv_int8 = k_cache.scalar_type() == torch::kInt8;
  a.k_scale = ptr_or_null<float>(k_scale);
  a.v_scale = ptr_or_null<float>(v_scale);
  if (a.kv_int8 && chan.empty()) TORCH_CHECK(a.k_scale && a.v_scale, "int8 KV needs scale pools");
  a.block_size = (int)block_size;
  a.block_stride = block_stride;
  a.scale_block_stride = scale_block_stride;
  a.q_out = q_out.data_ptr();
  a.num_q_heads = (int)num_q_heads;
  a.num_kv_heads = (int)num_kv_heads;
  a.head_dim = (int)head_dim;
  a.eps = (float)eps;
  if (part.has_value()) {
    CHECK_DT((*part), torch::kFloat32); CHECK_CONTIG((*part));
    TORCH_CHECK(splits >= 1 && part->numel() >= splits * (int64_t)T * qkv.stride(0),
                "qkv partials must hold splits x T x qkv width floats");
    a.part = part->data_ptr<float>();
    a.splits = (int)splits;
    a.part_stride = (int64_t)T * qkv.stride(0);
  }
  if (!chan.empty()) {
    // int8 channel mode: [scale, out_idx, n_out, side_k, side_v, side_block_stride, calib_amax, calib_sum]
    TORCH_CHECK(chan.size() == 8 && a.kv_int8, "channel mode: 8 entries and an int8 pool");
    a.kv_int8 = 2;
    a.ch_scale = reinterpret_cast<const float*>(chan[0]);
    a.out_idx = reinterpret_cast<const int*>(chan[1]);
    a.n_out = reinterpret_cast<const int*>(chan[2]);
    a.side_k = reinterpret_cast<void*>(chan[3]);
    a.side_v = reinterpret_cast<void*>(chan[4]);
    a.side_block_stride = chan[5];
    a.calib_amax = reinterpret_cast<float*>(chan[6]);
    a.calib_sum = reinterpret_cast<float*>(chan[7]);
    TORCH_CHECK(a.ch_scale && a.out_idx && a.n_out && a.side_k && a.side_v, "channel mode pointers");
  }
  b200::qknorm_rope_kvstore(a, T, stream());
}

void router_topk(Tensor logits, int64_t num_experts, int64_t topk, bool renorm, Tensor ids, Tensor weights,
                 c10::optional<Tensor> counts) {
  CHECK_CUDA(logits); CHECK_DT(logits, torch::kFloat32);
  TORCH_CHECK(logits.stride(1) == 1 && logits.size(1) >= num_experts, "router logits layout");
  CHECK_DT(ids, torch::kInt32); CHECK_DT(weights, torch::kFloat32); CHECK_CONTIG(ids); CHECK_CONTIG(weights);
  TORCH_CHECK(ids.numel() >= logits.size(0) * topk, "ids too small");
  b200::router_topk(logits.data_ptr<float>(), (int)logits.stride(0), (int)logits.size(0), (int)num_experts,
                    (int)topk, renorm, ids.data_ptr<int>(), weights.data_ptr<float>(), ptr_or_null<int>(counts),
                    stream());
}

// ---------------------------------------------------------------- CUDA IPC
// Expert-parallel peer buffers: one cudaMalloc per buffer, shared with the
// other ranks through cudaIpcGetMemHandle and mapped on the caller's device
// with cudaIpcOpenMemHandle (peer access enabled lazily).  These are plain
// NVLink peer mappings: no multicast object is created, and nothing but this
// extension's own ld/st kernels ever reads them.
#define IPC_CHECK(x)                                                                    \
  do {                                                                                  \
    cudaError_t e_ = (x);                                                               \
    TORCH_CHECK(e_ == cudaSuccess, #x " failed: ", cudaGetErrorString(e_));              \
  } while (0)

std::tuple<int64_t, Tensor> ipc_alloc(int64_t nbytes, int64_t device) {
  TORCH_CHECK(nbytes > 0, "ipc_alloc: size must be positive");
  c10::cuda::CUDAGuard guard((c10::DeviceIndex)device);
  void* p = nullptr;
  IPC_CHECK(cudaMalloc(&p, (size_t)nbytes));
  IPC_CHECK(cudaMemset(p, 0, (size_t)nbytes));
  cudaIpcMemHandle_t h;
  IPC_CHECK(cudaIpcGetMemHandle(&h, p));
  Tensor ht = torch::empty({(int64_t)sizeof(h)}, torch::kUInt8);
  std::memcpy(ht.data_ptr(), &h, sizeof(h));
  return {reinterpret_cast<int64_t>(p), ht};
}

// IPC handle of the cudaMalloc allocation that contains `ptr` (allocators hand out
// pieces of larger segments): returns (handle bytes, offset of ptr in the allocation).
std::tuple<Tensor, int64_t> ipc_export(int64_t ptr, int64_t device) {
  c10::cuda::CUDAGuard guard((c10::DeviceIndex)device);
  using RangeFn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);
  static RangeFn range = nullptr;
  if (range == nullptr) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    IPC_CHECK(cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q));
    TORCH_CHECK(q == cudaDriverEntryPointSuccess && p != nullptr, "cuMemGetAddressRange not available");
    range = reinterpret_cast<RangeFn>(p);
  }
  CUdeviceptr base = 0;
  size_t size = 0;
  TORCH_CHECK(range(&base, &size, (CUdeviceptr)ptr) == CUDA_SUCCESS, "ipc_export: pointer is not device memory");
  cudaIpcMemHandle_t h;
  IPC_CHECK(cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)));
  Tensor ht = torch::empty({(int64_t)sizeof(h)}, torch::kUInt8);
  std::memcpy(ht.data_ptr(), &h, sizeof(h));
  return {ht, (int64_t)(ptr - (int64_t)base)};
}

int64_t ipc_open(Tensor handle, int64_t device) {
  TORCH_CHECK(handle.numel() == (int64_t)sizeof(cudaIpcMemHandle_t) && handle.scalar_type() == torch::kUInt8,
              "ipc_open: expected a 64-byte handle");
  c10::cuda::CUDAGuard guard((c10::DeviceIndex)device);
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle.contiguous().data_ptr(), sizeof(h));
  void* p = nullptr;
  IPC_CHECK(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
  return reinterpret_cast<int64_t>(p);
}

void ipc_close(int64_t ptr, int64_t device) {
  c10::cuda::CUDAGuard guard((c10::DeviceIndex)device);
  IPC_CHECK(cudaIpcCloseMemHandle(reinterpret_cast<void*>(ptr)));
}

void ipc_free(int64_t ptr, int64_t device) {
  c10::cuda::CUDAGuard guard((c10::DeviceIndex)device);
  IPC_CHECK(cudaFree(reinterpret_cast<void*>(ptr)));
}

// A tensor view of device memory this module owns (no deleter: ipc_free releases it).
Tensor tensor_from_ptr(int64_t ptr, std::vector<int64_t> shape, c10::ScalarType dtype, int64_t device) {
  auto opts = torch::TensorOptions().dtype(dtype).device(torch::kCUDA, (c10::DeviceIndex)device);
  return torch::from_blob(reinterpret_cast<void*>(ptr), shape, opts);
}

void kv_blocks_copy(Tensor src_pool, Tensor src_ids, int64_t dst_ptr, Tensor dst_ids, int64_t block_bytes) {
  CHECK_CUDA(src_pool); CHECK_CONTIG(src_pool);
  CHECK_DT(src_ids, torch::kInt32); CHECK_DT(dst_ids, torch::kInt32); CHECK_CONTIG(src_ids); CHECK_CONTIG(dst_ids);
  TORCH_CHECK(src_ids.numel() == dst_ids.numel(), "kv_blocks_copy: id lists differ in length");
  TORCH_CHECK(src_pool.numel() * src_pool.element_size() % block_bytes == 0, "kv_blocks_copy: pool / block size");
  c10::cuda::CUDAGuard guard(src_pool.device());
  b200::kv_blocks_copy(src_pool.data_ptr(), src_ids.data_ptr<int>(), reinterpret_cast<void*>(dst_ptr),
                       dst_ids.data_ptr<int>(), (int)src_ids.numel(), block_bytes, stream());
}

void dequant_weights(Tensor q, Tensor scale, Tensor out, bool tiled) {
  CHECK_CUDA(q); CHECK_CONTIG(q); CHECK_CONTIG(scale); CHECK_CONTIG(out);
  TORCH_CHECK(q.scalar_type() == torch::kFloat8_e4m3fn, "weights must be e4m3");
  CHECK_DT(scale, torch::kFloat32); CHECK_DT(out, torch::kBFloat16);
  TORCH_CHECK(q.sizes() == out.sizes(), "out must have the weight's shape");
  const int64_t K = q.size(-1), N = q.size(-2), G = q.numel() / (N * K);
  TORCH_CHECK(scale.numel() == G * (N / 128) * (K / 128), "scale must be [G, N/128, K/128]");
  c10::cuda::CUDAGuard guard(q.device());
  b200::dequant_weights(q.data_ptr(), scale.data_ptr<float>(), out.data_ptr(), (int)G, (int)N, (int)K, tiled, stream());
}

static void router_impl(Tensor x, Tensor w, int64_t num_experts, int64_t topk, bool renorm, Tensor ids,
                        Tensor weights, c10::optional<Tensor> counts, c10::optional<Tensor> status,
                        c10::optional<Tensor> part, c10::optional<Tensor> tile_cnt, const b200::EpArgs* ep) {
  CHECK_CUDA(x); CHECK_CONTIG(x); CHECK_DT(x, torch::kBFloat16);
  CHECK_CONTIG(w); CHECK_DT(w, torch::kBFloat16);
  CHECK_DT(ids, torch::kInt32); CHECK_DT(weights, torch::kFloat32);
  TORCH_CHECK(x.size(1) == w.size(1) && w.size(0) >= num_experts, "router shapes");
  TORCH_CHECK(ids.numel() >= x.size(0) * topk && weights.numel() >= x.size(0) * topk, "router outputs too small");
  // the split-K scratch is used only when there is a counter for every token tile
  float* pp = nullptr;
  int* cp = nullptr;
  int part_tiles = 0;
  if (part.has_value()) {
    TORCH_CHECK(tile_cnt.has_value(), "router scratch needs the tile counters");
    CHECK_DT((*part), torch::kFloat32); CHECK_DT((*tile_cnt), torch::kInt32);
    if (tile_cnt->numel() >= (x.size(0) + 15) / 16) {
      pp = part->data_ptr<float>();
      cp = tile_cnt->data_ptr<int>();
      part_tiles = (int)(part->numel() / (16 * 128));
    }
  }
  b200::router_fused(x.data_ptr(), w.data_ptr(), (int)x.size(0), (int)x.size(1), (int)num_experts, (int)w.size(0),
                     (int)topk, renorm, ids.data_ptr<int>(), weights.data_ptr<float>(), ptr_or_null<int>(counts),
                     ptr_or_null<int>(status), stream(), pp, cp, part_tiles, ep);
}

void router_fused(Tensor x, Tensor w, int64_t num_experts, int64_t topk, bool renorm, Tensor ids, Tensor weights,
                  c10::optional<Tensor> counts, c10::optional<Tensor> status, c10::optional<Tensor> part,
                  c10::optional<Tensor> tile_cnt) {
  router_impl(x, w, num_experts, topk, renorm, ids, weights, counts, status, part, tile_cnt, nullptr);
}

// Router + expert-parallel dispatch in one launch (the top-k warps send the rows).
void router_dispatch(EP_ARGS_DECL, Tensor x, Tensor w, int64_t num_experts, int64_t topk, bool renorm, Tensor ids,
                     Tensor weights, c10::optional<Tensor> part, c10::optional<Tensor> tile_cnt) {
  auto a = EP_ARGS;
  TORCH_CHECK(x.size(1) == a.hidden, "hidden mismatch");
  router_impl(x, w, num_experts, topk, renorm, ids, weights, c10::nullopt, status, part, tile_cnt, &a);
}

// residual += bf16(sum of split-K partials); out = rmsnorm(residual) * weight
void rmsnorm_partials(Tensor part, int64_t splits, Tensor residual, Tensor weight, Tensor out, double eps) {
  CHECK_CUDA(part); CHECK_CONTIG(part); CHECK_DT(part, torch::kFloat32);
  CHECK_CONTIG(residual); CHECK_CONTIG(out); CHECK_DT(residual, torch::kBFloat16); CHECK_DT(out, torch::kBFloat16);
  const int H = (int)residual.size(-1);
  const int T = (int)(residual.numel() / H);
  TORCH_CHECK(part.numel() >= splits * (int64_t)T * H && weight.numel() == H && out.numel() == residual.numel(),
              "rmsnorm_partials shapes");
  b200::rmsnorm(nullptr, residual.data_ptr(), weight.data_ptr(), out.data_ptr(), residual.data_ptr(), T, H, (float)eps,
                stream(), part.data_ptr<float>(), (int)splits);
}

void splitk_reduce(Tensor part, int64_t splits, Tensor out) {
  CHECK_CUDA(part); CHECK_CONTIG(part); CHECK_DT(part, torch::kFloat32);
  TORCH_CHECK(out.dim() == 2 && out.stride(1) == 1, "out must be [T, N] with unit inner stride");
  const int64_t T = out.size(0), N = out.size(1);
  TORCH_CHECK(part.numel() >= splits * T * N, "partials too small");
  TORCH_CHECK(out.scalar_type() == torch::kBFloat16 || out.scalar_type() == torch::kFloat32, "out bf16 or fp32");
  b200::splitk_reduce(part.data_ptr<float>(), (int)splits, (int)T, (int)N, out.data_ptr(), (int)out.stride(0),
                      out.scalar_type() == torch::kBFloat16, stream());
}

void moe_permute(Tensor x, Tensor ids, Tensor counts, Tensor cursor, Tensor x_perm, Tensor slot_of_row,
                 c10::optional<Tensor> offsets_out) {
  CHECK_CUDA(x); CHECK_CONTIG(x); CHECK_CONTIG(x_perm); CHECK_DT(ids, torch::kInt32); CHECK_CONTIG(ids);
  CHECK_DT(counts, torch::kInt32); CHECK_DT(cursor, torch::kInt32); CHECK_DT(slot_of_row, torch::kInt32);
  const int T = (int)x.size(0), H = (int)x.size(1), topk = (int)ids.size(1), E = (int)counts.numel();
  TORCH_CHECK(ids.size(0) == T, "ids rows mismatch");
  TORCH_CHECK(x_perm.size(0) >= (int64_t)T * topk && slot_of_row.numel() >= (int64_t)T * topk, "x_perm too small");
  b200::moe_permute(x.data_ptr(), ids.data_ptr<int>(), T, topk, E, H, counts.data_ptr<int>(), cursor.data_ptr<int>(),
                    x_perm.data_ptr(), slot_of_row.data_ptr<int>(), ptr_or_null<int>(offsets_out), stream());
}

// int8 channel mode of the attention kernels: [dscale, out_idx, n_out, side_k, side_v, side_block_stride]
static void set_kv_channel(int* kv_int8, b200::KvChannel* ch, const std::vector<int64_t>& chan) {
  if (chan.empty()) return;
  TORCH_CHECK(chan.size() == 6 && *kv_int8, "channel mode: 6 entries and an int8 pool");
  *kv_int8 = 2;
  ch->dscale = reinterpret_cast<const float*>(chan[0]);
  ch->out_idx = reinterpret_cast<const int*>(chan[1]);
  ch->n_out = reinterpret_cast<const int*>(chan[2]);
  ch->side_k = reinterpret_cast<const void*>(chan[3]);
  ch->side_v = reinterpret_cast<const void*>(chan[4]);
  ch->side_block_stride = chan[5];
}

void decode_attn(Tensor q, Tensor k_cache, Tensor v_cache, c10::optional<Tensor> k_scale,
                 c10::optional<Tensor> v_scale, Tensor block_tables, Tensor seq_lens, Tensor out, Tensor part_o,
                 Tensor part_m, Tensor part_l, int64_t block_size, int64_t block_stride, int64_t num_kv_heads,
                 double scale, int64_t num_splits, int64_t split_len, c10::optional<Tensor> status,
                 std::vector<int64_t> chan) {
  CHECK_CUDA(q); CHECK_CONTIG(q); CHECK_CONTIG(out); CHECK_DT(q, torch::kBFloat16);
  CHECK_DT(block_tables, torch::kInt32); CHECK_DT(seq_lens, torch::kInt32); CHECK_CONTIG(block_tables);
  const int B = (int)q.size(0);
  const int nq = (int)q.size(1), D = (int)q.size(2);
  TORCH_CHECK(nq % num_kv_heads == 0, "q heads must be a multiple of kv heads");
  TORCH_CHECK(block_tables.size(0) >= B && seq_lens.numel() >= B, "metadata rows");
  b200::DecodeArgs a{};
  a.q = q.data_ptr();
  a.k_cache = k_cache.data_ptr();
  a.v_cache = v_cache.data_ptr();
  a.kv_int8 = k_cache.scalar_type() == torch::kInt8;
  a.k_scale = ptr_or_null<float>(k_scale);
  a.v_scale = ptr_or_null<float>(v_scale);
  a.block_tables = block_tables.data_ptr<int>();
  a.seq_lens = seq_lens.data_ptr<int>();
  a.max_blocks = (int)block_tables.size(1);
  a.block_size = (int)block_size;
  a.block_stride = block_stride;
  a.num_kv_heads = (int)num_kv_heads;
  a.group = nq / (int)num_kv_heads;
  a.head_dim = D;
  a.scale = (float)scale;
  a.num_splits = (int)num_splits;
  a.split_len = (int)split_len;
  a.part_o = part_o.data_ptr<float>();
  a.part_m = part_m.data_ptr<float>();
  a.part_l = part_l.data_ptr<float>();
  a.out = out.data_ptr();
  a.num_blocks = (int)k_cache.size(0);
  a.status = ptr_or_null<int>(status);
  set_kv_channel(&a.kv_int8, &a.ch, chan);
  if (num_splits > 1)
    TORCH_CHECK(part_m.numel() >= (int64_t)B * nq * num_splits && part_o.numel() >= (int64_t)B * nq * num_splits * D,
                "split workspace too small");
  b200::paged_decode_attn(a, B, stream());
}

void prefill_attn(Tensor q, Tensor k_cache, Tensor v_cache, c10::optional<Tensor> k_scale,
                  c10::optional<Tensor> v_scale, Tensor cu_seqlens_q, Tensor seq_lens, Tensor block_tables,
                  Tensor out, int64_t max_q_len, int64_t block_size, int64_t block_stride, int64_t num_kv_heads,
                  double scale, c10::optional<Tensor> status, std::vector<int64_t> chan) {
  CHECK_CUDA(q); CHECK_CONTIG(q); CHECK_CONTIG(out); CHECK_DT(q, torch::kBFloat16);
  CHECK_DT(cu_seqlens_q, torch::kInt32); CHECK_DT(seq_lens, torch::kInt32); CHECK_DT(block_tables, torch::kInt32);
  CHECK_CONTIG(block_tables); CHECK_CONTIG(cu_seqlens_q);
  const int B = (int)seq_lens.numel();
  const int nq = (int)q.size(1), D = (int)q.size(2);
  b200::PrefillArgs a{};
  a.q = q.data_ptr();
  a.k_cache = k_cache.data_ptr();
  a.v_cache = v_cache.data_ptr();
  a.kv_int8 = k_cache.scalar_type() == torch::kInt8;
  a.k_scale = ptr_or_null<float>(k_scale);
  a.v_scale = ptr_or_null<float>(v_scale);
  a.cu_seqlens_q = cu_seqlens_q.data_ptr<int>();
  a.seq_lens = seq_lens.data_ptr<int>();
  a.block_tables = block_tables.data_ptr<int>();
  a.max_blocks = (int)block_tables.size(1);
  a.block_size = (int)block_size;
  a.block_stride = block_stride;
  a.num_kv_heads = (int)num_kv_heads;
  a.group = nq / (int)num_kv_heads;
  a.head_dim = D;
  a.scale = (float)scale;
  a.out = out.data_ptr();
  a.num_blocks = (int)k_cache.size(0);
  a.status = ptr_or_null<int>(status);
  a.q_rows = (int)q.size(0);
  a.batch = B;
  set_kv_channel(&a.kv_int8, &a.ch, chan);
  b200::paged_prefill_attn(a, B, (int)max_q_len, stream());
}

void kv_int8_stage(Tensor k_cache, Tensor v_cache, c10::optional<Tensor> k_scale, c10::optional<Tensor> v_scale,
                   Tensor block_tables, Tensor seq_lens, Tensor stage, int64_t block_size, int64_t block_stride,
                   int64_t num_kv_heads, std::vector<int64_t> chan) {
  CHECK_CUDA(k_cache); CHECK_DT(k_cache, torch::kInt8); CHECK_DT(v_cache, torch::kInt8);
  CHECK_DT(block_tables, torch::kInt32); CHECK_DT(seq_lens, torch::kInt32); CHECK_CONTIG(block_tables);
  CHECK_DT(stage, torch::kBFloat16); CHECK_CONTIG(stage);
  const int64_t B = block_tables.size(0), mb = block_tables.size(1), D = k_cache.size(-1);
  TORCH_CHECK(seq_lens.numel() >= B, "seq_lens rows");
  TORCH_CHECK(stage.numel() >= B * mb * 2 * num_kv_heads * block_size * D, "stage too small");
  b200::KvStageArgs a{};
  a.k_cache = k_cache.data_ptr();
  a.v_cache = v_cache.data_ptr();
  a.kv_int8 = 1;
  a.k_scale = ptr_or_null<float>(k_scale);
  a.v_scale = ptr_or_null<float>(v_scale);
  set_kv_channel(&a.kv_int8, &a.ch, chan);
  a.block_tables = block_tables.data_ptr<int>();
  a.seq_lens = seq_lens.data_ptr<int>();
  a.batch = (int)B;
  a.max_blocks = (int)mb;
  a.block_size = (int)block_size;
  a.block_stride = block_stride;
  a.num_kv_heads = (int)num_kv_heads;
  a.head_dim = (int)D;
  a.stage = stage.data_ptr();
  b200::kv_int8_stage(a, stream());
}

void argmax(Tensor logits, Tensor out) {
  CHECK_CUDA(logits); CHECK_DT(logits, torch::kFloat32); CHECK_DT(out, torch::kInt32);
  TORCH_CHECK(logits.stride(1) == 1, "logits inner stride must be 1");
  b200::argmax_rows(logits.data_ptr<float>(), (int)logits.size(0), (int)logits.size(1), logits.stride(0),
                    out.data_ptr<int>(), stream());
}

void sample(Tensor logits, Tensor temperature, c10::optional<Tensor> top_k, c10::optional<Tensor> top_p,
            c10::optional<Tensor> min_p, Tensor seeds, c10::optional<Tensor> offsets, Tensor out,
            c10::optional<Tensor> allow, c10::optional<Tensor> allow_row, int64_t lp_k,
            c10::optional<Tensor> lp_top_v, c10::optional<Tensor> lp_top_i, c10::optional<Tensor> lp_chosen) {
  CHECK_CUDA(logits); CHECK_DT(logits, torch::kFloat32); CHECK_DT(temperature, torch::kFloat32);
  CHECK_DT(seeds, torch::kInt64); CHECK_DT(out, torch::kInt32);
  TORCH_CHECK(logits.stride(1) == 1, "logits inner stride must be 1");
  const int64_t B = logits.size(0);
  b200::SampleArgs a{};
  a.temperature = temperature.data_ptr<float>();
  a.top_k = ptr_or_null<int>(top_k);
  a.top_p = ptr_or_null<float>(top_p);
  a.min_p = ptr_or_null<float>(min_p);
  a.seeds = seeds.data_ptr<int64_t>();
  a.offsets = ptr_or_null<int64_t>(offsets);
  if (allow.has_value()) {
    TORCH_CHECK(allow_row.has_value(), "allow needs allow_row");
    CHECK_DT((*allow), torch::kInt32); CHECK_DT((*allow_row), torch::kInt32); CHECK_CONTIG((*allow));
    TORCH_CHECK(allow->dim() == 2 && allow_row->numel() >= B, "allow [masks, words], allow_row [B]");
    a.allow = reinterpret_cast<const uint32_t*>(allow->data_ptr<int>());
    a.allow_row = allow_row->data_ptr<int>();
    a.mask_words = (int)allow->size(1);
  }
  a.lp_k = (int)lp_k;
  if (lp_k > 0) {
    TORCH_CHECK(lp_top_v.has_value() && lp_top_i.has_value() && lp_chosen.has_value(), "log-prob outputs");
    CHECK_DT((*lp_top_v), torch::kFloat32); CHECK_DT((*lp_top_i), torch::kInt32);
    CHECK_DT((*lp_chosen), torch::kFloat32);
    TORCH_CHECK(lp_top_v->numel() >= B * lp_k && lp_top_i->numel() >= B * lp_k && lp_chosen->numel() >= B,
                "log-prob outputs too small");
    a.lp_top_v = lp_top_v->data_ptr<float>();
    a.lp_top_i = lp_top_i->data_ptr<int>();
    a.lp_chosen = lp_chosen->data_ptr<float>();
  }
  b200::sample_rows(logits.data_ptr<float>(), (int)logits.size(0), (int)logits.size(1), logits.stride(0), a,
                    out.data_ptr<int>(), stream());
}

void penalties(Tensor logits, Tensor rows, Tensor ids, Tensor gen_counts, Tensor presence, Tensor frequency,
               Tensor repetition) {
  CHECK_CUDA(logits); CHECK_DT(logits, torch::kFloat32);
  CHECK_DT(rows, torch::kInt32); CHECK_DT(ids, torch::kInt32); CHECK_DT(gen_counts, torch::kInt32);
  b200::apply_penalties(logits.data_ptr<float>(), logits.stride(0), rows.data_ptr<int>(), ids.data_ptr<int>(),
                        gen_counts.data_ptr<int>(), presence.data_ptr<float>(), frequency.data_ptr<float>(),
                        repetition.data_ptr<float>(), (int)rows.numel(), stream());
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "b200moe sm_100a kernels";
  m.def("gemm", &gemm);
  m.def("embed", &embed);
  m.def("rmsnorm", &rmsnorm);
  m.def("moe_combine", &moe_combine);
  m.def("qknorm_rope_kvstore", &qknorm_rope_kvstore);
  m.def("router_topk", &router_topk);
  m.def("moe_permute", &moe_permute);
  m.def("splitk_reduce", &splitk_reduce);
  m.def("rmsnorm_partials", &rmsnorm_partials);
  m.def("router_fused", &router_fused);
  m.def("dequant_weights", &dequant_weights);
  m.def("kv_blocks_copy", &kv_blocks_copy);
  m.def("ipc_alloc", &ipc_alloc);
  m.def("ipc_open", &ipc_open);
  m.def("ipc_export", &ipc_export);
  m.def("ipc_close", &ipc_close);
  m.def("ipc_free", &ipc_free);
  m.def("tensor_from_ptr", &tensor_from_ptr);
  m.def("decode_attn", &decode_attn);
  m.def("router_dispatch", &router_dispatch);
  m.def("prefill_attn", &prefill_attn);
  m.def("kv_int8_stage", &kv_int8_stage);
  m.def("argmax", &argmax);
  m.def("gemm_peer_scatter", &gemm_peer_scatter);
  m.def("ep_dispatch", &ep_dispatch);
  m.def("tp_slots_partial", &tp_slots_partial);
  m.def("tp_allreduce_rmsnorm", &tp_allreduce_rmsnorm);
  m.def("ep_scatter", &ep_scatter);
  m.def("ep_signal", &ep_signal);
  m.def("ep_wait_done", &ep_wait_done);
  m.def("sample", &sample);
  m.def("penalties", &penalties);
  m.attr("EPI_BF16") = (int)b200::kEpiBf16;
  m.attr("EPI_F32") = (int)b200::kEpiF32;
  m.attr("EPI_SILU_PAIR") = (int)b200::kEpiSiluPair;
  m.attr("EPI_SCATTER") = (int)b200::kEpiScatter;
}

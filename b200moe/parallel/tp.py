"""Tensor-parallel attention collectives fused into their consumer, over NVLink
peer memory (kernels: csrc/kernels/tp_comm.cu).

With ``attention_parallel="tp"`` every rank holds every token and a slice of the
heads and experts; twice per layer the ranks' partial sums must be added up and
fed to the residual RMSNorm.  The reference does that with an NCCL all-reduce
after its row-parallel O projection and after its experts
(nanovllm/layers/linear.py:152-160, nanovllm/models/qwen3_moe.py:414-418).
Here, for decode-size batches:

    O projection: the tcgen05 GEMM writes its fp32 (split-K) partial into this
    rank's symmetric buffer and its last CTA releases an epoch to every rank;
    MoE: ``tp_slots_partial`` sums the local experts' top-k slots into the buffer
    and releases;
    then ``tp_allreduce_rmsnorm`` waits for every rank's epoch, sums the W
    partials of each token over NVLink in rank order, adds the residual and
    normalises -- one kernel instead of all-reduce + add + norm, no NCCL.

The sum is the same on every rank (same data, same order), so the replicated
residual stream stays bit-identical.  Partial buffers rotate through three slots
(a peer is at most one step ahead; the third covers an odd count per forward);
batches above ``max_tokens`` use the NCCL path, where a ring or NVLS all-reduce
moves fewer bytes than every rank reading every peer's partial.
"""
from __future__ import annotations

import os

import torch

from b200moe import ops
from b200moe.parallel.p2p import PeerBuffers

FUSED_MAX_TOKENS = int(os.environ.get("B200MOE_TP_FUSED_MAX_TOKENS", "1024"))
MAX_SPLITS = 4


class TpComm:

    def __init__(self, symm: PeerBuffers, world: int, rank: int, hidden: int, max_tokens: int, device):
        self.symm, self.W, self.rank, self.H, self.max_tokens = symm, world, rank, hidden, max_tokens
        self.epoch = torch.zeros(1, dtype=torch.int32, device=device)
        self.prod_counter = torch.zeros(1, dtype=torch.int32, device=device)
        self.norm_counter = torch.zeros(1, dtype=torch.int32, device=device)
        self.status = ops.status_word(device)
        self.wait_ns = torch.zeros(world, dtype=torch.int64, device=device)
        self.flag_ptrs = symm["flags"][1]
        self.part = [symm[f"part{i}"] for i in range(3)]
        self._i, self._n = 0, 0

    @staticmethod
    def create(runner) -> "TpComm | None":
        """Allocate and map the symmetric buffers on every rank (a collective); None
        when peer memory is unavailable or ``B200MOE_TP_FUSED=0``."""
        if runner.device.type != "cuda" or os.environ.get("B200MOE_TP_FUSED", "1") == "0":
            return None
        W, rank = runner.world_size, runner.rank
        H = runner.args.hidden_size
        T = min(runner.config.max_num_batched_tokens, FUSED_MAX_TOKENS)
        di = runner.device.index if runner.device.index is not None else torch.cuda.current_device()
        symm = PeerBuffers(rank, W, di, "tp")
        for i in range(3):
            symm.alloc(f"part{i}", (MAX_SPLITS * T, H), torch.float32)
        symm.alloc("flags", (W,), torch.int32)
        if not symm.agree():
            symm.release()
            return None
        symm["flags"][0].zero_()
        torch.cuda.synchronize(di)
        return TpComm(symm, W, rank, H, T, runner.device)

    def close(self):
        self.symm.release()

    # ------------------------------------------------------------- per forward
    def begin_forward(self, sites: int):
        """Call at the start of every forward with the number of fused sums it will
        run, so the slot sequence is the same in eager steps and graph replays."""
        self._i, self._n = 0, sites

    def _slot(self) -> int:
        i = self._i
        self._i += 1
        return 2 if (self._n % 2 and i == self._n - 1) else i % 2

    def _dims(self, splits: int, T: int):
        return [self.W, self.rank, splits, T * self.H]

    def _norm(self, slot, splits, residual, norm_w, eps, out):
        ops.native().tp_allreduce_rmsnorm(self._dims(splits, residual.shape[0]), self.part[slot][1], self.flag_ptrs,
                                          self.epoch, self.norm_counter, self.status, self.wait_ns, residual,
                                          norm_w, out, eps, self.max_tokens)
        ops.count_launches()
        return out

    def o_proj_add_norm(self, attn, weight, scale, residual, norm_w, eps, out, tiled: bool):
        """residual += sum over ranks of attn @ W_o[:, rank's heads]^T; returns rmsnorm(residual) * norm_w."""
        T, K = attn.shape
        N = weight.shape[0]
        m_tiles = N // 128
        bn, splits = ops.plan_dense(T, m_tiles, K // 64, fp8=scale is not None, max_splits=MAX_SPLITS)
        slot = self._slot()
        part = self.part[slot][0][:splits * T].view(splits * T, N)
        release = [self.epoch.data_ptr(), self.prod_counter.data_ptr(), self.rank, 1, *self.flag_ptrs]
        ops.native().gemm(weight, scale, attn, ops.count_tensor(T, attn.device), None, part, bn, ops.EPI_F32, m_tiles,
                          0, 0, None, None, self.status, ops._trace[0], splits, T * N, tiled, release)
        ops.count_launches()
        return self._norm(slot, splits, residual, norm_w, eps, out)

    def slots_add_norm(self, slots, topk, residual, norm_w, eps, out):
        """residual += sum over ranks of the fixed-order top-k sum of this rank's expert slots;
        returns rmsnorm(residual) * norm_w."""
        T = residual.shape[0]
        slot = self._slot()
        ops.native().tp_slots_partial(self._dims(1, T), self.part[slot][1], self.flag_ptrs, self.epoch,
                                      self.prod_counter, self.status, self.wait_ns, slots, topk, T, self.H,
                                      self.max_tokens)
        ops.count_launches()
        return self._norm(slot, 1, residual, norm_w, eps, out)

    def wait_stats(self, reset: bool = True) -> dict:
        v = self.wait_ns.cpu().tolist()
        if reset:
            self.wait_ns.zero_()
        return {"allreduce_ms": [round(x / 1e6, 2) for x in v]}

"""Fused expert-parallel MoE over NVLink peer memory (kernels: csrc/kernels/ep_p2p.cu).

Buffers are symmetric (``torch.distributed._symmetric_memory``): every rank
allocates the same layout and gets the device addresses of every peer's copy.
Per MoE layer (no host synchronisation, CUDA-graph capturable):

    ep_dispatch  -> ep_count -> ep_scatter -> gate/up GEMM -> down GEMM with
    peer-scatter epilogue -> ep_signal -> ep_wait_done -> (model) moe_combine

The routed rows cross NVLink once (source -> owner, as P2P stores from the
dispatch kernel) and the weighted expert outputs cross once (owner -> source,
as P2P stores from the down GEMM's epilogue).  No TMA multicast, no library
kernel touches peer memory.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from b200moe import ops


class P2PMoE:

    def __init__(self, ep, symm):
        self.ep = ep
        self.symm = symm

    @staticmethod
    def create(ep) -> "P2PMoE | None":
        import torch.distributed._symmetric_memory as symm_mem
        runner = ep.runner
        cfg = runner.config
        args = runner.args
        W, rank, dev = ep.world, ep.rank, ep.device
        H, k = args.hidden_size, args.num_experts_per_tok
        slot_cap = cfg.max_num_batched_tokens * k
        cap = slot_cap
        group = dist.group.WORLD
        try:
            symm_mem.enable_symm_mem_for_group(group.group_name)
        except Exception:
            pass

        def alloc(*shape, dtype):
            t = symm_mem.empty(*shape, dtype=dtype, device=dev)
            t.zero_()
            h = symm_mem.rendezvous(t, group.group_name)
            return t, [int(p) for p in h.buffer_ptrs]

        symm = {}
        for name, shape, dt in (("recv_x", (W * cap, H), torch.bfloat16), ("recv_meta", (W * cap, 4), torch.int32),
                                ("counts", (W,), torch.int32), ("flags", (W,), torch.int32),
                                ("done", (W,), torch.int32), ("slots", (slot_cap, H), torch.bfloat16)):
            symm[name] = alloc(*shape, dtype=dt)
        torch.cuda.synchronize(dev)
        dist.barrier()
        self = P2PMoE(ep, symm)
        self.W, self.rank, self.H, self.cap, self.slot_cap = W, rank, H, cap, slot_cap
        self.owner = ep.owner.to(torch.int32)
        self.g2l = ep.g2l
        self.send_cursor = torch.zeros(W, dtype=torch.int32, device=dev)
        self.done_blocks = torch.zeros(1, dtype=torch.int32, device=dev)
        self.epoch = torch.zeros(1, dtype=torch.int32, device=dev)
        self.status = ops.status_word(dev)
        return self

    def _a(self):
        s = self.symm
        return ([self.W, self.rank, self.H, self.cap, self.slot_cap], self.owner, self.g2l, self.send_cursor,
                self.done_blocks, self.epoch, self.status, s["recv_x"][1], s["recv_meta"][1], s["counts"][1],
                s["flags"][1], s["done"][1])

    def moe(self, model, layer, x, ids, w, slots):
        """Returns the tensor holding this rank's (token, k) slots."""
        C = ops.native()
        a = self._a()
        T = x.shape[0]
        El = model.num_local_experts
        I = layer.w2.shape[-1]
        C.ep_dispatch(*a, x, ids, w.contiguous())
        ops.count_launches()
        cnt = model._buf("ep_counts", (2 * El,), torch.int32)
        cnt.zero_()
        C.ep_count(*a, cnt[:El])
        rows = self.W * self.cap
        xp = model._buf("x_perm", (rows, self.H), model.dtype)
        code = model._buf("slot_of_row", (rows,), torch.int32)
        sw = model._buf("ep_slot_w", (rows,), torch.float32)
        off = model._buf("ep_offsets", (El + 1,), torch.int32)
        C.ep_scatter(*a, cnt[:El], cnt[El:], xp, code, sw, off)
        h = model._buf("h_perm", (rows, I), model.dtype)
        expected = max(1, T * self.W)  # rows this rank expects on average
        ops.grouped_gate_up_silu(xp, layer.w13, layer.s13, cnt[:El], off, h, I,
                                 bn=ops.pick_bn(expected * model.args.num_experts_per_tok, I // 128, El, pair=True))
        C.gemm_peer_scatter(layer.w2, layer.s2, h, cnt[:El], off,
                            ops.pick_bn(expected * model.args.num_experts_per_tok, self.H // 128, El),
                            code, sw, self.symm["slots"][1], self.slot_cap, self.H, self.status)
        C.ep_signal(*a)
        C.ep_wait_done(*a)
        ops.count_launches(6)
        return self.symm["slots"][0]

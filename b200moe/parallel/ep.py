"""Expert parallelism across ranks: each rank owns E/world experts, tokens are
sharded by rank (data-parallel attention), and every MoE layer moves routed
rows to the experts' owners and the weighted results back to their
(token, k) slots.  The combine stays a fixed-order local sum, so results do
not depend on arrival order.

Backends:

* ``reference`` (CPU / gloo, and the ``loop`` backend): all-gather every rank's
  tokens, each rank computes its own experts' slot contributions for all of
  them, one all-reduce sums the (single-contributor) slots, each rank keeps
  its rows.  Exact and simple; the plumbing oracle (reference pattern:
  tests/archive/p2_min_repro.py, gloo world_size=2).
* ``nccl_a2a`` (CUDA baseline): count exchange + ``all_to_all_single`` of the
  routed rows, local grouped tcgen05 GEMMs, ``all_to_all_single`` back.  Needs
  one host read of the counts per layer, so it runs eagerly.
* ``fused`` (CUDA product path): dispatch and combine written as P2P stores
  into peers' symmetric buffers inside the MoE kernels (b200moe/parallel/p2p.py);
  falls back to ``nccl_a2a`` when peer access is unavailable.

Reference: the replicated-hidden EP with one all_reduce per layer,
nanovllm/models/qwen3_moe.py:69-75, 414-418.
"""
from __future__ import annotations

import os

import torch
import torch.distributed as dist

from b200moe import ops


class ExpertParallel:

    def __init__(self, runner, backend: str):
        self.runner = runner
        self.world = runner.world_size
        self.rank = runner.rank
        self.device = runner.device
        args = runner.args
        self.E = args.num_experts
        model = runner.model
        owner = torch.empty(self.E, dtype=torch.int64)
        g2l = torch.full((self.E,), -1, dtype=torch.int32)
        ge_local = torch.full((self.E,), -1, dtype=torch.int32)  # index of each expert on its owner
        placement = [None] * self.world
        from b200moe.engine.model_runner import expert_placement
        for r in range(self.world):
            placement[r] = expert_placement(runner.config, r, self.world)
            for le, ge in enumerate(placement[r]):
                owner[ge] = r
                ge_local[ge] = le
                if r == self.rank:
                    g2l[ge] = le
        assert placement[self.rank] == model.expert_ids
        self.owner = owner.to(self.device)
        self.g2l = g2l.to(self.device)
        self.ge_local = ge_local.to(self.device)
        self.num_local = len(placement[self.rank])
        cuda = self.device.type == "cuda"
        if backend == "loop" or not cuda:
            self.backend = "reference"
        else:
            self.backend = "nccl_a2a" if backend in ("nccl_a2a", "fused") else backend
        self.p2p = None
        if cuda and backend == "fused":
            # B200MOE_EP_STRICT=1 (set by bench.py): a fused path that cannot be set up
            # is an error, not a silent fall-back to the NCCL baseline
            strict = os.environ.get("B200MOE_EP_STRICT", "0") == "1"
            try:
                from b200moe.parallel.p2p import P2PMoE
                self.p2p = P2PMoE.create(self)
                if self.p2p is not None:
                    self.backend = "fused"
            except Exception as exc:  # no peer access: NCCL baseline
                if strict:
                    raise
                print(f"[ep] fused P2P path unavailable ({exc}); using nccl_a2a", flush=True)
                self.p2p = None
            if self.p2p is None and strict:
                raise RuntimeError("expert parallelism: the fused peer-memory path was requested "
                                   "(B200MOE_EP_STRICT=1) but could not be set up on every rank")

    @property
    def graph_safe(self) -> bool:
        return self.backend == "fused"

    # --------------------------------------------------------- reference
    def moe_reference(self, model, layer, x, ids, w):
        T, H = x.shape
        k = ids.shape[1]
        n = torch.tensor([T], dtype=torch.int64, device=x.device)
        sizes = [torch.zeros_like(n) for _ in range(self.world)]
        dist.all_gather(sizes, n)
        sizes = [int(s) for s in sizes]
        Tm = max(max(sizes), 1)
        pad = lambda t, fill=0: torch.cat([t, t.new_full((Tm - T, *t.shape[1:]), fill)]) if T < Tm else t
        xs = [torch.empty(Tm, H, dtype=x.dtype, device=x.device) for _ in range(self.world)]
        is_ = [torch.empty(Tm, k, dtype=ids.dtype, device=x.device) for _ in range(self.world)]
        ws = [torch.empty(Tm, k, dtype=w.dtype, device=x.device) for _ in range(self.world)]
        dist.all_gather(xs, pad(x.contiguous()))
        dist.all_gather(is_, pad(ids.contiguous(), -1))
        dist.all_gather(ws, pad(w.contiguous()))
        allx = torch.cat([t[:s] for t, s in zip(xs, sizes)])
        alli = torch.cat([t[:s] for t, s in zip(is_, sizes)])
        allw = torch.cat([t[:s] for t, s in zip(ws, sizes)])
        part = model.experts_reference(layer, allx, alli, allw)  # [sumT, k, H] fp32, zeros off-rank
        dist.all_reduce(part)
        start = sum(sizes[:self.rank])
        return part[start:start + T].sum(dim=1).to(x.dtype)

    def combine_wait(self):
        """What the combine kernel waits on before reading the slots (fused path), else None."""
        return self.p2p.combine_wait() if self.backend == "fused" else None

    # --------------------------------------------------------------- fused
    def route_dispatch(self, model, layer, x):
        """Fused path: router and dispatch in one launch, (ids, weights); None where it
        does not apply (other backends, or the router shape)."""
        if self.backend != "fused" or not x.is_cuda:
            return None
        return self.p2p.route_dispatch(model, layer, x)

    def moe_fused(self, model, layer, x, ids, w, slots, dispatched: bool = False):
        if self.backend == "fused":
            return self.p2p.moe(model, layer, x, ids, w, slots, dispatched)
        if self.backend == "reference":
            out = self.moe_reference(model, layer, x, ids, w)
            slots.zero_()
            slots.view(x.shape[0], ids.shape[1], -1)[:, 0].copy_(out)
            return slots
        return self._moe_a2a(model, layer, x, ids, w, slots)

    def _moe_a2a(self, model, layer, x, ids, w, slots):
        T, H = x.shape
        k = ids.shape[1]
        W = self.world
        dev = x.device
        flat_ids = ids.reshape(-1).long()
        dest = self.owner[flat_ids]
        order = torch.argsort(dest, stable=True)
        send_counts = torch.bincount(dest, minlength=W)
        recv_counts = torch.empty_like(send_counts)
        dist.all_to_all_single(recv_counts, send_counts)
        counts = torch.stack([send_counts, recv_counts]).cpu()  # the one host sync per layer
        sc, rc = counts[0].tolist(), counts[1].tolist()
        R = sum(rc)
        if model.profiler is not None:
            model.profiler.observe("moe.local_pairs", R)  # expert-parallel load on this rank
        send_x = x.index_select(0, order // k)
        meta = torch.stack([flat_ids[order].to(torch.int32),
                            w.reshape(-1)[order].contiguous().view(torch.int32)], dim=1)
        recv_x = torch.empty(R, H, dtype=x.dtype, device=dev)
        recv_meta = torch.empty(R, 2, dtype=torch.int32, device=dev)
        dist.all_to_all_single(recv_x, send_x, rc, sc)
        dist.all_to_all_single(recv_meta, meta, rc, sc)
        out = torch.empty(R, H, dtype=x.dtype, device=dev)
        if R:
            El = model.num_local_experts
            le = self.g2l[recv_meta[:, 0].long()].view(R, 1).contiguous()
            rw = recv_meta[:, 1].contiguous().view(torch.float32)
            cnt = model._buf("ep_counts", (2 * El,), torch.int32)
            cnt.zero_()
            cnt[:El].copy_(torch.bincount(le.view(-1).long(), minlength=El).to(torch.int32))
            xp = model._buf("x_perm", (R, H), model.dtype)
            sor = model._buf("slot_of_row", (R,), torch.int32)
            off = model._buf("ep_offsets", (El + 1,), torch.int32)
            ops.moe_permute(recv_x, le, cnt[:El], cnt[El:], xp, sor, off)
            I = layer.w2.shape[-1]
            h = model._buf("h_perm", (R, I), model.dtype)
            ops.grouped_gate_up_silu(xp, layer.w13, layer.s13, cnt[:El], off, h, I, tiled=model.weights_tiled)
            ops.grouped_down_scatter(h, layer.w2, layer.s2, cnt[:El], off, sor, rw, out, tiled=model.weights_tiled)
        back = torch.empty(T * k, H, dtype=x.dtype, device=dev)
        dist.all_to_all_single(back, out, sc, rc)
        slots.index_copy_(0, order, back)
        return slots

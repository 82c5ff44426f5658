"""Fused expert-parallel MoE over NVLink peer memory (kernels: csrc/kernels/ep_p2p.cu).

Buffers are symmetric: every rank allocates the same layout (one cudaMalloc
per buffer), shares it through a CUDA IPC handle, and maps every peer's copy
on its own device (plain NVLink peer mappings, no multicast object).
Per MoE layer, five launches, no host synchronisation, CUDA-graph capturable:

    ep_dispatch (rows + per-expert counts to the owners, epoch flag)
    -> ep_scatter (waits for every source; expert-sorted rows from the count matrix)
    -> gate/up GEMM -> down GEMM (peer-scatter epilogue; its last CTA releases the
       done epoch) -> (model) moe_combine (waits for every owner's done epoch)

The routed rows cross NVLink once (source -> owner, as P2P stores from the
dispatch kernel) and the weighted expert outputs cross once (owner -> source,
as P2P stores from the down GEMM's epilogue).  Peer memory is touched only by
plain loads and stores of these kernels; no TMA load and no library kernel
ever reads it.
"""
from __future__ import annotations

import os

import torch
import torch.distributed as dist

from b200moe import ops


class PeerBuffers:
    """Symmetric device buffers: every rank allocates the same named buffers (one
    cudaMalloc each), shares them through CUDA IPC handles and maps every peer's
    copy on its own device -- plain NVLink peer mappings, no multicast object.
    Every rank takes part in every exchange even after a local failure, so the
    collective sequence stays aligned; ``agree`` settles whether all ranks
    succeeded.  Peer memory is read and written only by this repository's own
    ld/st kernels."""

    def __init__(self, rank: int, world: int, device_index: int, tag: str):
        self.rank, self.world, self.di, self.tag = rank, world, device_index, tag
        self.ok = True
        self.bufs: dict[str, tuple] = {}
        self._owned, self._opened = [], []

    def alloc(self, name: str, shape: tuple, dtype) -> tuple:
        """(local tensor or None, [device pointer of every rank's copy])."""
        C = ops.native()
        nbytes = torch.empty(0, dtype=dtype).element_size()
        for d in shape:
            nbytes *= d
        ptr, blob = None, None
        if self.ok:
            try:
                ptr, handle = C.ipc_alloc(nbytes, self.di)
                self._owned.append(ptr)
                blob = bytes(handle.numpy())
            except Exception as exc:  # noqa: BLE001 - reported, then the caller falls back
                print(f"[{self.tag}] ipc_alloc failed on rank {self.rank}: {exc}", flush=True)
                self.ok = False
        handles = [None] * self.world
        dist.all_gather_object(handles, blob)
        ptrs = []
        for r, h in enumerate(handles):
            if not self.ok or h is None:
                self.ok = False
                break
            if r == self.rank:
                ptrs.append(ptr)
                continue
            try:
                q = C.ipc_open(torch.frombuffer(bytearray(h), dtype=torch.uint8), self.di)
                self._opened.append(q)
                ptrs.append(q)
            except Exception as exc:  # noqa: BLE001
                print(f"[{self.tag}] ipc_open of rank {r} failed on rank {self.rank}: {exc}", flush=True)
                self.ok = False
                break
        out = ((C.tensor_from_ptr(ptr, list(shape), dtype, self.di) if self.ok else None), ptrs)
        self.bufs[name] = out
        return out

    def __getitem__(self, name: str) -> tuple:
        return self.bufs[name]

    def agree(self) -> bool:
        """True when every rank allocated and mapped every buffer (a collective)."""
        torch.cuda.synchronize(self.di)
        verdict = torch.tensor([1 if self.ok else 0], dtype=torch.int32, device=torch.device("cuda", self.di))
        dist.all_reduce(verdict, op=dist.ReduceOp.MIN)
        return bool(int(verdict.item()))

    def release(self):
        """Unmap the peers' buffers and free this rank's, after a device sync and a
        barrier so that no peer still writes into them (a collective)."""
        if not self._owned and not self._opened:
            return
        C = ops.native()
        torch.cuda.synchronize(self.di)
        if dist.is_initialized():
            dist.barrier()
        for p in self._opened:
            C.ipc_close(p, self.di)
        self.bufs.clear()
        for p in self._owned:
            C.ipc_free(p, self.di)
        self._owned, self._opened = [], []


class P2PMoE:

    def __init__(self, ep, symm):
        self.ep = ep
        self.symm = symm

    @staticmethod
    def create(ep) -> "P2PMoE | None":
        runner = ep.runner
        cfg = runner.config
        args = runner.args
        W, rank, dev = ep.world, ep.rank, ep.device
        H, k = args.hidden_size, args.num_experts_per_tok
        slot_cap = cfg.max_num_batched_tokens * k
        cap = slot_cap
        di = dev.index if dev.index is not None else torch.cuda.current_device()
        symm = PeerBuffers(rank, W, di, "ep")
        self = P2PMoE(ep, symm)
        El = ep.num_local
        for name, shape, dt in (("recv_x", (W * cap, H), torch.bfloat16), ("recv_meta", (W * cap, 4), torch.int32),
                                ("counts", (W * El,), torch.int32), ("flags", (W,), torch.int32),
                                ("done", (W,), torch.int32), ("slots", (slot_cap, H), torch.bfloat16)):
            symm.alloc(name, shape, dt)
        self.device_index = di
        if not symm.agree():
            self.close()
            return None
        self.W, self.rank, self.H, self.cap, self.slot_cap = W, rank, H, cap, slot_cap
        self.El, self.E = El, ep.E
        self.owner = ep.owner.to(torch.int32)
        self.g2l = ep.g2l
        self.ge_local = ep.ge_local
        self.send_cursor = torch.zeros(W, dtype=torch.int32, device=dev)
        self.ecur = torch.zeros(ep.E, dtype=torch.int32, device=dev)
        self.cta_done = torch.zeros(1, dtype=torch.int32, device=dev)
        self.done_blocks = torch.zeros(1, dtype=torch.int32, device=dev)
        self.epoch = torch.zeros(1, dtype=torch.int32, device=dev)
        self.status = ops.status_word(dev)
        # device ns waited, summed: [each source's dispatch flag (ep_scatter) | each owner's done epoch (combine)]
        self.wait_ns = torch.zeros(2 * W, dtype=torch.int64, device=dev)
        return self

    def wait_stats(self, reset: bool = True) -> dict:
        """Milliseconds this rank's kernels spent waiting on each peer since the last reset:
        ``dispatch_ms[r]`` for rank r's rows to arrive, ``combine_ms[r]`` for rank r's
        expert outputs.  The rank the others wait on most is the straggler."""
        v = self.wait_ns.cpu().tolist()
        if reset:
            self.wait_ns.zero_()
        W = self.W
        return {"dispatch_ms": [round(x / 1e6, 2) for x in v[:W]],
                "combine_ms": [round(x / 1e6, 2) for x in v[W:2 * W]]}

    def close(self):
        """Release the symmetric buffers (a collective: every rank reaches it together)."""
        self.symm.release()

    def _a(self):
        s = self.symm
        return ([self.W, self.rank, self.H, self.cap, self.slot_cap, self.El, self.E], self.owner, self.g2l,
                self.ge_local, self.send_cursor, self.ecur, self.done_blocks, self.epoch, self.status, self.wait_ns,
                s["recv_x"][1], s["recv_meta"][1], s["counts"][1], s["flags"][1], s["done"][1])

    def combine_wait(self):
        """(this rank's done array, epoch, status, wait_ns) for the combine kernel's wait."""
        return self.symm["done"][0], self.epoch, self.status, self.wait_ns

    # B200MOE_EP_ROUTER_DISPATCH=1: the router's top-k warps send the routed rows
    # themselves (one launch instead of router + ep_dispatch).  Off by default: only a
    # token tile's last CTA holds the top-k, so two CTAs send all rows of 32 tokens, and
    # at one rank x 32 tokens the fused launch took 37 us against 15 + 11 us for the
    # router and the 32-block dispatch kernel.
    ROUTER_DISPATCH = os.environ.get("B200MOE_EP_ROUTER_DISPATCH", "0") == "1"

    def route_dispatch(self, model, layer, x):
        """Router + dispatch in one launch: (ids, weights) as ``model.route`` returns
        them, or None where the fused router does not apply (more than 128 experts,
        a non-bf16 router weight)."""
        a = model.args
        if not self.ROUTER_DISPATCH or a.num_experts > 128 or layer.router.dtype != torch.bfloat16:
            return None
        T, k = x.shape[0], a.num_experts_per_tok
        ids = model._buf("ids", (T * k,), torch.int32).view(T, k)
        w = model._buf("topw", (T * k,), torch.float32).view(T, k)
        part, cnt = ops.router_scratch(x.device)
        ops.native().router_dispatch(*self._a(), x, layer.router, a.num_experts, k, a.norm_topk_prob, ids, w, part,
                                     cnt)
        ops.count_launches()
        return ids, w

    def moe(self, model, layer, x, ids, w, slots, dispatched: bool = False):
        """Returns the tensor holding this rank's (token, k) slots; the caller's combine
        waits on ``combine_wait()`` before reading it.  ``dispatched``: the router
        already sent the rows (``route_dispatch``)."""
        C = ops.native()
        a = self._a()
        T = x.shape[0]
        El = model.num_local_experts
        I = layer.w2.shape[-1]
        if not dispatched:
            C.ep_dispatch(*a, x, ids, w.contiguous())
            ops.count_launches()
        rows = self.W * self.cap
        cnt = model._buf("ep_counts", (El,), torch.int32)
        off = model._buf("ep_offsets", (El + 1,), torch.int32)
        xp = model._buf("x_perm", (rows, self.H), model.dtype)
        code = model._buf("slot_of_row", (rows,), torch.int32)
        sw = model._buf("ep_slot_w", (rows,), torch.float32)
        C.ep_scatter(*a, cnt, xp, code, sw, off)
        if model.profiler is not None:
            model.profiler.observe("moe.local_pairs", cnt.sum())
        h = model._buf("h_perm", (rows, I), model.dtype)
        expected = max(1, T * self.W)  # rows this rank expects on average
        k = model.args.num_experts_per_tok
        # prefill-size steps: bf16 GEMMs on the resident dequantised copy when the rank keeps
        # one (the same bits as per-tile dequantisation, without re-converting every tile);
        # the rows this rank receives are estimated by the rows it sends (balanced routing)
        if model._bf16_experts(T * k) and getattr(layer, "w13_bf16", None) is not None:
            w13, s13, w2, s2, tiled = layer.w13_bf16, None, layer.w2_bf16, None, False
        else:
            w13, s13, w2, s2, tiled = layer.w13, layer.s13, layer.w2, layer.s2, model.weights_tiled
        ops.grouped_gate_up_silu(xp, w13, s13, cnt, off, h, I,
                                 bn=ops.pick_bn(expected * k, I // 128, El, pair=True), tiled=tiled)
        C.gemm_peer_scatter(w2, s2, h, cnt, off, ops.pick_bn(expected * k, self.H // 128, El),
                            code, sw, self.symm["slots"][1], self.slot_cap, self.H, self.status,
                            tiled, self.epoch, self.cta_done, self.symm["done"][1], self.rank)
        ops.count_launches(2)
        return self.symm["slots"][0]

"""Pinned host pool for evicted KV blocks (reference: nanovllm/engine/kv_offload.py:31-126).

Each slot holds one whole KV block (every layer, K and V: the pool layout makes
that one contiguous slab).  Copies run on a dedicated stream and never block
the host:

* ``put(block)``   device -> host copy on the copy stream; the compute stream
  waits on the copy's event before its next kernel, so the block can be handed
  out again right away without its old bytes being overwritten early;
* ``get(slot, block)`` host -> device copy, ordered the same way;
* a slot is reused only after its last copy's event completed.

The reference copies synchronously with a full device synchronise
(model_runner.py:284-305).  A full pool returns -1 (the caller drops the block,
as the reference does).
"""
from __future__ import annotations

import torch


class HostBlockPool:

    def __init__(self, num_slots: int, kv_pool, device):
        self.kv = kv_pool
        self.device = torch.device(device)
        self.num_slots = num_slots
        cuda = self.device.type == "cuda"
        shape = tuple(kv_pool.data.shape[1:])
        self.host = torch.empty((num_slots, *shape), dtype=kv_pool.data.dtype, pin_memory=cuda)
        self.free = list(range(num_slots - 1, -1, -1))  # LIFO
        self.in_use: set[int] = set()
        self._events: dict[int, object] = {}
        self.stream = torch.cuda.Stream(self.device) if cuda else None
        self.puts = self.gets = self.full = 0

    def has_room(self) -> bool:
        return bool(self.free)

    def _slot_ready(self, slot: int):
        ev = self._events.pop(slot, None)
        if ev is not None:
            ev.synchronize()

    def put(self, block_id: int) -> int:
        if not self.free:
            self.full += 1
            return -1
        slot = self.free.pop()
        self._slot_ready(slot)
        src = self.kv.block_view(block_id)
        if self.stream is None:
            self.host[slot].copy_(src)
        else:
            cur = torch.cuda.current_stream(self.device)
            self.stream.wait_stream(cur)           # the block's last writes are done
            with torch.cuda.stream(self.stream):
                self.host[slot].copy_(src, non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(self.stream)
            cur.wait_event(ev)                     # no later kernel overwrites the block early
            self._events[slot] = ev
        self.in_use.add(slot)
        self.puts += 1
        return slot

    def get(self, slot: int, block_id: int):
        if slot not in self.in_use:
            raise KeyError(f"host slot {slot} is not in use")
        dst = self.kv.block_view(block_id)
        if self.stream is None:
            dst.copy_(self.host[slot])
        else:
            cur = torch.cuda.current_stream(self.device)
            self.stream.wait_stream(cur)
            with torch.cuda.stream(self.stream):
                dst.copy_(self.host[slot], non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(self.stream)
            cur.wait_event(ev)                     # the next forward reads the revived block
            self._events[slot] = ev
        self.gets += 1

    def release(self, slot: int):
        if slot in self.in_use:
            self.in_use.remove(slot)
            self.free.append(slot)

    def view(self, slot: int) -> torch.Tensor:
        self._slot_ready(slot)
        return self.host[slot]

    def metrics(self) -> dict:
        return {"kv_offload_host_slots": self.num_slots, "kv_offload_host_in_use": len(self.in_use),
                "kv_offload_pool_full_total": self.full}

"""Paged-KV block allocator with a chained-hash prefix cache.

Behaviour matches the reference BlockManager (nanovllm/engine/block_manager.py:34-342):

* blocks are reference counted; a full block gets an xxh64 hash chained on its
  predecessor's hash, so a prompt prefix maps to a unique hash chain;
* reuse victims come from two tiers: never-cached ("fresh") blocks first, then
  the least-recently-used cached-but-unreferenced block (touch on admission
  hit).  ``B200MOE_LRU_EVICT=0`` (or the reference's ``NANOVLLM_LRU_EVICT=0``)
  falls back to a plain release-order FIFO;
* optional host offload: an evicted cached block is copied to a pinned host
  slot through an executor (``offload_put`` / ``offload_get`` /
  ``offload_release``) and revived on a later prefix hit; the device hash map
  and the host map never describe the same hash at once;
* the speculative (overlap-pipeline) helpers ``total_launch_shortfall`` /
  ``may_append_at`` check block coverage at launch-time length.

The free pool is two insertion-ordered dicts instead of the reference's deque
plus side sets, so every pop and touch is O(1).
"""
from __future__ import annotations

import os
from collections import OrderedDict
from itertools import count

import numpy as np
import xxhash

from b200moe.engine.sequence import Sequence


def _lru_default() -> bool:
    v = os.environ.get("B200MOE_LRU_EVICT", os.environ.get("NANOVLLM_LRU_EVICT", "1"))
    return v == "1"


class Block:
    __slots__ = ("block_id", "ref_count", "hash", "token_ids")

    def __init__(self, block_id: int):
        self.block_id = block_id
        self.ref_count = 0
        self.hash = -1
        self.token_ids: list[int] = []

    def update(self, h: int, token_ids: list[int]):
        self.hash = h
        self.token_ids = token_ids

    def reset(self):
        self.ref_count = 1
        self.hash = -1
        self.token_ids = []


class BlockManager:

    def __init__(self, num_blocks: int, block_size: int):
        self.block_size = block_size
        self.blocks = [Block(i) for i in range(num_blocks)]
        self.hash_to_block_id: dict[int, int] = {}
        self.used_block_ids: set[int] = set()
        self._stamp = count()
        # free pool: id -> release stamp, each dict in release (or touch) order
        self._fresh: OrderedDict[int, int] = OrderedDict((i, next(self._stamp)) for i in range(num_blocks))
        self._lru: OrderedDict[int, int] = OrderedDict()
        self.lru_enabled = _lru_default()
        self.prefix_cache_hit_tokens = 0
        self.allocations = 0
        self.reclaims = 0
        self.evictions = 0
        self._offload_exec = None
        self._host_map: dict[int, tuple[int, list[int]]] = {}
        self.host_puts = 0
        self.host_revives = 0
        self.host_drops = 0

    # ------------------------------------------------------------------ pool
    @property
    def num_free_blocks(self) -> int:
        return len(self._fresh) + len(self._lru)

    @property
    def free_block_ids(self) -> list[int]:
        """Free ids in victim order (fresh tier first, then LRU)."""
        return list(self._fresh) + list(self._lru)

    def _pop_free(self) -> int:
        if self.lru_enabled:
            if self._fresh:
                return self._fresh.popitem(last=False)[0]
            bid = self._lru.popitem(last=False)[0]
            self.evictions += 1
            return bid
        # FIFO over both tiers by release stamp
        f = next(iter(self._fresh.items()), None)
        c = next(iter(self._lru.items()), None)
        if c is None or (f is not None and f[1] < c[1]):
            return self._fresh.popitem(last=False)[0]
        return self._lru.popitem(last=False)[0]

    def _take_specific(self, block_id: int):
        if self._lru.pop(block_id, None) is None:
            self._fresh.pop(block_id)

    # --------------------------------------------------------------- offload
    def set_offload_executor(self, executor):
        """``executor.call(name, *args)`` runs a byte mover on every rank."""
        self._offload_exec = executor

    def _release_host_entry(self, h: int):
        entry = self._host_map.pop(h, None)
        if entry is not None:
            self._offload_exec.call("offload_release", entry[0])

    @staticmethod
    def compute_hash(token_ids: list[int], prefix: int = -1) -> int:
        h = xxhash.xxh64()
        if prefix != -1:
            h.update(prefix.to_bytes(8, "little"))
        h.update(np.asarray(token_ids, dtype=np.int64).tobytes())
        return h.intdigest()

    def _allocate_block(self) -> int:
        block_id = self._pop_free()
        block = self.blocks[block_id]
        assert block.ref_count == 0, "free block with live references"
        if block.hash != -1 and self.hash_to_block_id.get(block.hash) == block_id:
            if self._offload_exec is not None:
                slot = self._offload_exec.call("offload_put", block_id)
                if slot != -1:
                    self._release_host_entry(block.hash)
                    self._host_map[block.hash] = (slot, list(block.token_ids))
                    self.host_puts += 1
                else:
                    self.host_drops += 1
            del self.hash_to_block_id[block.hash]
        block.reset()
        self.used_block_ids.add(block_id)
        self.allocations += 1
        return block_id

    def _revive_from_host(self, h: int) -> int:
        slot, token_ids = self._host_map.pop(h)
        block_id = self._allocate_block()
        self._offload_exec.call("offload_get", slot, block_id)
        self._offload_exec.call("offload_release", slot)
        self.blocks[block_id].update(h, token_ids)
        self.hash_to_block_id[h] = block_id
        self.host_revives += 1
        return block_id

    def _deallocate_block(self, block_id: int):
        block = self.blocks[block_id]
        assert block.ref_count == 0
        self.used_block_ids.remove(block_id)
        if block.hash != -1:
            self._lru[block_id] = next(self._stamp)
        else:
            self._fresh[block_id] = next(self._stamp)
        self.reclaims += 1

    # ------------------------------------------------------------- admission
    def can_allocate(self, seq: Sequence, touch: bool = True) -> int:
        """Number of prefix blocks served from cache, or -1 if the sequence
        cannot be admitted.  The last (possibly partial) block is never a hit."""
        h = -1
        cached = 0
        new_blocks = seq.num_blocks
        for i in range(seq.num_blocks - 1):
            toks = seq.block_tokens(i)
            h = self.compute_hash(toks, h)
            bid = self.hash_to_block_id.get(h, -1)
            if bid != -1 and self.blocks[bid].token_ids == toks:
                cached += 1
                if touch and self.lru_enabled and bid in self._lru:
                    self._lru.move_to_end(bid)
                if bid in self.used_block_ids:
                    new_blocks -= 1
                continue
            if self._offload_exec is not None:
                entry = self._host_map.get(h)
                if entry is not None and entry[1] == toks:
                    cached += 1
                    continue
            break
        if self.num_free_blocks < new_blocks:
            return -1
        return cached

    def allocate(self, seq: Sequence, num_cached_blocks: int):
        assert num_cached_blocks >= 0, "can_allocate returned -1 (insufficient KV)"
        assert not seq.block_table
        self.prefix_cache_hit_tokens += num_cached_blocks * self.block_size
        h = -1
        for i in range(num_cached_blocks):
            h = self.compute_hash(seq.block_tokens(i), h)
            if h not in self.hash_to_block_id:
                seq.block_table.append(self._revive_from_host(h))
                continue
            bid = self.hash_to_block_id[h]
            block = self.blocks[bid]
            if bid in self.used_block_ids:
                block.ref_count += 1
            else:
                block.ref_count = 1
                self._take_specific(bid)
                self.used_block_ids.add(bid)
            seq.block_table.append(bid)
        for _ in range(num_cached_blocks, seq.num_blocks):
            seq.block_table.append(self._allocate_block())
        seq.cached_len = num_cached_blocks * self.block_size

    def deallocate(self, seq: Sequence):
        for bid in reversed(seq.block_table):
            block = self.blocks[bid]
            block.ref_count -= 1
            if block.ref_count == 0:
                self._deallocate_block(bid)
        seq.cached_len = 0
        seq.block_table.clear()

    def can_append(self, seq: Sequence) -> bool:
        return self.num_free_blocks >= (len(seq) % self.block_size == 1)

    def may_append(self, seq: Sequence):
        if len(seq) % self.block_size == 1:
            seq.block_table.append(self._allocate_block())

    # ------------------------------------------------ overlap (speculative)
    def _blocks_needed(self, seq: Sequence, launch_len: int) -> int:
        need = (launch_len - 1) // self.block_size + 1
        return max(0, need - len(seq.block_table))

    def can_append_at(self, seq: Sequence, launch_len: int) -> bool:
        return self.num_free_blocks >= self._blocks_needed(seq, launch_len)

    def total_launch_shortfall(self, seqs: list[Sequence], launch_lens: list[int]) -> int:
        """Blocks a whole speculative decode batch allocates sequentially; the
        sum (not each term) must fit the free pool."""
        return sum(self._blocks_needed(s, n) for s, n in zip(seqs, launch_lens))

    def may_append_at(self, seq: Sequence, launch_len: int):
        while self._blocks_needed(seq, launch_len) > 0:
            seq.block_table.append(self._allocate_block())

    def hash_blocks(self, seq: Sequence, num_new_tokens: int | None = None):
        """Register hashes of blocks that became full during the last step."""
        q = seq.chunk_len if num_new_tokens is None else num_new_tokens
        start = seq.cached_len // self.block_size
        end = (seq.cached_len + q) // self.block_size
        if start == end:
            return
        h = self.blocks[seq.block_table[start - 1]].hash if start > 0 else -1
        for i in range(start, end):
            block = self.blocks[seq.block_table[i]]
            toks = seq.block_tokens(i)
            h = self.compute_hash(toks, h)
            block.update(h, toks)
            if h in self._host_map:
                self._release_host_entry(h)
            self.hash_to_block_id[h] = block.block_id

    def metrics(self) -> dict:
        cap = len(self.blocks)
        used = len(self.used_block_ids)
        return {
            "kv_blocks_capacity": cap,
            "kv_blocks_used": used,
            "kv_cache_utilization": used / cap if cap else 0.0,
            "kv_prefix_hit_tokens_total": self.prefix_cache_hit_tokens,
            "kv_block_allocations_total": self.allocations,
            "kv_block_reclaims_total": self.reclaims,
            "kv_lru_size": len(self._lru),
            "kv_lru_evictions_total": self.evictions,
            "kv_lru_enabled": int(self.lru_enabled),
            "kv_offload_host_entries": len(self._host_map),
            "kv_offload_puts_total": self.host_puts,
            "kv_offload_revives_total": self.host_revives,
            "kv_offload_drops_total": self.host_drops,
        }

    def clear_prefix_cache(self):
        """Forget reusable hashes; blocks held by live requests keep their data."""
        if self._offload_exec is not None:
            for h in list(self._host_map):
                self._release_host_entry(h)
        self._host_map.clear()
        self.hash_to_block_id.clear()
        for block in self.blocks:
            block.hash = -1
            block.token_ids = []
        while self._lru:
            bid, stamp = self._lru.popitem(last=False)
            self._fresh[bid] = stamp

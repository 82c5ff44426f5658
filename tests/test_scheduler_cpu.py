"""Scheduler and BlockManager invariants, driven directly (no model).

Mirrors the reference's pure-CPU scheduler suites (tests/p8_scheduler_gaps.py,
p16_lru_evict.py, p16_priority_sched.py, p25_review_repro.py,
p30_kv_offload_hostmap.py) with tests of our own."""
import random
from types import SimpleNamespace

import pytest

from b200moe.engine.block_manager import BlockManager
from b200moe.engine.scheduler import Scheduler
from b200moe.engine.sequence import Sequence, SequenceStatus
from b200moe.sampling_params import SamplingParams

BS = 16


@pytest.fixture(autouse=True)
def _bs():
    Sequence.block_size = BS
    yield


def cfg(**kw):
    c = dict(max_num_seqs=8, max_num_batched_tokens=256, eos=-1, kvcache_block_size=BS,
             scheduler_policy="fcfs", prefill_chunk_size=32, scheduler_starvation_steps=4,
             num_kvcache_blocks=64, dp_size=1)
    c.update(kw)
    return SimpleNamespace(**c)


def seq(n, start=0, **sp):
    return Sequence(list(range(start, start + n)), SamplingParams(**sp))


def run_step(sch, batch, tok=7):
    return sch.postprocess(batch.sequences, [tok] * len(batch.sequences), batch.mode, None,
                           batch.query_lens, batch.prefill_flags)


# ------------------------------------------------------------ block manager
def test_prefix_hash_chain_and_refcounts():
    bm = BlockManager(16, BS)
    a = seq(40)
    assert bm.can_allocate(a) == 0
    bm.allocate(a, 0)
    bm.hash_blocks(a, 40)
    b = seq(40)  # same tokens: two full blocks hit, the partial third never does
    assert bm.can_allocate(b) == 2
    bm.allocate(b, 2)
    assert b.block_table[:2] == a.block_table[:2] and b.block_table[2] != a.block_table[2]
    assert bm.blocks[a.block_table[0]].ref_count == 2
    bm.deallocate(a)
    assert bm.blocks[b.block_table[0]].ref_count == 1
    bm.deallocate(b)
    assert bm.num_free_blocks == 16 and not bm.used_block_ids


def test_fresh_blocks_before_lru_and_touch_on_hit():
    bm = BlockManager(6, BS)
    cached = []
    for i in range(3):
        s = seq(16 + 1, start=1000 * (i + 1))  # one full block + 1
        bm.allocate(s, bm.can_allocate(s))
        bm.hash_blocks(s, 17)
        cached.append((s.block_table[0], list(s.tokens)))
        bm.deallocate(s)
    # all free; 3 cached blocks in LRU order (0 oldest)
    assert len(bm._lru) == 3
    # re-admit the first prefix: it is touched and becomes MRU
    s0 = Sequence(cached[0][1])
    assert bm.can_allocate(s0) == 1
    # allocating fresh blocks consumes the fresh tier before any cached block
    fresh_before = len(bm._fresh)
    b = bm._allocate_block()
    assert b not in dict(bm._lru) and len(bm._fresh) == fresh_before - 1
    # exhaust fresh blocks, then the coldest cached block (prefix 1, not the touched 0) is evicted
    while bm._fresh:
        bm._allocate_block()
    victim = bm._allocate_block()
    assert victim == cached[1][0]
    assert bm.evictions == 1


def test_fifo_mode(monkeypatch):
    monkeypatch.setenv("B200MOE_LRU_EVICT", "0")
    bm = BlockManager(4, BS)
    assert not bm.lru_enabled
    ids = [bm._allocate_block() for _ in range(4)]
    assert ids == [0, 1, 2, 3]


def test_speculative_cumulative_shortfall():
    bm = BlockManager(4, BS)
    seqs = [seq(16) for _ in range(2)]
    for s in seqs:
        bm.allocate(s, 0)
    # each needs one more block at launch length 17: per-seq fits (1 free), sum does not
    bm._allocate_block()
    assert all(bm.can_append_at(s, 17) for s in seqs)
    assert bm.total_launch_shortfall(seqs, [17, 17]) > bm.num_free_blocks


class FakeOffload:
    """Host pool stand-in mirroring slot accounting (reference test p30 hostmap)."""

    def __init__(self, slots):
        self.free = list(range(slots))
        self.in_use = set()
        self.calls = []

    def call(self, name, *args):
        self.calls.append(name)
        if name == "offload_put":
            if not self.free:
                return -1
            s = self.free.pop()
            self.in_use.add(s)
            return s
        if name == "offload_release":
            self.in_use.discard(args[0])
            self.free.append(args[0])
        return None


def test_offload_put_revive_and_slot_invariant():
    bm = BlockManager(3, BS)
    ex = FakeOffload(2)
    bm.set_offload_executor(ex)
    rng = random.Random(0)
    for step in range(40):
        s = Sequence([rng.randrange(4) for _ in range(BS)] + [1])
        n = bm.can_allocate(s)
        if n < 0:
            continue
        bm.allocate(s, n)
        bm.hash_blocks(s, len(s))
        bm.deallocate(s)
        assert len(ex.in_use) == len(bm._host_map)
        assert not set(bm._host_map) & set(bm.hash_to_block_id)
    assert bm.host_puts > 0


# ---------------------------------------------------------------- scheduler
def test_fcfs_prefill_first_and_chunk_only_first():
    sch = Scheduler(cfg(max_num_batched_tokens=100))
    a, b = seq(80), seq(80, start=500)
    sch.add(a)
    sch.add(b)
    batch = sch.schedule()
    assert batch.mode == "prefill" and batch.sequences == [a]
    assert batch.query_lens == [80]
    run_step(sch, batch)
    batch = sch.schedule()
    # b (80) does not fit the remaining 100? it does (only b waits) -> whole
    assert batch.sequences == [b]


def test_fcfs_first_sequence_chunked():
    sch = Scheduler(cfg(max_num_batched_tokens=50))
    a = seq(120)
    sch.add(a)
    b1 = sch.schedule()
    assert b1.query_lens == [50]
    run_step(sch, b1)
    b2 = sch.schedule()
    assert b2.query_lens == [50] and b2.prefill_flags == [True]
    run_step(sch, b2)
    b3 = sch.schedule()
    assert b3.query_lens == [20]
    run_step(sch, b3)
    assert a.output_len == 1
    assert sch.schedule().mode == "decode"


def test_stall_free_decode_first_and_bounded_chunks():
    sch = Scheduler(cfg(scheduler_policy="stall_free", prefill_chunk_size=32, max_num_batched_tokens=64))
    a = seq(20)
    sch.add(a)
    run_step(sch, sch.schedule())
    b = seq(100, start=300)
    sch.add(b)
    batch = sch.schedule()
    assert batch.mode == "mixed"
    assert batch.sequences[0] is a and batch.prefill_flags == [False, True]
    assert batch.query_lens == [1, 32]


def test_stall_free_skips_unadmittable_head():
    sch = Scheduler(cfg(scheduler_policy="stall_free", num_kvcache_blocks=4, max_num_batched_tokens=256,
                        prefill_chunk_size=256))
    big, small = seq(200), seq(10, start=900)
    sch.add(big)
    sch.add(small)
    batch = sch.schedule()
    assert batch.sequences == [small]
    assert sch.kv_admission_skips_total == 1 and list(sch.waiting) == [big]


def test_priority_and_starvation():
    sch = Scheduler(cfg(scheduler_policy="stall_free", max_num_batched_tokens=16, prefill_chunk_size=16,
                        scheduler_starvation_steps=3))
    low = seq(16, priority=5)
    sch.add(low)
    order = []
    for i in range(6):
        sch.add(seq(16, start=100 * (i + 1), priority=0))
        batch = sch.schedule()
        order.append(max((s.params.priority for s, f in zip(batch.sequences, batch.prefill_flags) if f), default=None))
        run_step(sch, batch)
    assert 5 in order, "the starved low-priority request must eventually run"
    assert order[0] == 0 and order.index(5) >= 2


def test_preempt_lowest_priority_newest():
    sch = Scheduler(cfg(num_kvcache_blocks=3, max_num_batched_tokens=256))
    a = seq(16, priority=0)
    b = seq(16, start=100, priority=1)
    sch.add(a)
    sch.add(b)
    run_step(sch, sch.schedule())  # both prefilled: 2 blocks + 1 free
    batch = sch.schedule()  # both need a new block at len 17 -> one preemption
    assert batch.mode == "decode"
    assert sch.preemptions == 1 and b.status == SequenceStatus.WAITING and a in batch.sequences


def test_cancel_frees_blocks():
    sch = Scheduler(cfg())
    a = seq(40)
    sch.add(a)
    run_step(sch, sch.schedule())
    used = len(sch.block_manager.used_block_ids)
    assert used > 0
    assert sch.cancel(a.seq_id)
    assert a.finish_reason == "cancelled" and not sch.block_manager.used_block_ids
    assert not sch.cancel(12345)


def test_finish_on_eos_stop_length():
    sch = Scheduler(cfg(eos=99))
    a = seq(10, max_tokens=3)
    b = seq(10, start=50, max_tokens=10, stop_token_ids=[42])
    c = seq(10, start=70, max_tokens=10)
    for s in (a, b, c):
        sch.add(s)
    batch = sch.schedule()
    events = sch.postprocess(batch.sequences, [5, 42, 99], "prefill", None, batch.query_lens, batch.prefill_flags)
    fin = {e[0]: e[2] for e in events}
    assert fin[b.seq_id] and b.finish_reason == "stop"
    assert fin[c.seq_id] and c.finish_reason == "stop"
    assert not fin[a.seq_id]
    while not a.is_finished:
        run_step(sch, sch.schedule(), tok=5)
    assert a.finish_reason == "length" and a.output_len == 3


def test_speculative_schedule_defers_instead_of_preempting():
    sch = Scheduler(cfg(num_kvcache_blocks=2))
    a, b = seq(16), seq(16, start=100)
    sch.add(a)
    sch.add(b)
    batch = sch.schedule()
    run_step(sch, batch)
    nxt = sch.schedule(speculative=True, inflight=[a, b])
    assert nxt.mode == "defer" and sch.preemptions == 0


def test_dp_ranks_bind_and_balance():
    sch = Scheduler(cfg(dp_size=2, num_kvcache_blocks=8, max_num_batched_tokens=64), dp_size=2)
    seqs = [seq(20, start=100 * i) for i in range(4)]
    for s in seqs:
        sch.add(s)
    batch = sch.schedule()
    ranks = sorted(s.dp_rank for s in batch.sequences)
    assert set(ranks) == {0, 1}
    for r, bm in enumerate(sch.block_managers):
        owned = [s for s in batch.sequences if s.dp_rank == r]
        assert len(bm.used_block_ids) == sum(len(s.block_table) for s in owned)
    m = sch.metrics()
    assert m["kv_blocks_capacity"] == 16


# ------------------------------------------------------------------- fuzzer
def _check_invariants(sch, live, offloads, carried):
    for r, bm in enumerate(sch.block_managers):
        fresh, lru, used = set(bm._fresh), set(bm._lru), bm.used_block_ids
        assert not fresh & lru and not (fresh | lru) & used
        assert fresh | lru | used == set(range(len(bm.blocks)))
        refs = [0] * len(bm.blocks)
        for s in live:
            if max(s.dp_rank, 0) != r or not s.block_table:
                continue
            assert len(set(s.block_table)) == len(s.block_table), "a block twice in one table"
            assert len(s.block_table) * BS >= s.cached_len + s.chunk_len
            for b in s.block_table:
                refs[b] += 1
        for b, blk in enumerate(bm.blocks):
            assert blk.ref_count == refs[b], (b, blk.ref_count, refs[b])
            assert (refs[b] > 0) == (b in used)
            if refs[b] == 0:
                carried[r].discard(b)
            elif refs[b] > 1 and b not in carried[r]:
                assert blk.hash != -1, "only hashed full blocks are shared"
        for h, b in bm.hash_to_block_id.items():
            assert bm.blocks[b].hash == h
        if offloads:
            ex = offloads[r]
            assert len(ex.in_use) == len(bm._host_map)
            assert not set(bm._host_map) & set(bm.hash_to_block_id)


@pytest.mark.parametrize("policy", ["fcfs", "stall_free", "stall_free_lpm"])
@pytest.mark.parametrize("lru,offload,dp", [(True, False, 1), (False, False, 1), (True, True, 1), (True, False, 2)])
def test_scheduler_block_manager_fuzz(policy, lru, offload, dp, monkeypatch):
    """Random arrivals sharing prefixes, chunked prefills, preemption under a
    small pool, cancels, prefix-cache clears and EOS finishes; the block pool
    invariants (tiers partition the ids, reference counts equal table
    occurrences, only hashed blocks are shared, offload slots match the host
    map) hold after every step, and every block is free at the end."""
    monkeypatch.setenv("B200MOE_LRU_EVICT", "1" if lru else "0")
    rng = random.Random(hash((policy, lru, offload, dp)) & 0xFFFF)
    sch = Scheduler(cfg(scheduler_policy=policy, num_kvcache_blocks=24, max_num_batched_tokens=64,
                        prefill_chunk_size=32, max_num_seqs=6, eos=3, dp_size=dp), dp_size=dp)
    offloads = []
    if offload:
        for bm in sch.block_managers:
            offloads.append(FakeOffload(6))
            bm.set_offload_executor(offloads[-1])
    prefixes = [[rng.randrange(5, 50) for _ in range(rng.choice([16, 32, 48]))] for _ in range(4)]
    pending = []
    for _ in range(60):
        n = rng.randrange(1, 100)
        base = rng.choice(prefixes) if rng.random() < 0.6 else []
        toks = (base + [rng.randrange(5, 50) for _ in range(n)])[:120]
        pending.append(Sequence(toks, SamplingParams(max_tokens=rng.randrange(1, 24), ignore_eos=rng.random() < 0.5,
                                                     priority=rng.randrange(4), temperature=0.0)))
    all_seqs = list(pending)
    carried = [set() for _ in range(dp)]
    steps = 0
    while pending or not sch.is_finished():
        steps += 1
        assert steps < 5000, "scheduler made no progress"
        for _ in range(rng.randrange(0, 3)):
            if pending:
                sch.add(pending.pop())
        if rng.random() < 0.05:
            live = list(sch.waiting) + list(sch.running)
            if live:
                assert sch.cancel(rng.choice(live).seq_id)
        if rng.random() < 0.01:
            # blocks held across a clear keep their sharers but lose their hash
            for r, bm in enumerate(sch.block_managers):
                carried[r] |= set(bm.used_block_ids)
            sch.clear_prefix_cache()
        batch = sch.schedule()
        live = list(sch.waiting) + list(sch.running)
        _check_invariants(sch, live, offloads, carried)
        if batch.sequences:
            toks = [rng.choice([3, 7, 11, 13]) for _ in batch.sequences]
            sch.postprocess(batch.sequences, toks, batch.mode, None, batch.query_lens, batch.prefill_flags)
        live = list(sch.waiting) + list(sch.running)
        _check_invariants(sch, live, offloads, carried)
    for bm in sch.block_managers:
        assert not bm.used_block_ids and bm.num_free_blocks == len(bm.blocks)
    assert all(s.finish_reason in ("length", "stop", "cancelled") for s in all_seqs)
    assert {s.finish_reason for s in all_seqs} >= {"length", "stop"}
    assert sum(bm.prefix_cache_hit_tokens for bm in sch.block_managers) > 0


def test_build_plan_matches_per_row_definition():
    """The vectorised decode rows of build_plan equal the per-row definition: decode
    rows first (their id is the last token, or 0 with a feed row when the token is
    still on the device), positions, KV slots through the block table, context
    lengths, padded block tables; prefill rows continue from their cached length."""
    import random as rnd
    import numpy as np
    from b200moe.engine.sequence import Sequence
    from b200moe.engine.step_plan import build_plan
    from b200moe.sampling_params import SamplingParams
    rng = rnd.Random(5)
    bs = 16
    Sequence.block_size = bs
    seqs, qlens, flags = [], [], []
    for j in range(30):
        n = rng.randint(1, 90)
        s = Sequence([rng.randrange(1000) for _ in range(n)], SamplingParams(temperature=0.0))
        prefill = j % 4 == 0
        s.cached_len = rng.randint(0, n - 1) if prefill else n - 1
        q = (n - s.cached_len) if prefill else 1
        s.block_table = rng.sample(range(500), -(-(n + 1) // bs))
        seqs.append(s)
        qlens.append(q)
        flags.append(prefill)
    feed = {id(s): k for k, s in enumerate(seqs) if not flags[k] and k % 3 == 0}
    plan = build_plan(seqs, qlens, flags, bs, max_blocks=8, feed=feed)
    order = sorted(range(len(seqs)), key=lambda i: (flags[i], i))
    ids, pos, slots, lens, src = [], [], [], [], []
    for i in order:
        s = seqs[i]
        if flags[i]:
            start = s.cached_len
            toks = s.tokens[start:start + qlens[i]]
            fs = [-1] * qlens[i]
        elif id(s) in feed:
            start, toks, fs = len(s), [0], [feed[id(s)]]
        else:
            start, toks, fs = len(s) - 1, [s.last], [-1]
        p = list(range(start, start + qlens[i]))
        ids += toks
        pos += p
        slots += [s.block_table[x // bs] * bs + x % bs for x in p]
        lens.append(start + qlens[i])
        src += fs
    assert plan.num_decode == sum(1 for f in flags if not f)
    assert plan.input_ids.tolist() == ids and plan.positions.tolist() == pos
    assert plan.slot_mapping.tolist() == slots and plan.seq_lens.tolist() == lens
    assert plan.feed_src.tolist() == src
    for r, i in enumerate(order):
        bt = seqs[i].block_table
        assert plan.block_tables[r, :len(bt)].tolist() == bt and not plan.block_tables[r, len(bt):].any()
    assert plan.rows.tolist() == order and np.all(np.diff(plan.cu_seqlens_q) == [qlens[i] for i in order])

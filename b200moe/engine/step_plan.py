"""Host-side step plan: the flat arrays one forward step needs.

The driver turns a :class:`ScheduledBatch` into one plan per rank (with
data-parallel attention every rank runs its own rows).  A plan is a handful of
numpy arrays, cheap to ship to worker processes and packed into ONE pinned
int32 buffer on the device side, so a step costs a single host-to-device copy
(the reference builds ~8 tensors with separate pinned copies,
nanovllm/engine/model_runner.py:595-699).

Row order inside a plan: decode rows (one new token) first, then prefill
rows; ``rows`` maps plan rows back to batch rows.
"""
from __future__ import annotations

from dataclasses import dataclass

import itertools

import numpy as np


@dataclass
class StepPlan:
    input_ids: np.ndarray        # int32 [T]
    positions: np.ndarray        # int32 [T]
    slot_mapping: np.ndarray     # int32 [T]
    cu_seqlens_q: np.ndarray     # int32 [B + 1]
    seq_lens: np.ndarray         # int32 [B]
    block_tables: np.ndarray     # int32 [B, max_blocks]
    num_decode: int
    max_q_len: int
    max_seq_len: int
    rows: np.ndarray             # int32 [B]: batch row of each plan row
    temperature: np.ndarray      # float32 [B]
    top_k: np.ndarray | None = None
    top_p: np.ndarray | None = None
    min_p: np.ndarray | None = None
    seeds: np.ndarray | None = None
    offsets: np.ndarray | None = None
    # penalties: flat (row, token, generated count) triples + per-row coefficients
    pen_rows: np.ndarray | None = None
    pen_ids: np.ndarray | None = None
    pen_counts: np.ndarray | None = None
    presence: np.ndarray | None = None
    frequency: np.ndarray | None = None
    repetition: np.ndarray | None = None
    logprobs_k: int = 0
    grammar_rows: np.ndarray | None = None
    grammar_mask: np.ndarray | None = None   # int32 [n, words] allowed-token bitmask
    # int32 [T]: row of the previous step whose sampled token (still on the
    # device) is this token's id, -1 = use input_ids (launch-ahead decode)
    feed_src: np.ndarray | None = None

    @property
    def num_rows(self) -> int:
        return int(self.seq_lens.shape[0])

    @property
    def num_tokens(self) -> int:
        return int(self.input_ids.shape[0])

    @property
    def is_pure_decode(self) -> bool:
        return self.num_decode == self.num_rows and self.num_rows > 0

    @property
    def all_greedy(self) -> bool:
        return bool(self.temperature.size == 0 or (self.temperature < 1e-3).all())

    @property
    def needs_full_sampler(self) -> bool:
        return (not self.all_greedy or self.pen_rows is not None or self.grammar_rows is not None
                or self.logprobs_k > 0)


def empty_plan(max_blocks: int = 1) -> StepPlan:
    z = np.zeros(0, np.int32)
    return StepPlan(z, z, z, np.zeros(1, np.int32), z, np.zeros((0, max_blocks), np.int32), 0, 0, 0, z,
                    np.zeros(0, np.float32))


def build_plan(seqs, query_lens, prefill_flags, block_size: int, max_blocks: int | None = None,
               rows: list[int] | None = None, feed: dict | None = None) -> StepPlan:
    """Plan for the given batch rows (one rank's share of a batch).

    ``feed``: {id(sequence): row of the previous step's plan} for decode rows whose
    input token is the previous step's sampled token, not yet read back to the host
    (the sequence is one token longer than its host state)."""
    n = len(seqs)
    rows = list(range(n)) if rows is None else rows
    order = sorted(range(n), key=lambda i: (bool(prefill_flags[i]), i))
    nd = sum(1 for i in range(n) if not prefill_flags[i])
    qlens = np.fromiter((query_lens[i] for i in order), dtype=np.int64, count=n)
    T = int(qlens.sum())
    cu = np.zeros(n + 1, np.int32)
    np.cumsum(qlens, out=cu[1:])
    ids = np.empty(T, np.int32)
    pos = np.empty(T, np.int32)
    slots = np.empty(T, np.int32)
    seq_lens = np.empty(n, np.int32)
    mb = max_blocks or max((len(seqs[i].block_table) for i in order), default=1) or 1
    tables = np.zeros((n, mb), np.int32)
    feed_src = np.full(T, -1, np.int32) if feed else None
    # decode rows (first nd of ``order``, one token each): vectorised -- in steady decoding they
    # are nearly every row, and per-row numpy calls cost about 10 us each
    if nd:
        dec = [seqs[i] for i in order[:nd]]
        start = np.fromiter((len(sq) - 1 for sq in dec), np.int64, nd)
        if feed:
            fsrc = np.fromiter((feed.get(id(sq), -1) for sq in dec), np.int64, nd)
            fed = fsrc >= 0
            start += fed                       # the token sampled by the step in flight
            feed_src[:nd] = fsrc
            ids[:nd] = np.fromiter((0 if f else sq.last for sq, f in zip(dec, fed.tolist())), np.int32, nd)
        else:
            ids[:nd] = np.fromiter((sq.last for sq in dec), np.int32, nd)
        nbt = np.fromiter((len(sq.block_table) for sq in dec), np.int64, nd)
        if int(nbt.max()) > mb or (nbt < start // block_size + 1).any():
            r = int(np.argmax((nbt > mb) | (nbt < start // block_size + 1)))
            raise RuntimeError(f"seq {dec[r].seq_id}: block table has {int(nbt[r])} blocks, step needs "
                               f"{int(start[r]) // block_size + 1} (max {mb})")
        for r, sq in enumerate(dec):
            tables[r, :len(sq.block_table)] = sq.block_table
        pos[:nd] = start
        slots[:nd] = tables[np.arange(nd), start // block_size] * block_size + start % block_size
        seq_lens[:nd] = start + 1
    for r in range(nd, n):
        i = order[r]
        s = seqs[i]
        q = int(qlens[r])
        a, b = int(cu[r]), int(cu[r + 1])
        start = s.cached_len
        ids[a:b] = s.tokens[start:start + q]
        p = np.arange(start, start + q, dtype=np.int64)
        pos[a:b] = p
        bt = np.asarray(s.block_table, dtype=np.int64)
        need = int(p[-1]) // block_size + 1
        if bt.size < need or bt.size > mb:
            raise RuntimeError(f"seq {s.seq_id}: block table has {bt.size} blocks, step needs {need} (max {mb})")
        slots[a:b] = bt[p // block_size] * block_size + p % block_size
        seq_lens[r] = start + q
        tables[r, :bt.size] = bt
    temps = np.fromiter((seqs[i].params.temperature for i in order), dtype=np.float32, count=n)
    plan = StepPlan(ids, pos, slots, cu, seq_lens, tables, nd,
                    int(qlens[nd:].max()) if n > nd else 0,
                    int(seq_lens.max()) if n else 0,
                    np.asarray([rows[i] for i in order], np.int32), temps)
    plan.feed_src = feed_src
    _sampling_meta(plan, [seqs[i] for i in order])
    return plan


def validate_plan(plan: StepPlan, num_blocks: int, block_size: int, vocab: int, feed_rows: int) -> None:
    """Reject a plan whose indices would make a kernel read or write outside its
    buffers: block ids outside the pool, KV slots outside the pool, token ids
    outside the vocabulary, feed rows outside the previous step's token buffer.
    The kernels trust these indices (the embedding kernel alone re-checks its
    ids), so this host check stands in for device bounds checks on the hot path.
    A few vectorised min / max reductions: microseconds for a 256-row plan."""
    if plan.num_rows == 0:
        return

    def bad(what, lo, hi, arr):
        raise ValueError(f"step plan: {what} outside [{lo}, {hi}) (min {int(arr.min())}, max {int(arr.max())})")

    if plan.block_tables.size and (plan.block_tables.min() < 0 or plan.block_tables.max() >= num_blocks):
        bad("block id", 0, num_blocks, plan.block_tables)
    limit = num_blocks * block_size
    if plan.slot_mapping.size and (plan.slot_mapping.min() < 0 or plan.slot_mapping.max() >= limit):
        bad("KV slot", 0, limit, plan.slot_mapping)
    if plan.input_ids.size and (plan.input_ids.min() < 0 or plan.input_ids.max() >= vocab):
        bad("token id", 0, vocab, plan.input_ids)
    if plan.feed_src is not None and plan.feed_src.size and plan.feed_src.max() >= feed_rows:
        bad("feed row", -1, feed_rows, plan.feed_src)
    cap = plan.block_tables.shape[1] * block_size
    if plan.seq_lens.min() < 1 or plan.seq_lens.max() > cap:
        bad("context length", 1, cap + 1, plan.seq_lens)


def _sampling_meta(plan: StepPlan, seqs):
    n = len(seqs)
    if any(s.params.top_k != -1 for s in seqs):
        plan.top_k = np.fromiter((s.params.top_k for s in seqs), np.int32, n)
    if any(s.params.top_p < 1.0 for s in seqs):
        plan.top_p = np.fromiter((s.params.top_p for s in seqs), np.float32, n)
    if any(s.params.min_p > 0.0 for s in seqs):
        plan.min_p = np.fromiter((s.params.min_p for s in seqs), np.float32, n)
    if not plan.all_greedy:
        plan.seeds = np.fromiter(((s.params.seed if s.params.seed is not None else s.seq_id * 7919 + 17) for s in seqs),
                                 np.int64, n)
        plan.offsets = np.fromiter((s.num_tokens for s in seqs), np.int64, n)
    plan.logprobs_k = max((s.params.logprobs or 0 for s in seqs), default=0)
    penalised = [(r, s) for r, s in enumerate(seqs) if s.penalty is not None]
    if penalised:
        rws, ids, cnt = [], [], []
        pres = np.zeros(n, np.float32)
        freq = np.zeros(n, np.float32)
        rep = np.ones(n, np.float32)
        for r, s in penalised:
            p = s.params
            pres[r], freq[r], rep[r] = p.presence_penalty, p.frequency_penalty, p.repetition_penalty
            generated = s.penalty.generated
            # the repetition penalty covers prompt tokens too; its table includes every generated token
            table = (s.penalty.seen(itertools.islice(s.tokens, s.prompt_len)) if p.repetition_penalty != 1.0
                     else generated)
            for t in table:
                rws.append(r)
                ids.append(t)
                cnt.append(generated.get(t, 0))
        if rws:
            plan.pen_rows = np.asarray(rws, np.int32)
            plan.pen_ids = np.asarray(ids, np.int32)
            plan.pen_counts = np.asarray(cnt, np.int32)
            plan.presence, plan.frequency, plan.repetition = pres, freq, rep
    g_rows = [r for r, s in enumerate(seqs) if s.grammar is not None]
    if g_rows:
        plan.grammar_rows = np.asarray(g_rows, np.int32)


PACK_FIELDS = ("input_ids", "positions", "slot_mapping", "cu_seqlens_q", "seq_lens", "logits_indices",
               "prefill_cu", "feed_src", "block_tables")


def pack_plan(plan: StepPlan, out: np.ndarray | None = None) -> tuple[np.ndarray, dict]:
    """Concatenate the int32 arrays into one buffer; returns (buffer, {name: (offset, size)})."""
    nd = plan.num_decode
    cu = plan.cu_seqlens_q
    parts = {
        "input_ids": plan.input_ids, "positions": plan.positions, "slot_mapping": plan.slot_mapping,
        "cu_seqlens_q": cu, "seq_lens": plan.seq_lens,
        "logits_indices": (cu[1:] - 1).astype(np.int32),
        "prefill_cu": (cu[nd:] - cu[nd]).astype(np.int32),
        "feed_src": plan.feed_src if plan.feed_src is not None else np.full(plan.input_ids.size, -1, np.int32),
        "block_tables": plan.block_tables.reshape(-1),
    }
    total = sum(p.size for p in parts.values())
    buf = out[:total] if out is not None and out.size >= total else np.empty(total, np.int32)
    offs = {}
    o = 0
    for name in PACK_FIELDS:
        arr = parts[name]
        buf[o:o + arr.size] = arr
        offs[name] = (o, arr.size)
        o += arr.size
    return buf, offs


def pack_sampling(plan: StepPlan, out: np.ndarray | None = None) -> tuple[np.ndarray, dict]:
    """Every per-row sampling array of a step in ONE int32 buffer, so the sampler's
    inputs cross to the device in a single copy: temperature, top-k / top-p / min-p,
    Philox seeds and counters, penalty triples and coefficients, and the grammar
    bitmasks with the mask index of each row.  Floats travel as their bits; int64
    fields start on an even word so their device views are 8-byte aligned.
    Returns (buffer, {name: (word offset, words, numpy dtype)})."""
    B = plan.num_rows
    parts: list[tuple[str, np.ndarray]] = [("temperature", plan.temperature.astype(np.float32, copy=False))]
    for name in ("top_k", "top_p", "min_p"):
        arr = getattr(plan, name)
        if arr is not None:
            parts.append((name, arr))
    if not plan.all_greedy:
        seeds = plan.seeds if plan.seeds is not None else np.zeros(B, np.int64)
        parts.append(("seeds", seeds.astype(np.int64, copy=False)))
        if plan.offsets is not None:
            parts.append(("offsets", plan.offsets.astype(np.int64, copy=False)))
    if plan.pen_rows is not None:
        parts += [("pen_rows", plan.pen_rows), ("pen_ids", plan.pen_ids), ("pen_counts", plan.pen_counts),
                  ("presence", plan.presence), ("frequency", plan.frequency), ("repetition", plan.repetition)]
    if plan.grammar_rows is not None:
        row_mask = np.full(B, -1, np.int32)
        row_mask[plan.grammar_rows] = np.arange(plan.grammar_rows.size, dtype=np.int32)
        parts += [("allow_row", row_mask), ("allow", plan.grammar_mask.astype(np.int32, copy=False).reshape(-1))]
    words = 0
    layout = {}
    for name, arr in parts:
        if arr.dtype.itemsize == 8 and words % 2:
            words += 1
        n = arr.size * arr.dtype.itemsize // 4
        layout[name] = (words, n, arr.dtype)
        words += n
    buf = out[:words] if out is not None and out.size >= words else np.empty(words, np.int32)
    for name, arr in parts:
        o, n, _ = layout[name]
        buf[o:o + n] = np.ascontiguousarray(arr).view(np.int32).reshape(-1)
    return buf, layout

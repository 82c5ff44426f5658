"""Backend-equivalence probe: the evidence behind the five-layer equivalence gate.

    python -m b200moe.equivalence --model qwen3-30b-a3b --random-init --switch attention \
        --baseline sdpa --candidate paged --prompts 100 --max-tokens 128 --output eq.json

The layers follow the reference's numerics policy (docs/numerics-policy.md §3,
scripts/p6_decide_attention_equivalence.py) and apply to any backend switch
(``attention``: sdpa vs paged kernels; ``moe``: per-expert loop vs grouped kernel):

* **L1 structural** (attention only): the native kernels against the fp32
  reference over page-boundary lengths, shuffled pages and a poisoned tail
  (garbage past each sequence's last key) -> ``max_abs``.
* **L2 numerical**: the baseline's greedy continuations are scored teacher-
  forced (same token prefix) under both backends; a *flip* is a position
  whose top-1 differs.  Reported: flip rate and the baseline's logit gap
  between the two choices at every flip (the gate wants flips only at
  near-ties).
* **L3 output**: greedy outputs of both backends: first-token agreement,
  degenerate outputs (a token or short n-gram looping), longest common
  prefix, token agreement and edit distance (the last three reported only:
  after one near-tie flip the continuations legitimately diverge).
* **L4 self-determinism**: every backend repeated; outputs must be identical.
L5 (serving SLOs) comes from the online benchmark and is gated separately.
"""
from __future__ import annotations

import argparse
import json
import random
from pathlib import Path

import torch

from b200moe.benchmarking import percentile


# ----------------------------------------------------------------- helpers
def longest_common_prefix(a: list[int], b: list[int]) -> int:
    n = 0
    for x, y in zip(a, b):
        if x != y:
            break
        n += 1
    return n


def edit_distance(a: list[int], b: list[int]) -> int:
    """Levenshtein distance over token ids (two-row dynamic programme)."""
    prev = list(range(len(b) + 1))
    for i, x in enumerate(a, 1):
        cur = [i] + [0] * len(b)
        for j, y in enumerate(b, 1):
            cur[j] = min(prev[j] + 1, cur[j - 1] + 1, prev[j - 1] + (x != y))
        prev = cur
    return prev[-1]


def is_degenerate(tokens: list[int], run: int = 16, max_period: int = 4) -> bool:
    """True when the tail repeats one token or an n-gram (n <= max_period) for
    at least ``run`` tokens: the looping failure mode of broken numerics."""
    if len(tokens) < run:
        return False
    tail = tokens[-run:]
    return any(all(tail[i] == tail[i % p] for i in range(run)) for p in range(1, max_period + 1))


def _set_backend(llm, switch: str, name: str):
    llm.executor.call("set_attention_backend" if switch == "attention" else "set_moe_backend", name)


def _greedy(llm, prompts, max_tokens):
    from b200moe import SamplingParams
    sp = SamplingParams(temperature=0.0, max_tokens=max_tokens, ignore_eos=True)
    return [list(o["token_ids"]) for o in llm.generate(prompts, sp, use_tqdm=False)]


# ----------------------------------------------------------------- layers
def structural_check(device: str | None = None, seed: int = 0) -> dict:
    """L1: native decode / prefill attention against the fp32 reference on
    adversarial paging layouts; CPU-only hosts report the reference path."""
    from b200moe import ops
    from b200moe.engine.kv_cache import KVPool
    dev = device or ("cuda" if torch.cuda.is_available() else "cpu")
    g = torch.Generator(device="cpu").manual_seed(seed)
    D, nq, nkv, bs = 128, 32, 4, 16
    lens = [1, bs - 1, bs, bs + 1, 3 * bs, 5 * bs + 7]
    nb = sum(-(-L // bs) for L in lens) + 2
    pool = KVPool(nb, 1, nkv, bs, D, torch.bfloat16, dev)
    pool.data.copy_((torch.randn(pool.data.shape, generator=g) * 30).to(torch.bfloat16))  # poison everything
    perm = torch.randperm(nb - 1, generator=g).tolist()  # shuffled pages
    tables = torch.zeros(len(lens), max(-(-L // bs) for L in lens), dtype=torch.int32)
    i = 0
    layer = pool.layer(0)
    for b, L in enumerate(lens):
        n = -(-L // bs)
        tables[b, :n] = torch.tensor(perm[i:i + n])
        i += n
        pos = torch.arange(L)
        slots = (tables[b][pos // bs].long() * bs + pos % bs).to(torch.int32).to(dev)
        # V ~ 0.05 N(0, 1) keeps outputs below ~0.2, where half a bf16 ulp is ~5e-4,
        # so the 2e-3 bound measures the kernel rather than output rounding
        layer.store(slots, torch.randn(L, nkv, D, generator=g).to(torch.bfloat16).to(dev),
                    (0.05 * torch.randn(L, nkv, D, generator=g)).to(torch.bfloat16).to(dev))
    tables = tables.to(dev)
    seq = torch.tensor(lens, dtype=torch.int32, device=dev)
    q = torch.randn(len(lens), nq, D, generator=g).to(torch.bfloat16).to(dev)
    B, scale = len(lens), D ** -0.5
    ref = torch.empty(B, nq, D, device=dev)
    ops._attention_ref(q, layer, tables, seq, torch.arange(B + 1, dtype=torch.int32), scale, ref)
    out = torch.empty(B, nq, D, dtype=torch.bfloat16, device=dev)
    ws = (torch.empty(B * nq * 4, D, device=dev), torch.empty(B * nq * 4, device=dev),
          torch.empty(B * nq * 4, device=dev))
    ops.decode_attention(q, layer, tables, seq, scale, out, 64, 4, ws)
    dec = (out.float() - ref).abs().max().item()
    cu = torch.tensor([0] + list(torch.tensor(lens).cumsum(0)), dtype=torch.int32, device=dev)
    qp = torch.randn(int(cu[-1]), nq, D, generator=g).to(torch.bfloat16).to(dev)
    refp = torch.empty(qp.shape, device=dev)
    ops._attention_ref(qp, layer, tables, seq, cu.cpu(), scale, refp)
    outp = torch.empty(qp.shape, dtype=torch.bfloat16, device=dev)
    ops.prefill_attention(qp, layer, cu, seq, tables, max(lens), scale, outp)
    pre = (outp.float() - refp).abs().max().item()
    return {"device": dev, "decode_max_abs": dec, "prefill_max_abs": pre, "max_abs": max(dec, pre),
            "lengths": lens, "block_size": bs}


def teacher_forced(llm, switch, baseline, candidate, prompts, continuations) -> dict:
    """L2: top-1 flips between backends at the generated positions of the baseline's outputs."""
    flips, compared, margins = 0, 0, []
    for prompt, cont in zip(prompts, continuations):
        seq = list(prompt) + list(cont)
        logits = {}
        for name in (baseline, candidate):
            _set_backend(llm, switch, name)
            logits[name] = llm.executor.call("score_tokens", seq)
        llm.scheduler.clear_prefix_cache()  # scoring overwrote low KV blocks
        lo = len(prompt) - 1
        a, b = logits[baseline][lo:len(seq) - 1], logits[candidate][lo:len(seq) - 1]
        ta, tb = a.argmax(-1), b.argmax(-1)
        diff = (ta != tb).nonzero().flatten().tolist()
        flips += len(diff)
        compared += len(ta)
        for i in diff:
            margins.append(float(a[i, ta[i]] - a[i, tb[i]]))
    _set_backend(llm, switch, baseline)
    return {"flips": flips, "compared_positions": compared, "flip_rate": flips / compared if compared else 0.0,
            "flip_margins": margins, "flip_margin_max": max(margins) if margins else 0.0}


def run_probe(llm, switch: str, baseline: str, candidate: str, prompts: list, max_tokens: int,
              repeats: int = 3, l1: bool = True, l2: bool = True) -> dict:
    outs, determinism = {}, {}
    for name in (baseline, candidate):
        _set_backend(llm, switch, name)
        runs = []
        for r in range(repeats):
            if r:
                llm.scheduler.clear_prefix_cache()
            runs.append(_greedy(llm, prompts, max_tokens))
        outs[name] = runs[0]
        determinism[name] = all(x == runs[0] for x in runs)
    _set_backend(llm, switch, baseline)
    A, B = outs[baseline], outs[candidate]
    lcps = [longest_common_prefix(x, y) for x, y in zip(A, B)]
    eds = [edit_distance(x, y) / max(len(x), 1) for x, y in zip(A, B)]
    comparison = {
        "requests": len(A),
        "first_token_agreement_rate": sum(x[:1] == y[:1] for x, y in zip(A, B)) / max(len(A), 1),
        "degenerate_baseline": sum(map(is_degenerate, A)), "degenerate_candidate": sum(map(is_degenerate, B)),
        "request_token_identical": sum(x == y for x, y in zip(A, B)) / max(len(A), 1),
        "request_token_agreement_mean": sum(sum(p == q for p, q in zip(x, y)) / max(len(x), 1)
                                            for x, y in zip(A, B)) / max(len(A), 1),
        "lcp_p50": percentile(lcps, 0.5), "lcp_mean": sum(lcps) / max(len(lcps), 1),
        "edit_distance_ratio_p50": percentile(eds, 0.5), "edit_distance_ratio_max": max(eds) if eds else 0.0,
    }
    payload = {"schema_version": 1, "switch": switch, "baseline": baseline, "candidate": candidate,
               "max_tokens": max_tokens, "repeats": repeats, "comparison": comparison, "determinism": determinism,
               "samples": [{"prompt_len": len(p), "baseline": a, "candidate": b}
                           for p, a, b in list(zip(prompts, A, B))[:12]]}
    if l1 and switch == "attention":
        payload["l1"] = structural_check()
    if l2:
        payload["l2"] = teacher_forced(llm, switch, baseline, candidate, prompts, A)
    return payload


def main(argv=None):
    p = argparse.ArgumentParser(description="backend-equivalence probe (gate evidence)")
    p.add_argument("--model", default="tiny-moe")
    p.add_argument("--random-init", action="store_true")
    p.add_argument("--device", default=None)
    p.add_argument("--switch", choices=("attention", "moe"), default="attention")
    p.add_argument("--baseline", default=None)
    p.add_argument("--candidate", default=None)
    p.add_argument("--prompts", type=int, default=16)
    p.add_argument("--prompt-len", type=int, default=64)
    p.add_argument("--max-tokens", type=int, default=32)
    p.add_argument("--repeats", type=int, default=3)
    p.add_argument("--no-l2", action="store_true")
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--kvcache-block-size", type=int, default=16)
    p.add_argument("--output", default="equivalence.json")
    a = p.parse_args(argv)
    base = a.baseline or ("sdpa" if a.switch == "attention" else "loop")
    cand = a.candidate or ("paged" if a.switch == "attention" else "fused")
    from b200moe import LLM
    kw = dict(enforce_eager=True, kvcache_block_size=a.kvcache_block_size, max_num_seqs=max(a.prompts, 1),
              max_model_len=a.prompt_len + a.max_tokens + 16,
              max_num_batched_tokens=max(4096, a.prompt_len + a.max_tokens + 16), seed=a.seed)
    if a.random_init:
        kw["random_init"] = "seeded"
    if a.device:
        kw["device"] = a.device
    llm = LLM(a.model, **kw)
    try:
        vocab = llm.config.hf_config.vocab_size
        rng = random.Random(a.seed)
        prompts = [[rng.randrange(vocab) for _ in range(a.prompt_len)] for _ in range(a.prompts)]
        payload = run_probe(llm, a.switch, base, cand, prompts, a.max_tokens, a.repeats, l2=not a.no_l2)
    finally:
        llm.exit()
    Path(a.output).write_text(json.dumps(payload, indent=2))
    print(json.dumps(payload["comparison"]))
    return payload


if __name__ == "__main__":
    main()

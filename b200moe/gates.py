"""Frozen acceptance gates for A/B decisions and backend equivalence.

    python -m b200moe.gates ab --kind moe --input sweep.json --output moe-decision.json [--markdown x.md]
    python -m b200moe.gates ab --kind graph --input sweep.json --output graph-decision.json
    python -m b200moe.gates equivalence --input eq.json [--slo online.json] --output eq-decision.json

The thresholds below are fixed before any measurement and must not be tuned
after seeing results (the reference's practice, scripts/p5_decide.py and
scripts/p6_decide_attention_equivalence.py).  Every decision is an auditable
JSON (thresholds, per-check observations, decision, sha256 of the evidence
file) plus an optional Markdown table.

A/B gates read the offline driver's summary (``b200moe.bench_offline``):
throughput medians, TPOT p95 medians and run-to-run CV per (backend, batch).
The equivalence gate reads ``b200moe.equivalence`` output (layers L1-L4) and,
optionally, an online benchmark (``b200moe.bench_online``) for L5.
"""
from __future__ import annotations

import argparse
import hashlib
import json
from pathlib import Path

ATTENTION_GATES = {
    "baseline": "sdpa", "candidate": "paged", "batches": [16, 32],
    "tpot_ratio_max": 0.90, "throughput_ratio_min": 1.00, "cv_max": 0.05,
}
MOE_GATES = {
    "baseline": "loop", "candidate": "fused", "batches": [16, 32],
    "throughput_ratio_min": 1.08, "tpot_ratio_max": 1.00, "cv_max": 0.05,
}
GRAPH_GATES = {
    "b1_gain_min": 0.15, "b8_gain_min": 0.05, "regression_ratio_min": 0.98, "cv_max": 0.05,
    "memory_delta_max_gib": 2.0,
}
EQUIVALENCE_GATES = {
    "structural_max_abs": 2e-3,          # L1
    "flip_rate_max": 0.005,              # L2 (strict <)
    "flip_margin_max": 0.5,              # L2 (strict <)
    "first_token_agreement_min": 0.99,   # L3
    "degenerate_max": 0,                 # L3
    "determinism_required": True,        # L4
    "slo_rate_min": 1.0,                 # L5: every load point keeps 100 % standard SLO
    "report_only": ["request_token_identical", "request_token_agreement_mean", "lcp_p50", "lcp_mean",
                    "edit_distance_ratio_p50", "edit_distance_ratio_max"],
}


def sha256_file(path) -> str | None:
    p = Path(path)
    return hashlib.sha256(p.read_bytes()).hexdigest() if p.is_file() else None


def _ratio(a, b):
    return None if a is None or b in (None, 0) else a / b


def _index(summary: list[dict], key: str) -> dict:
    """(backend-ish key, batch) -> matrix-phase summary row."""
    return {(r[key], int(r["batch"])): r for r in summary if r.get("phase", "matrix") == "matrix"}


def decide_ab(payload: dict, kind: str) -> dict:
    """attention / moe: candidate vs baseline at the gated batches."""
    gates = ATTENTION_GATES if kind == "attention" else MOE_GATES
    key = "attention_backend" if kind == "attention" else "backend"
    idx = _index(payload["summary"], key)
    checks = []
    for b in gates["batches"]:
        base, cand = idx.get((gates["baseline"], b)), idx.get((gates["candidate"], b))
        if base is None or cand is None:
            checks.append({"batch": b, "pass": False, "reason": "missing benchmark point"})
            continue
        tpot = _ratio(cand["tpot_p95_median_s"], base["tpot_p95_median_s"])
        thr = _ratio(cand["throughput_median"], base["throughput_median"])
        ok = (tpot is not None and thr is not None and tpot <= gates["tpot_ratio_max"]
              and thr >= gates["throughput_ratio_min"] and cand["throughput_cv"] <= gates["cv_max"])
        checks.append({"batch": b, "tpot_ratio": tpot, "throughput_ratio": thr, "candidate_cv": cand["throughput_cv"],
                       "pass": ok})
    ver = payload.get("verification") or {}
    gate_ok = ver.get("passed", True)
    adopt = bool(checks) and all(c["pass"] for c in checks) and gate_ok
    return {"mode": kind, "thresholds": gates, "checks": checks, "verification_passed": gate_ok,
            "adopt": adopt, "decision": f"adopt_{gates['candidate']}" if adopt else f"keep_{gates['baseline']}"}


def decide_graph(payload: dict) -> dict:
    """Decode CUDA graphs vs eager: gains at batch 1 and 8, no regression elsewhere, bounded memory."""
    g = GRAPH_GATES
    idx = _index(payload["summary"], "graph_mode")
    checks = []
    for b in sorted({k[1] for k in idx}):
        e, c = idx.get(("eager", b)), idx.get(("graphs", b))
        if e is None or c is None:
            continue
        ratio = _ratio(c["throughput_median"], e["throughput_median"])
        need = g["b1_gain_min"] if b == 1 else g["b8_gain_min"] if b == 8 else None
        ok = ratio is not None and c["throughput_cv"] <= g["cv_max"] and (
            ratio >= 1 + need if need is not None else ratio >= g["regression_ratio_min"])
        checks.append({"batch": b, "throughput_ratio": ratio, "required": (1 + need) if need is not None
                       else g["regression_ratio_min"], "candidate_cv": c["throughput_cv"], "pass": ok})
    mem = payload.get("graph_memory_delta_gib")
    if mem is not None:
        checks.append({"name": "memory_delta_gib", "value": mem, "threshold": g["memory_delta_max_gib"],
                       "pass": mem <= g["memory_delta_max_gib"]})
    have = {c.get("batch") for c in checks}
    if not {1, 8} <= have:
        checks.append({"name": "coverage", "pass": False, "reason": "batches 1 and 8 are required"})
    adopt = bool(checks) and all(c["pass"] for c in checks)
    return {"mode": "graph", "thresholds": g, "checks": checks, "adopt": adopt,
            "decision": "adopt_graphs" if adopt else "keep_eager"}


def decide_equivalence(eq: dict, slo: dict | None = None) -> dict:
    g = EQUIVALENCE_GATES
    comp, det = eq["comparison"], eq.get("determinism", {})
    checks = []
    if "l1" in eq:
        v = eq["l1"]["max_abs"]
        checks.append({"layer": "L1", "name": "structural_max_abs", "value": v, "threshold": g["structural_max_abs"],
                       "pass": v < g["structural_max_abs"]})
    if "l2" in eq:
        l2 = eq["l2"]
        checks.append({"layer": "L2", "name": "top1_flip_rate", "value": l2["flip_rate"],
                       "threshold": g["flip_rate_max"], "pass": l2["flip_rate"] < g["flip_rate_max"],
                       "detail": {"flips": l2["flips"], "compared_positions": l2["compared_positions"]}})
        checks.append({"layer": "L2", "name": "flip_margin_max", "value": l2["flip_margin_max"],
                       "threshold": g["flip_margin_max"], "pass": l2["flip_margin_max"] < g["flip_margin_max"]})
    checks.append({"layer": "L3", "name": "first_token_agreement", "value": comp["first_token_agreement_rate"],
                   "threshold": g["first_token_agreement_min"],
                   "pass": comp["first_token_agreement_rate"] >= g["first_token_agreement_min"]})
    degen = max(comp["degenerate_baseline"], comp["degenerate_candidate"])
    checks.append({"layer": "L3", "name": "degenerate_outputs", "value": degen, "threshold": g["degenerate_max"],
                   "pass": degen <= g["degenerate_max"]})
    checks.append({"layer": "L4", "name": "per_backend_determinism", "value": det, "threshold": "all true",
                   "pass": bool(det) and all(det.values())})
    if slo is not None:
        rates = [p["slo_standard_rate"] for p in slo.get("points", [])]
        worst = min(rates) if rates else 0.0
        checks.append({"layer": "L5", "name": "online_slo_standard_rate_min", "value": worst,
                       "threshold": g["slo_rate_min"], "pass": bool(rates) and worst >= g["slo_rate_min"]})
    adopt = all(c["pass"] for c in checks)
    return {"mode": "equivalence", "switch": eq.get("switch"), "baseline": eq.get("baseline"),
            "candidate": eq.get("candidate"), "thresholds": g, "checks": checks,
            "reported_only": {k: comp.get(k) for k in g["report_only"]}, "adopt": adopt,
            "decision": f"adopt_{eq.get('candidate')}" if adopt else f"keep_{eq.get('baseline')}"}


def markdown(decision: dict) -> str:
    lines = [f"# {decision['mode']} decision: **{decision['decision']}**", "",
             "| check | value | threshold | pass |", "|---|---:|---:|---|"]
    for c in decision["checks"]:
        name = c.get("name") or f"batch {c.get('batch')}"
        if "layer" in c:
            name = f"{c['layer']} {name}"
        value = c.get("value", c.get("throughput_ratio"))
        if isinstance(value, float):
            value = f"{value:.6g}"
        thr = c.get("threshold", c.get("required", ""))
        lines.append(f"| {name} | `{value}` | {thr} | {'yes' if c['pass'] else 'NO'} |")
    if decision.get("reported_only"):
        lines += ["", "Reported only: " + json.dumps(decision["reported_only"])]
    return "\n".join(lines) + "\n"


def write_decision(decision: dict, evidence: str, output: str, md: str | None = None, extra: dict | None = None):
    decision = {"schema_version": 1, "input": evidence, "evidence_sha256": sha256_file(evidence), **decision,
                **(extra or {})}
    out = Path(output)
    out.parent.mkdir(parents=True, exist_ok=True)
    out.write_text(json.dumps(decision, indent=2))
    if md:
        Path(md).write_text(markdown(decision))
    return decision


def main(argv=None):
    p = argparse.ArgumentParser(description="frozen A/B and equivalence gates")
    sub = p.add_subparsers(dest="cmd", required=True)
    ab = sub.add_parser("ab")
    ab.add_argument("--kind", choices=("attention", "moe", "graph"), required=True)
    eq = sub.add_parser("equivalence")
    eq.add_argument("--slo", default=None, help="online benchmark JSON for L5")
    for sp in (ab, eq):
        sp.add_argument("--input", required=True)
        sp.add_argument("--output", required=True)
        sp.add_argument("--markdown", default=None)
    a = p.parse_args(argv)
    payload = json.loads(Path(a.input).read_text())
    extra = None
    if a.cmd == "ab":
        d = decide_graph(payload) if a.kind == "graph" else decide_ab(payload, a.kind)
    else:
        slo = json.loads(Path(a.slo).read_text()) if a.slo else None
        d = decide_equivalence(payload, slo)
        if a.slo:
            extra = {"slo_input": a.slo, "slo_sha256": sha256_file(a.slo)}
    d = write_decision(d, a.input, a.output, a.markdown, extra)
    print(markdown(d))
    return d


if __name__ == "__main__":
    main()

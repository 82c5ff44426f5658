"""Decision gates and the equivalence probe on CPU."""
import json

import pytest

from b200moe import equivalence as eqm
from b200moe import gates


def _row(backend, batch, thr, tpot, cv=0.01, key="backend", **kw):
    return {"phase": "matrix", key: backend, "batch": batch, "throughput_median": thr, "tpot_p95_median_s": tpot,
            "throughput_cv": cv, **kw}


def test_moe_ab_gate():
    summary = [_row("loop", 16, 100, 0.05), _row("fused", 16, 120, 0.04), _row("loop", 32, 150, 0.06),
               _row("fused", 32, 170, 0.05)]
    d = gates.decide_ab({"summary": summary, "verification": {"passed": True}}, "moe")
    assert d["adopt"] and d["decision"] == "adopt_fused"
    summary[3]["throughput_median"] = 155  # 1.033x < 1.08x
    assert gates.decide_ab({"summary": summary}, "moe")["decision"] == "keep_loop"
    d = gates.decide_ab({"summary": summary[:2]}, "moe")  # batch 32 missing
    assert not d["adopt"] and any(c.get("reason") == "missing benchmark point" for c in d["checks"])
    ok = [_row("loop", b, 100, 0.05) for b in (16, 32)] + [_row("fused", b, 200, 0.02) for b in (16, 32)]
    assert not gates.decide_ab({"summary": ok, "verification": {"passed": False}}, "moe")["adopt"]


def test_attention_and_graph_gates():
    att = [_row(b, n, t, p, key="attention_backend") for b, t, p in (("sdpa", 100, 0.1), ("paged", 130, 0.05))
           for n in (16, 32)]
    assert gates.decide_ab({"summary": att}, "attention")["adopt"]
    g = [_row(m, b, t, 0.1, key="graph_mode") for m, b, t in
         (("eager", 1, 100), ("graphs", 1, 130), ("eager", 8, 400), ("graphs", 8, 440), ("eager", 64, 900),
          ("graphs", 64, 890))]
    d = gates.decide_graph({"summary": g, "graph_memory_delta_gib": 0.7})
    assert d["adopt"], d
    g[1]["throughput_median"] = 110  # only +10 % at batch 1
    assert gates.decide_graph({"summary": g})["decision"] == "keep_eager"
    assert not gates.decide_graph({"summary": g[2:]})["adopt"]  # batch 1 missing


def test_equivalence_gate_layers():
    eq = {"switch": "attention", "baseline": "sdpa", "candidate": "paged",
          "comparison": {"first_token_agreement_rate": 1.0, "degenerate_baseline": 0, "degenerate_candidate": 0,
                         "request_token_identical": 0.4},
          "determinism": {"sdpa": True, "paged": True}, "l1": {"max_abs": 1.2e-4},
          "l2": {"flip_rate": 0.002, "flips": 2, "compared_positions": 1000, "flip_margin_max": 0.31}}
    slo = {"points": [{"slo_standard_rate": 1.0}, {"slo_standard_rate": 1.0}]}
    d = gates.decide_equivalence(eq, slo)
    assert d["adopt"] and {c["layer"] for c in d["checks"]} == {"L1", "L2", "L3", "L4", "L5"}
    assert d["reported_only"]["request_token_identical"] == 0.4
    eq["l2"]["flip_margin_max"] = 0.9  # a flip away from a near-tie
    assert gates.decide_equivalence(eq)["decision"] == "keep_sdpa"
    eq["l2"]["flip_margin_max"] = 0.1
    eq["determinism"]["paged"] = False
    assert not gates.decide_equivalence(eq)["adopt"]


def test_probe_helpers():
    assert eqm.longest_common_prefix([1, 2, 3], [1, 2, 4]) == 2
    assert eqm.edit_distance([1, 2, 3], [1, 3]) == 1 and eqm.edit_distance([], [1, 2]) == 2
    assert eqm.is_degenerate([5] * 20) and eqm.is_degenerate([1, 2] * 10)
    assert not eqm.is_degenerate(list(range(30)))


def test_probe_end_to_end_and_cli(tmp_path):
    """Both MoE paths on the CPU run the fp32 oracle: the probe must report
    identity, and the gate CLI must adopt and write auditable files."""
    out = tmp_path / "eq.json"
    payload = eqm.main(["--model", "tiny-moe", "--random-init", "--device", "cpu", "--switch", "moe", "--prompts", "3",
                        "--prompt-len", "12", "--max-tokens", "6", "--repeats", "2", "--output", str(out)])
    c = payload["comparison"]
    assert c["first_token_agreement_rate"] == 1.0 and c["request_token_identical"] == 1.0
    assert payload["determinism"] == {"loop": True, "fused": True}
    assert payload["l2"]["flip_rate"] == 0.0 and payload["l2"]["compared_positions"] == 3 * 6
    d = gates.main(["equivalence", "--input", str(out), "--output", str(tmp_path / "d.json"),
                    "--markdown", str(tmp_path / "d.md")])
    assert d["adopt"] and d["evidence_sha256"]
    assert "adopt_fused" in (tmp_path / "d.md").read_text()
    assert json.loads((tmp_path / "d.json").read_text())["decision"] == "adopt_fused"


def test_structural_check_cpu():
    r = eqm.structural_check("cpu")
    assert r["max_abs"] < gates.EQUIVALENCE_GATES["structural_max_abs"]

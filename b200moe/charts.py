"""Render metric charts from evidence JSON as standalone SVG (no plotting library).

    python -m b200moe.charts --offline sweep.json --online online.json \
        --bench bench_lines.jsonl --micro micro.jsonl --out assets/charts

Charts (each only when its input is given):
  offline_throughput.svg   output tok/s by batch, one line per MoE / attention backend
                           (``b200moe.bench_offline`` summary)
  capacity_curve.svg       standard-SLO success rate and TPOT p95 against achieved QPS
                           (``b200moe.bench_online`` points)
  scaling.svg              bench.py value against GPU count (one JSON line per run)
  kernel_roofline.svg      microbench fraction of the measured HBM / tensor peak per kernel
Every chart carries a footnote naming its source file and the file's sha256, like
the reference's renderer (scripts/render_metrics.py), which needs matplotlib.
"""
from __future__ import annotations

import argparse
import hashlib
import json
import math
from pathlib import Path
from xml.sax.saxutils import escape

PALETTE = ("#2563EB", "#EA580C", "#0D9488", "#7C3AED", "#DC2626", "#9CA3AF")
W, H = 720, 420
ML, MR, MT, MB = 70, 160, 50, 70  # margins: the legend sits on the right


def _nice_ticks(lo: float, hi: float, n: int = 5) -> list[float]:
    if hi <= lo:
        hi = lo + 1.0
    raw = (hi - lo) / n
    mag = 10 ** math.floor(math.log10(raw))
    step = min((m * mag for m in (1, 2, 2.5, 5, 10) if m * mag >= raw), default=10 * mag)
    start = math.floor(lo / step) * step
    ticks, v = [], start
    while v <= hi + step * 0.5:
        ticks.append(round(v, 10))
        v += step
    return ticks


def _fmt(v: float) -> str:
    if v == 0:
        return "0"
    if abs(v) >= 1000:
        return f"{v / 1000:g}k"
    return f"{v:g}"


class Chart:
    """A minimal SVG chart: axes, grid, ticks, line or grouped-bar series, legend, footnote."""

    def __init__(self, title: str, xlabel: str, ylabel: str, footnote: str = ""):
        self.title, self.xlabel, self.ylabel, self.footnote = title, xlabel, ylabel, footnote
        self.series: list[tuple[str, list[tuple[float, float]], str]] = []
        self.categories: list[str] | None = None

    def line(self, name: str, points, dashed: bool = False):
        self.series.append((name, sorted(points), "dash" if dashed else "line"))

    def bars(self, categories: list[str], name: str, values: list[float]):
        self.categories = categories
        self.series.append((name, list(enumerate(values)), "bar"))

    def svg(self) -> str:
        pw, ph = W - ML - MR, H - MT - MB
        ys = [y for _, pts, _ in self.series for _, y in pts if y is not None]
        ymax = max(ys) if ys else 1.0
        yt = _nice_ticks(0.0, ymax * 1.05)
        y0, y1 = yt[0], yt[-1]
        if self.categories is not None:
            xs = list(range(len(self.categories)))
            x0, x1 = -0.5, len(self.categories) - 0.5
        else:
            xs = [x for _, pts, _ in self.series for x, _ in pts]
            x0, x1 = (min(xs), max(xs)) if xs else (0.0, 1.0)
            if x1 == x0:
                x0, x1 = x0 - 1, x1 + 1
        sx = lambda x: ML + (x - x0) / (x1 - x0) * pw
        sy = lambda y: MT + ph - (y - y0) / (y1 - y0) * ph
        out = [f'<svg xmlns="http://www.w3.org/2000/svg" width="{W}" height="{H}" font-family="sans-serif" '
               f'font-size="11"><rect width="100%" height="100%" fill="white"/>',
               f'<text x="{ML}" y="28" font-size="14" font-weight="bold">{escape(self.title)}</text>']
        for t in yt:
            out.append(f'<line x1="{ML}" x2="{ML + pw}" y1="{sy(t):.1f}" y2="{sy(t):.1f}" stroke="#E5E7EB"/>')
            out.append(f'<text x="{ML - 6}" y="{sy(t) + 4:.1f}" text-anchor="end">{_fmt(t)}</text>')
        if self.categories is not None:
            for i, c in enumerate(self.categories):
                out.append(f'<text x="{sx(i):.1f}" y="{MT + ph + 16}" text-anchor="middle">{escape(c)}</text>')
        else:
            for t in _nice_ticks(x0, x1):
                if x0 <= t <= x1:
                    out.append(f'<text x="{sx(t):.1f}" y="{MT + ph + 16}" text-anchor="middle">{_fmt(t)}</text>')
        out.append(f'<line x1="{ML}" x2="{ML + pw}" y1="{MT + ph}" y2="{MT + ph}" stroke="#6B7280"/>')
        out.append(f'<line x1="{ML}" x2="{ML}" y1="{MT}" y2="{MT + ph}" stroke="#6B7280"/>')
        out.append(f'<text x="{ML + pw / 2:.1f}" y="{H - MB + 40}" text-anchor="middle">{escape(self.xlabel)}</text>')
        out.append(f'<text transform="translate(18,{MT + ph / 2:.1f}) rotate(-90)" text-anchor="middle">'
                   f'{escape(self.ylabel)}</text>')
        nbar = sum(1 for *_, k in self.series if k == "bar")
        bw = 0.8 / max(nbar, 1)
        bi = 0
        for si, (name, pts, kind) in enumerate(self.series):
            col = PALETTE[si % len(PALETTE)]
            if kind == "bar":
                for x, y in pts:
                    if y is None:
                        continue
                    left = sx(x - 0.4 + bi * bw)
                    out.append(f'<rect x="{left:.1f}" y="{sy(y):.1f}" width="{bw * pw / (x1 - x0):.1f}" '
                               f'height="{sy(y0) - sy(y):.1f}" fill="{col}"/>')
                bi += 1
            else:
                pp = [(x, y) for x, y in pts if y is not None]
                d = " ".join(f"{sx(x):.1f},{sy(y):.1f}" for x, y in pp)
                dash = ' stroke-dasharray="5,4"' if kind == "dash" else ""
                out.append(f'<polyline points="{d}" fill="none" stroke="{col}" stroke-width="2"{dash}/>')
                out += [f'<circle cx="{sx(x):.1f}" cy="{sy(y):.1f}" r="3" fill="{col}"/>' for x, y in pp]
            ly = MT + 14 + 18 * si
            out.append(f'<rect x="{W - MR + 14}" y="{ly - 9}" width="12" height="10" fill="{col}"/>')
            out.append(f'<text x="{W - MR + 32}" y="{ly}">{escape(name)}</text>')
        if self.footnote:
            out.append(f'<text x="6" y="{H - 8}" font-size="9" fill="#9CA3AF">{escape(self.footnote)}</text>')
        out.append("</svg>")
        return "\n".join(out)


def _source(path: str) -> str:
    data = Path(path).read_bytes()
    return f"source: {Path(path).name} sha256 {hashlib.sha256(data).hexdigest()[:16]}"


def offline_chart(path: str) -> Chart:
    payload = json.loads(Path(path).read_text())
    ch = Chart("Offline output throughput by batch", "batch (concurrent requests)", "output tok/s", _source(path))
    groups: dict[str, list] = {}
    for s in payload["summary"]:
        if s.get("phase", "matrix") != "matrix":
            continue
        key = f"{s['backend']} / {s['attention_backend']}" + (f" / {s['graph_mode']}" if s.get("graph_mode") else "")
        groups.setdefault(key, []).append((s["batch"], s["throughput_median"]))
    for k, pts in sorted(groups.items()):
        ch.line(k, pts)
    return ch


def capacity_chart(path: str) -> Chart:
    payload = json.loads(Path(path).read_text())
    pts = payload["points"]
    ch = Chart("Online capacity: SLO success and TPOT p95", "achieved QPS", "rate / seconds", _source(path))
    ch.line("standard SLO rate", [(p["achieved_qps"], p["slo_standard_rate"]) for p in pts])
    ch.line("strict SLO rate", [(p["achieved_qps"], p["slo_strict_rate"]) for p in pts], dashed=True)
    ch.line("TPOT p95 (s)", [(p["achieved_qps"], p.get("tpot_p95_s")) for p in pts])
    return ch


def scaling_chart(path: str) -> Chart:
    rows = [json.loads(l) for l in Path(path).read_text().splitlines() if l.strip().startswith("{")]
    rows = [r for r in rows if "value" in r and "n_gpus" in r]
    ch = Chart("Throughput against GPU count", "GPUs", rows[0]["unit"] if rows else "value", _source(path))
    for impl in sorted({r.get("impl", "b200moe") for r in rows}):
        ch.line(impl, [(r["n_gpus"], r["value"]) for r in rows if r.get("impl", "b200moe") == impl])
    return ch


def roofline_chart(path: str) -> Chart:
    rows = [json.loads(l) for l in Path(path).read_text().splitlines() if l.strip().startswith("{")]
    rows = [r for r in rows if "kernel" in r and ("hbm_frac" in r or "tc_frac" in r)]
    names = [f"{r['kernel']}@{r.get('tokens', r.get('seqs', ''))}" for r in rows]
    ch = Chart("Kernels: fraction of measured peak", "kernel @ tokens", "fraction of peak", _source(path))
    ch.bars(names, "HBM", [r.get("hbm_frac") for r in rows])
    ch.bars(names, "tensor", [r.get("tc_frac") for r in rows])
    return ch


def render(out_dir: str, offline=None, online=None, bench=None, micro=None) -> list[str]:
    out = Path(out_dir)
    out.mkdir(parents=True, exist_ok=True)
    written = []
    for path, fn, name in ((offline, offline_chart, "offline_throughput.svg"),
                           (online, capacity_chart, "capacity_curve.svg"),
                           (bench, scaling_chart, "scaling.svg"), (micro, roofline_chart, "kernel_roofline.svg")):
        if path:
            (out / name).write_text(fn(path).svg())
            written.append(str(out / name))
    return written


def main(argv=None):
    p = argparse.ArgumentParser(description="render evidence charts as SVG")
    p.add_argument("--offline")
    p.add_argument("--online")
    p.add_argument("--bench", help="JSON lines of bench.py runs")
    p.add_argument("--micro", help="JSON lines of b200moe.microbench")
    p.add_argument("--out", default="assets/charts")
    a = p.parse_args(argv)
    for f in render(a.out, a.offline, a.online, a.bench, a.micro):
        print(f)


if __name__ == "__main__":
    main()

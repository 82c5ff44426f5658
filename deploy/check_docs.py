"""Docs consistency linter for the product documents (stdlib only).

    python deploy/check_docs.py [--root DIR] [FILES...]

Checks, in the product documents (the root-level readme and design notes, and
docs/**/*.md; or the files given):
  1. relative links ``[text](path)`` point at files that exist;
  2. image targets ``![..](path)`` exist;
  3. code spans (inline and fenced) that name a repository file
     (b200moe/..., tests/..., deploy/..., baseline/..., bench.py, setup.py)
     or a module run as ``python -m b200moe.x`` point at real files;
  4. no hand-maintained counts that go stale on every commit (``N tests
     passed`` / ``N commits ahead``): refer to the command that prints them.
Exit status 0 = clean, 1 = problems (listed on stderr).  Behaviour follows the
reference's linter (scripts/check_docs.py:1-114).
"""
from __future__ import annotations

import argparse
import re
import sys
from pathlib import Path

LINK = re.compile(r"(?<!!)\[[^\]]*\]\(([^)\s]+)\)")
IMAGE = re.compile(r"!\[[^\]]*\]\(([^)\s]+)\)")
CODE_SPAN = re.compile(r"`([^`\n]+)`")
FENCE = re.compile(r"^```.*?^```", re.S | re.M)
REPO_PATH = re.compile(r"(?<![\w./-])((?:b200moe|tests|deploy|baseline|profiles)/[\w/.\-]+\.(?:py|sh|cu|cuh|h|cpp|md|txt|json|service|example)"
                       r"|bench\.py|setup\.py|__graft_entry__\.py)")
MODULE = re.compile(r"python3?\s+-m\s+(b200moe(?:\.\w+)+)")
STALE = re.compile(r"\b\d+\s+(?:tests?\s+)?passed\b|\b\d+\s+commits?\s+ahead\b", re.I)


def default_docs(root: Path) -> list[Path]:
    out = [root / n for n in ("README.md", "DESIGN.md") if (root / n).is_file()]
    docs = root / "docs"
    if docs.is_dir():
        out += sorted(docs.rglob("*.md"))
    return out


def _target(t: str) -> str:
    t = t.strip()
    if t.startswith(("<", "http://", "https://", "mailto:", "#")):
        return ""
    return t.split("#", 1)[0]


def module_exists(root: Path, mod: str) -> bool:
    base = root.joinpath(*mod.split("."))
    return base.with_suffix(".py").is_file() or (base / "__main__.py").is_file() or (base / "__init__.py").is_file()


def check_file(root: Path, path: Path) -> list[str]:
    rel = path.relative_to(root).as_posix() if path.is_relative_to(root) else str(path)
    text = path.read_text(encoding="utf-8")
    problems = []
    for pat, kind in ((LINK, "dead link"), (IMAGE, "missing image")):
        for m in pat.finditer(text):
            t = _target(m.group(1))
            if t and not (path.parent / t).exists() and not (root / t).exists():
                problems.append(f"{rel}: {kind} -> {t}")
    spans = [m.group(1) for m in CODE_SPAN.finditer(FENCE.sub("", text))]
    spans += [b for b in FENCE.findall(text)]
    for span in spans:
        for m in REPO_PATH.finditer(span):
            if not (root / m.group(1)).exists():
                problems.append(f"{rel}: code names a missing file -> {m.group(1)}")
        for m in MODULE.finditer(span):
            if not module_exists(root, m.group(1)):
                problems.append(f"{rel}: code runs a missing module -> {m.group(1)}")
    for m in STALE.finditer(text):
        problems.append(f"{rel}: hand-maintained count goes stale -> {m.group(0)!r}")
    return problems


def main(argv=None) -> int:
    p = argparse.ArgumentParser()
    p.add_argument("--root", default=str(Path(__file__).resolve().parents[1]))
    p.add_argument("files", nargs="*")
    a = p.parse_args(argv)
    root = Path(a.root).resolve()
    files = [Path(f).resolve() for f in a.files] or default_docs(root)
    problems = [x for f in files for x in check_file(root, f)]
    for x in problems:
        print(x, file=sys.stderr)
    print(f"check_docs: {len(files)} file(s), {len(problems)} problem(s)")
    return 1 if problems else 0


if __name__ == "__main__":
    sys.exit(main())

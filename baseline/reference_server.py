"""The UNMODIFIED reference OpenAI server (installed in baseline/_ref) on a random-init
checkpoint of the named architecture, for the online workload's reference arm:

    python baseline/reference_server.py --arch qwen3-30b-a3b -- --port 8124 --tensor-parallel-size 1 ...

Everything after ``--`` goes to the reference's own server CLI (``s4000-server``,
nanovllm/entrypoints/openai/api_server.py); ``--model`` is set to the checkpoint,
which is written in the reference's format by ``reference_arm.write_checkpoint``
(reused when a finished one exists).  Nothing from b200moe is imported.
"""
from __future__ import annotations

import argparse
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
import reference_arm as ra  # noqa: E402


def main(argv=None) -> int:
    argv = list(sys.argv[1:] if argv is None else argv)
    rest = []
    if "--" in argv:
        i = argv.index("--")
        argv, rest = argv[:i], argv[i + 1:]
    p = argparse.ArgumentParser()
    p.add_argument("--arch", default="qwen3-30b-a3b", choices=sorted(ra.ARCH))
    p.add_argument("--seed", type=int, default=0)
    a = p.parse_args(argv)
    if not os.path.isdir(os.path.join(ra.REF, "nanovllm")):
        print(f"reference not installed: no package at {os.path.join(ra.REF, 'nanovllm')}", file=sys.stderr)
        return 2
    ckpt = ra.checkpoint_dir(a.arch)
    if not os.path.exists(os.path.join(ckpt, ra.COMPLETE)):
        ra.write_checkpoint(ckpt, ra.ARCH[a.arch], seed=a.seed)
    sys.path.insert(0, ra.REF)
    for var in ("TORCHELASTIC_USE_AGENT_STORE", "TORCHELASTIC_RESTART_COUNT"):
        os.environ.pop(var, None)
    from nanovllm.entrypoints.openai.api_server import main as serve  # the reference package
    return serve(["--model", ckpt, *rest]) or 0


if __name__ == "__main__":
    sys.exit(main())

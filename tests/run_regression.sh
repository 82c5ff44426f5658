#!/bin/bash
# One-command regression, fast-fail, cheapest tier first:
#   1. every CPU test (scheduler, engine, faults, gloo ranks, API, benchmark maths);
#   2. with a GPU visible: kernel numerics against fp32 references, engine-level
#      GPU tests (graphs, overlap, int8 KV, offload, PD), the allocation-free
#      decode path, the 2-GPU tests when two GPUs are visible, and the smoke run.
#   tests/run_regression.sh [extra pytest args]
set -euo pipefail
cd "$(dirname "$0")/.."
run() { echo "== $*"; "$@"; }
run python -m pytest tests -x -q -m "not gpu" "$@"
if python -c 'import sys, torch; sys.exit(0 if torch.cuda.is_available() else 1)'; then
  run python -m pytest tests/test_kernels_gpu.py -x -q "$@"
  run python -m pytest tests/test_model_gpu.py tests/test_pd_gpu.py -x -q "$@"
  run python -m pytest tests/test_zz_no_alloc.py -x -q "$@"
  if [ "$(python -c 'import torch; print(torch.cuda.device_count())')" -ge 2 ]; then
    run python -m pytest tests/test_multi_gpu.py -x -q "$@"
  fi
  run python -c 'import __graft_entry__ as g; g.smoke()'
else
  echo "== no GPU visible: GPU tiers skipped"
fi

#!/bin/bash
# Smoke-test every replica started by serve_dp.sh: deploy/smoke_dp.sh REPLICAS [BASE_PORT]
set -euo pipefail
ROOT=$(cd "$(dirname "$0")/.." && pwd)
N=${1:?replica count}
PORT0=${2:-${B200MOE_PORT:-8000}}
for ((i = 0; i < N; i++)); do
  port=$((PORT0 + i))
  for _ in $(seq 1 360); do curl -fsS "http://127.0.0.1:$port/health" >/dev/null 2>&1 && break; sleep 5; done
  "$ROOT/deploy/smoke_serve.sh" "http://127.0.0.1:$port"
done

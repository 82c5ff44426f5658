#!/bin/bash
# Start the server with the settings of the environment file (systemd passes
# them itself; a manual start reads the file here).
set -euo pipefail
ROOT=$(cd "$(dirname "$0")/.." && pwd)
ENV_FILE=${B200MOE_ENV_FILE:-/etc/b200moe/serve.env}
if [ -z "${B200MOE_MODEL:-}${NANOVLLM_MODEL:-}" ] && [ -r "$ENV_FILE" ]; then
  set -a
  # shellcheck disable=SC1090
  . "$ENV_FILE"
  set +a
fi
: "${B200MOE_MODEL:=${NANOVLLM_MODEL:-}}"
: "${B200MOE_MODEL:?B200MOE_MODEL is not set; edit $ENV_FILE}"
export B200MOE_MODEL
PY=${B200MOE_PYTHON:-python3}
cd "$ROOT"
export PYTHONPATH="$ROOT${PYTHONPATH:+:$PYTHONPATH}"
exec "$PY" -m b200moe.entrypoints.openai.api_server "$@"

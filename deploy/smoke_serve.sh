#!/bin/bash
# Smoke-test a running server: health, model list, one completion, one
# streamed chat completion, metrics.  Usage: deploy/smoke_serve.sh [base_url]
set -euo pipefail
BASE=${1:-http://127.0.0.1:${B200MOE_PORT:-8000}}
AUTH=()
if [ -n "${B200MOE_API_KEY:-}" ]; then AUTH=(-H "Authorization: Bearer $B200MOE_API_KEY"); fi
fail() { echo "SMOKE FAIL: $*" >&2; exit 1; }
curl -fsS "${AUTH[@]}" "$BASE/health" >/dev/null || fail "/health"
MODEL=$(curl -fsS "${AUTH[@]}" "$BASE/v1/models" | python3 -c 'import json,sys; print(json.load(sys.stdin)["data"][0]["id"])') \
  || fail "/v1/models"
OUT=$(curl -fsS "${AUTH[@]}" -H 'Content-Type: application/json' "$BASE/v1/completions" \
  -d "{\"model\":\"$MODEL\",\"prompt\":\"Hello\",\"max_tokens\":8,\"temperature\":0}") || fail "/v1/completions"
echo "$OUT" | python3 -c 'import json,sys; d=json.load(sys.stdin); assert d["usage"]["completion_tokens"] > 0' \
  || fail "completion usage"
STREAM=$(curl -fsS -N "${AUTH[@]}" -H 'Content-Type: application/json' "$BASE/v1/chat/completions" \
  -d "{\"model\":\"$MODEL\",\"messages\":[{\"role\":\"user\",\"content\":\"Hi\"}],\"max_tokens\":8,\"stream\":true}") \
  || fail "streamed chat"
echo "$STREAM" | grep -q 'data: \[DONE\]' || fail "stream did not end with [DONE]"
curl -fsS "${AUTH[@]}" "$BASE/metrics" | grep -q '^b200moe_' || fail "/metrics"
echo "SMOKE OK ($BASE, model $MODEL)"

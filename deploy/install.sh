#!/bin/bash
# Install b200moe as a service.
#   deploy/install.sh [--prefix /opt/b200moe] [--user b200moe] [--python PY] [--no-venv] [--no-systemd]
# * never installs torch: the venv is created with --system-site-packages so the
#   host's CUDA-matched torch is used (or --no-venv uses PY directly);
# * builds the sm_100a extension in place and checks that it imports;
# * installs the systemd unit and /etc/b200moe/serve.env (kept if present).
set -euo pipefail
ROOT=$(cd "$(dirname "$0")/.." && pwd)
PREFIX=/opt/b200moe
SVC_USER=$(id -un)
PY=python3
VENV=1
SYSTEMD=1
while [ $# -gt 0 ]; do
  case "$1" in
    --prefix) PREFIX=$2; shift 2 ;;
    --user) SVC_USER=$2; shift 2 ;;
    --python) PY=$2; shift 2 ;;
    --no-venv) VENV=0; shift ;;
    --no-systemd) SYSTEMD=0; shift ;;
    *) echo "unknown option $1" >&2; exit 2 ;;
  esac
done
"$PY" -c 'import torch; assert torch.version.cuda, "CUDA build of torch required"' \
  || { echo "a CUDA build of torch must already be installed for $PY" >&2; exit 1; }
if [ "$VENV" = 1 ]; then
  "$PY" -m venv --system-site-packages "$PREFIX/venv"
  PY="$PREFIX/venv/bin/python"
  # service dependencies only; --no-deps keeps pip away from torch
  "$PY" -m pip install --no-deps fastapi uvicorn starlette pydantic safetensors 2>/dev/null \
    || echo "note: offline host, using the service dependencies already on the system"
fi
(cd "$ROOT" && TORCH_CUDA_ARCH_LIST=10.0a MAX_JOBS=${MAX_JOBS:-8} "$PY" setup.py build_ext --inplace)
(cd "$ROOT" && "$PY" -c 'import b200moe, b200moe.ops as o; o.native(); print("b200moe", b200moe.__version__, "extension ok")')
if [ "$SYSTEMD" = 1 ]; then
  sudo mkdir -p /etc/b200moe
  [ -f /etc/b200moe/serve.env ] || sudo install -m 600 "$ROOT/deploy/serve.env.example" /etc/b200moe/serve.env
  sed -e "s#@USER@#$SVC_USER#g" -e "s#@APP_DIR@#$ROOT#g" -e "s#@PYTHON@#$PY#g" "$ROOT/deploy/b200moe.service" \
    | sudo tee /etc/systemd/system/b200moe.service >/dev/null
  sudo systemctl daemon-reload
  echo "installed: edit /etc/b200moe/serve.env, then: sudo systemctl enable --now b200moe"
fi

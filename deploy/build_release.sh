#!/bin/bash
# Release tarball of the committed tree plus the built sm_100a extension.
#   deploy/build_release.sh [OUT_DIR]   -> OUT_DIR/b200moe-<version>-<commit>.tar.gz
set -euo pipefail
ROOT=$(cd "$(dirname "$0")/.." && pwd)
OUT=${1:-$ROOT/dist}
cd "$ROOT"
git diff --quiet HEAD -- b200moe deploy setup.py || { echo "uncommitted changes; commit first" >&2; exit 1; }
VER=$(python3 -c 'import re; print(re.search(r"__version__\s*=\s*\"([^\"]+)\"", open("b200moe/__init__.py").read()).group(1))')
SHA=$(git rev-parse --short HEAD)
NAME=b200moe-$VER-$SHA
mkdir -p "$OUT"
STAGE=$(mktemp -d)
git archive --format=tar --prefix="$NAME/" HEAD | tar -x -C "$STAGE"
for so in b200moe/_C*.so; do
  [ -e "$so" ] && cp "$so" "$STAGE/$NAME/b200moe/"
done
python3 "$ROOT/deploy/check_docs.py" --root "$STAGE/$NAME"
tar -C "$STAGE" -czf "$OUT/$NAME.tar.gz" "$NAME"
rm -r "$STAGE"
echo "$OUT/$NAME.tar.gz"

#!/usr/bin/env bash
# Installs the unmodified reference (iZonex/saint-llm) into baseline/_ref for the
# `bench.py --impl reference` arm and the reference-parity tests.
#
#   baseline/install_reference.sh <path-to-reference-checkout>
#   SAINT_LLM_REFERENCE=<path> baseline/install_reference.sh
#
# The official route is an offline pip install; the reference's packages use the
# `hatchling` build backend, which is not in the offline wheelhouse, so pip cannot build
# them.  Every reference package is pure Python in a src/ layout, so the fallback places
# each `src/saint_llm_*` tree into the target directory unchanged -- the same files a
# wheel install would lay down.
set -u
REF=${1:-${SAINT_LLM_REFERENCE:-}}
if [ -z "$REF" ] || [ ! -d "$REF/packages" ]; then
  echo "usage: $0 <reference checkout with packages/*/src> (or set SAINT_LLM_REFERENCE)" >&2
  exit 2
fi
HERE=$(cd "$(dirname "$0")" && pwd)
DEST="$HERE/_ref"
WHEELS=${SAINT_LLM_WHEELHOUSE:-/opt/wheelhouse}
mkdir -p "$DEST"
if python -m pip install --no-index --no-build-isolation --find-links "$WHEELS" \
      --target "$DEST" "$REF" > "$HERE/install_reference.log" 2>&1; then
  echo "pip install ok"
  exit 0
fi
echo "pip install failed (see install_reference.log); copying pure-python src trees"
for pkg in "$REF"/packages/*/src/saint_llm_*; do
  rm -rf "$DEST/$(basename "$pkg")"
  cp -r "$pkg" "$DEST/"
done
ls "$DEST"

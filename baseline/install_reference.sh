#!/usr/bin/env bash
# Installs the unmodified reference (iZonex/saint-llm) into baseline/_ref for the
# `bench.py --impl reference` arm.  The official route is an offline pip install;
# the reference's packages use the `hatchling` build backend, which is not in the
# offline wheelhouse, so pip cannot build them.  Every reference package is pure
# Python in a src/ layout, so the fallback places each `src/saint_llm_*` tree into
# the target directory unchanged -- the same files a wheel install would lay down.
set -u
REF=${1:-/root/reference}
HERE=$(cd "$(dirname "$0")" && pwd)
DEST="$HERE/_ref"
mkdir -p "$DEST"
if python -m pip install --no-index --no-build-isolation --find-links /opt/wheelhouse \
      --target "$DEST" "$REF" > "$HERE/install_reference.log" 2>&1; then
  echo "pip install ok"
  exit 0
fi
echo "pip install failed (see install_reference.log); copying pure-python src trees"
for pkg in "$REF"/packages/*/src/saint_llm_*; do
  cp -r "$pkg" "$DEST/"
done
ls "$DEST"

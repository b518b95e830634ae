#!/bin/sh
# Builds the reference's own CPU decode (pipelines/decode_native.c, one C file) into oracle/_ref/
# as the checker for the GPU decode. Test infrastructure: nothing in the engine links it.
# Flags follow the reference's own build of that file (decode_native.py: -O3 -ffp-contract=off),
# without which its float results change. Reads the reference tree at $IXB_REFERENCE
# (default /root/reference); does nothing when it is absent.
set -e
REF="${IXB_REFERENCE:-/root/reference}"
SRC="$REF/src/ignite_xdna/pipelines/decode_native.c"
HERE="$(cd "$(dirname "$0")" && pwd)"
[ -f "$SRC" ] || { echo "reference decode source not found; oracle/_ref not built"; exit 0; }
mkdir -p "$HERE/_ref"
gcc -O3 -ffp-contract=off -fPIC -shared -o "$HERE/_ref/decode_native.so" "$SRC" -lm
echo "built $HERE/_ref/decode_native.so"

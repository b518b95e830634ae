#!/bin/sh
# Builds the reference's own CPU decode (pipelines/decode_native.c) and preprocessing
# (pipelines/preprocess_simd.c), one C file each, into oracle/_ref/ as the checkers for the GPU
# decode and letterbox ingress. Test infrastructure: nothing in the engine links them.
# Flags follow the reference's own build of the decode (decode_native.py: -O3 -ffp-contract=off),
# without which its float results change; the preprocessing builds without AVX2 or OpenMP, its
# scalar path, which the reference states produces the same bytes. Reads the reference tree at $IXB_REFERENCE
# (default /root/reference); does nothing when it is absent.
set -e
REF="${IXB_REFERENCE:-/root/reference}"
SRC="$REF/src/ignite_xdna/pipelines/decode_native.c"
HERE="$(cd "$(dirname "$0")" && pwd)"
[ -f "$SRC" ] || { echo "reference decode source not found; oracle/_ref not built"; exit 0; }
mkdir -p "$HERE/_ref"
gcc -O3 -ffp-contract=off -fPIC -shared -o "$HERE/_ref/decode_native.so" "$SRC" -lm
gcc -O3 -ffp-contract=off -fPIC -shared -o "$HERE/_ref/preprocess_simd.so" \
    "$REF/src/ignite_xdna/pipelines/preprocess_simd.c" -lm
echo "built $HERE/_ref/decode_native.so $HERE/_ref/preprocess_simd.so"

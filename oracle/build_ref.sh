#!/bin/sh
# Compiles pieces of the reference that build standalone into oracle/_ref/
# (git-ignored).  Test infrastructure: used only to pin the oracle and to make
# the golden fixtures under tests/golden/.  Needs the reference checkout, named
# by XQ_REFERENCE (default: a `reference` directory beside this repository);
# the GPU box never runs this (it has no reference checkout).
#
#   src/bridge/ggml_d3d12.cpp:77-158  d3d12_gdn_supported + d3d12_gdn_emulate
#     (the reference's host mirror of its GATED_DELTA_NET shader).  The rest of
#     that file needs D3D12 and the ggml fork, so only this range is compiled,
#     against oracle/ref_shim/ggml_shim.h, with oracle/ref_shim/gdn_harness.cpp
#     generating the selftest inputs (ggml_d3d12.cpp:174-369 protocol).
set -eu
HERE=$(cd "$(dirname "$0")" && pwd)
REF=${XQ_REFERENCE:-$(cd "$HERE/../.." && pwd)/reference}
SRC="$REF/src/bridge/ggml_d3d12.cpp"
OUT="$HERE/_ref"
if [ ! -f "$SRC" ]; then
    echo "build_ref: reference source not found ($SRC); skipping" >&2
    exit 0
fi
mkdir -p "$OUT"
# Guard the line range: both functions must start where expected.
sed -n '77p' "$SRC" | grep -q '^bool d3d12_gdn_supported(const ggml_tensor\* op) {$'
sed -n '113p' "$SRC" | grep -q '^void d3d12_gdn_emulate(const ggml_tensor\* op, float\* out) {$'
sed -n '158p' "$SRC" | grep -q '^}$'
{
    echo '#include "ggml_shim.h"'
    sed -n '77,158p' "$SRC"
} > "$OUT/gdn_emulate_ref.cpp"
${CXX:-g++} -O2 -ffp-contract=off -fPIC -shared -std=c++17 -I"$HERE/ref_shim" \
    -o "$OUT/libxq_gdn_ref.so" "$OUT/gdn_emulate_ref.cpp" "$HERE/ref_shim/gdn_harness.cpp"
echo "build_ref: $OUT/libxq_gdn_ref.so"

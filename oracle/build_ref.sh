#!/bin/sh
# TEST INFRASTRUCTURE ONLY. Compiles the reference's own Int8Blocks.cpp and
# Sampler.cpp, unchanged and in place under the reference tree, against the
# two small shims in oracle/ref_shim (eacp's fp16 helpers, ea_data_structures'
# Span/Vector), into oracle/_ref/libhf_ref.so. Nothing from the reference is
# copied into this repository; the output directory is git-ignored.
# Usage: build_ref.sh [reference-root]   (the checkout of the reference project)
set -e
here="$(cd "$(dirname "$0")" && pwd)"
ref="${1:-/root/reference}"
lib="$ref/Lib"
if [ ! -f "$lib/HuggingFaceEACP/Kernels/Int8Blocks.cpp" ]; then
    echo "reference tree not found at $ref; oracle/_ref not built" >&2
    exit 0
fi
mkdir -p "$here/_ref"
g++ -std=c++20 -O2 -fPIC -shared \
    -I"$here/ref_shim" -I"$lib" \
    "$lib/HuggingFaceEACP/Kernels/Int8Blocks.cpp" \
    "$lib/HuggingFaceEACP/Sampling/Sampler.cpp" \
    "$here/ref_bridge.cpp" \
    -o "$here/_ref/libhf_ref.so"
echo "built $here/_ref/libhf_ref.so"

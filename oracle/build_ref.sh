#!/bin/sh
# TEST INFRASTRUCTURE ONLY. Compiles, unchanged and in place under the
# reference tree, the reference's own Kernels/Int8Blocks.cpp,
# Sampling/Sampler.cpp, Tokenizer/{Tokenizer,ByteFallback,Metaspace,
# SpecialTokens}.cpp and Tests/Decoder/ReferenceDecoder.h (its scalar
# double-precision forward pass) against the small shims in oracle/ref_shim
# (eacp's fp16 helpers, ea_data_structures' Span/Vector/Array, Miro's JSON
# reader and UTF-8 decoder, and a stand-in for Tests/Decoder/Common.h), into
# oracle/_ref/libhf_ref.so. Nothing from the
# reference is copied into this repository; the output directory is
# git-ignored.
#
# Usage: build_ref.sh [reference-root]   (the checkout of the reference project;
# default $HF_REFERENCE_ROOT). Without a reference tree nothing is built.
#
# ReferenceDecoder.h includes "Common.h", which a quoted include finds in the
# including file's directory. The header is therefore reached through a
# symbolic link in a build directory whose other link, Common.h, points at the
# stand-in: the reference file itself is read where it lies, not copied.
set -e
here="$(cd "$(dirname "$0")" && pwd)"
ref="${1:-${HF_REFERENCE_ROOT:-}}"
lib="$ref/Lib"
if [ -z "$ref" ] || [ ! -f "$lib/HuggingFaceEACP/Kernels/Int8Blocks.cpp" ]; then
    echo "reference tree not found (argument or HF_REFERENCE_ROOT); oracle/_ref not built" >&2
    exit 0
fi
out="$here/_ref"
obj="$out/obj"
mkdir -p "$obj"
flags="-std=c++20 -O2 -fPIC"
g++ $flags -I"$here/ref_shim" -I"$lib" -c "$lib/HuggingFaceEACP/Kernels/Int8Blocks.cpp" -o "$obj/int8_blocks.o"
g++ $flags -I"$here/ref_shim" -I"$lib" -c "$lib/HuggingFaceEACP/Sampling/Sampler.cpp" -o "$obj/sampler.o"
g++ $flags -I"$here/ref_shim" -I"$lib" -c "$here/ref_bridge.cpp" -o "$obj/ref_bridge.o"
for part in Tokenizer ByteFallback Metaspace SpecialTokens; do
    g++ $flags -I"$here/ref_shim" -I"$lib" -c "$lib/HuggingFaceEACP/Tokenizer/$part.cpp" -o "$obj/tokenizer_$part.o"
done
g++ $flags -I"$here/ref_shim" -I"$lib" -c "$here/ref_tokenizer_bridge.cpp" -o "$obj/ref_tokenizer_bridge.o"
links="$out/links/Decoder"
mkdir -p "$links"
ln -sf "$ref/Tests/Decoder/ReferenceDecoder.h" "$links/ReferenceDecoder.h"
ln -sf "$here/ref_shim/decoder/Common.h" "$links/Common.h"
g++ $flags -I"$here/ref_shim" -I"$out/links" -c "$here/ref_decoder_bridge.cpp" -o "$obj/ref_decoder_bridge.o"
g++ -shared -o "$out/libhf_ref.so" "$obj/int8_blocks.o" "$obj/sampler.o" "$obj/ref_bridge.o" "$obj/ref_decoder_bridge.o" \
    "$obj"/tokenizer_*.o "$obj/ref_tokenizer_bridge.o"
rm -f "$obj"/*.o "$links/ReferenceDecoder.h" "$links/Common.h"
echo "built $out/libhf_ref.so"

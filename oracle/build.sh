#!/bin/sh
# TEST INFRASTRUCTURE ONLY. Builds the C oracle into oracle/_build/liboracle.so.
set -e
here="$(cd "$(dirname "$0")" && pwd)"
mkdir -p "$here/_build"
gcc -std=c11 -O3 -march=x86-64-v3 -ffp-contract=off -fPIC -shared -pthread \
    "$here/oracle.c" -o "$here/_build/liboracle.so" -lm
echo "built $here/_build/liboracle.so"

#!/bin/sh
# Builds the CPU oracle library (test infrastructure) into oracle/_build/.
set -e
HERE=$(cd "$(dirname "$0")" && pwd)
mkdir -p "$HERE/_build"
gcc -O2 -ffp-contract=off -fopenmp -fPIC -shared -o "$HERE/_build/libbsa_oracle.so" "$HERE/bsa_oracle.c" -lm
echo "$HERE/_build/libbsa_oracle.so"

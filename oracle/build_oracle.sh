#!/usr/bin/env bash
# TEST INFRASTRUCTURE: builds the CPU oracle (cwen_oracle.c, this repo's own
# restatement) into oracle/liboracle.so.  Needs only gcc.
set -euo pipefail
here="$(cd "$(dirname "$0")" && pwd)"
gccdir="$(dirname "$(gcc -print-libgcc-file-name)")"
gcc -B"$gccdir/" -O2 -std=c11 -ffp-contract=off -fno-math-errno -fopenmp -fPIC -shared \
    -I"$here/../cwen_b200/host" -o "$here/liboracle.so" \
    "$here/cwen_oracle.c" "$here/../cwen_b200/host/synth.c" -lm -lpthread

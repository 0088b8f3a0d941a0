#!/usr/bin/env bash
# TEST INFRASTRUCTURE: compiles the reference engine (run.c, unmodified, read
# where it lies) into oracle/_ref/ for parity checks and the CPU baseline.
# Two builds: AVX-512 (the reference's AVX512=1 flags minus -march=native, so
# the library runs on any AVX-512 host) and AVX2 (its default flags).
# Usage: oracle/build_ref.sh [REFERENCE_DIR]  (default: $CWEN_REFERENCE_DIR, else
# a checkout named "reference" beside this repository)
set -euo pipefail
here="$(cd "$(dirname "$0")" && pwd)"
ref="${1:-${CWEN_REFERENCE_DIR:-$here/../../reference}}"
out="$here/_ref"
if [ ! -f "$ref/run.c" ]; then
  echo "build_ref: no reference at $ref (prebuilt libraries in $out are used as-is)" >&2
  exit 0
fi
mkdir -p "$out"
gccdir="$(dirname "$(gcc -print-libgcc-file-name)")"
CC="gcc -B$gccdir/"
base="-O3 -std=gnu11 -fopenmp -fPIC -mavx2 -mfma -mf16c -fno-math-errno -fno-trapping-math -fomit-frame-pointer"
avx512="-mavx512f -mavx512bw -mavx512vl -mavx512dq -mavx512vnni -DCWEN_AVX512"
src="$here/ref_harness.c $here/../cwen_b200/host/synth.c"
inc="-I$ref -I$here/../cwen_b200/host"
$CC $base $avx512 $inc -shared -o "$out/libcwref_avx512.so" $src -lm -lpthread
$CC $base $inc -shared -o "$out/libcwref_avx2.so" $src -lm -lpthread
# the reference CLI itself, for running on a GGUF file
$CC $base $avx512 -o "$out/run_avx512" "$ref/run.c" -lm
$CC $base -o "$out/run_avx2" "$ref/run.c" -lm
echo "build_ref: built $(ls "$out" | tr '\n' ' ')"

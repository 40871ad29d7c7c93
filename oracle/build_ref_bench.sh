#!/usr/bin/env bash
# Build the reference's own benchmark driver (kmeans/bench/main.cu, compiled
# unmodified from the read-only reference tree) twice, into oracle/_ref/:
#   mpkmeans_bench_ref   linked against oracle/_ref/libmpkref.so (the reference)
#   mpkmeans_bench_b200  linked against mpkmeans_b200/libmpkmeans_b200.so, with
#                        include/mpkmeans.h placed where main.cu includes it
#                        ("mpkmeans/mpkmeans.h")
# The second binary is the drop-in check: the reference's driver program runs
# on this library through the C ABI alone, and its --csv rows can be compared
# with the first binary's.  Both travel with the working tree (git-ignored).
# Usage: oracle/build_ref_bench.sh [REF_ROOT]   (needs libmpkref.so and
# libmpkmeans_b200.so built first)
set -euo pipefail
REF="${1:-${MPK_REFERENCE_ROOT:-/root/reference}}"
HERE="$(cd "$(dirname "$0")" && pwd)"
ROOT="$(cd "$HERE/.." && pwd)"
OUT="$HERE/_ref"
MAIN="$REF/kmeans/bench/main.cu"
if [ ! -f "$MAIN" ]; then
  echo "build_ref_bench.sh: $MAIN not found" >&2
  exit 1
fi
for lib in "$OUT/libmpkref.so" "$ROOT/mpkmeans_b200/libmpkmeans_b200.so"; do
  if [ ! -f "$lib" ]; then
    echo "build_ref_bench.sh: $lib is not built" >&2
    exit 1
  fi
done
NVCC="${NVCC:-nvcc}"
FLAGS="-O3 -std=c++17 -gencode arch=compute_100a,code=sm_100a -lineinfo -DMPK_STATS"
INC_B200="$OUT/include_b200"
mkdir -p "$INC_B200/mpkmeans"
cp "$ROOT/include/mpkmeans.h" "$INC_B200/mpkmeans/mpkmeans.h"

"$NVCC" $FLAGS -I"$REF/kmeans/include" -c "$MAIN" -o "$OUT/bench_main_ref.o"
"$NVCC" -gencode arch=compute_100a,code=sm_100a -o "$OUT/mpkmeans_bench_ref" "$OUT/bench_main_ref.o" \
  -L"$OUT" -lmpkref -lcublas -Xlinker -rpath -Xlinker '$ORIGIN'

"$NVCC" $FLAGS -I"$INC_B200" -c "$MAIN" -o "$OUT/bench_main_b200.o"
"$NVCC" -gencode arch=compute_100a,code=sm_100a -o "$OUT/mpkmeans_bench_b200" "$OUT/bench_main_b200.o" \
  -L"$ROOT/mpkmeans_b200" -lmpkmeans_b200 -lcublas -Xlinker -rpath -Xlinker '$ORIGIN/../../mpkmeans_b200'

rm -f "$OUT/bench_main_ref.o" "$OUT/bench_main_b200.o"
echo "built $OUT/mpkmeans_bench_ref and $OUT/mpkmeans_bench_b200"

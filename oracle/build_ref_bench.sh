#!/usr/bin/env bash
# Build the reference's own driver programs, compiled unmodified from the
# read-only reference tree, twice each into oracle/_ref/:
#   <name>_ref   linked against oracle/_ref/libmpkref.so (the reference)
#   <name>_b200  linked against mpkmeans_b200/libmpkmeans_b200.so, with this
#                library's headers placed where the programs include them
#                ("mpkmeans/mpkmeans.h", "mpemu/mpemu.h")
# Programs: mpkmeans_bench (kmeans/bench/main.cu) and, from gemm-emulation/bench,
# mpemu_test_split, mpemu_test_split_fp16, mpemu_test_refine, mpemu_test_concat
# (the reference's self-checking tests), mpemu_bench and mpemu_bench_mw (its
# accuracy/speed drivers) and mpemu_accum_probe.
# The _b200 binaries are the drop-in check: the reference's programs run on
# this library through the C ABI alone.  All travel with the working tree
# (git-ignored).
# Usage: oracle/build_ref_bench.sh REF_ROOT (or MPK_REFERENCE_ROOT)   (needs libmpkref.so and
# libmpkmeans_b200.so built first)
set -euo pipefail
REF="${1:-${MPK_REFERENCE_ROOT:-}}"
if [ -z "$REF" ]; then
  echo "$(basename "$0"): give the reference checkout as the first argument or in MPK_REFERENCE_ROOT" >&2
  exit 2
fi
HERE="$(cd "$(dirname "$0")" && pwd)"
ROOT="$(cd "$HERE/.." && pwd)"
OUT="$HERE/_ref"
if [ ! -d "$REF/kmeans/bench" ] || [ ! -d "$REF/gemm-emulation/bench" ]; then
  echo "build_ref_bench.sh: reference driver sources not found under $REF" >&2
  exit 1
fi
for lib in "$OUT/libmpkref.so" "$ROOT/mpkmeans_b200/libmpkmeans_b200.so"; do
  if [ ! -f "$lib" ]; then
    echo "build_ref_bench.sh: $lib is not built" >&2
    exit 1
  fi
done
NVCC="${NVCC:-nvcc}"
ARCH="-gencode arch=compute_100a,code=sm_100a"
FLAGS="-O3 -std=c++17 $ARCH -lineinfo -DMPK_STATS"
INC_B200="$OUT/include_b200"
mkdir -p "$INC_B200/mpkmeans" "$INC_B200/mpemu"
cp "$ROOT/include/mpkmeans.h" "$INC_B200/mpkmeans/mpkmeans.h"
cp "$ROOT/include/mpemu.h" "$INC_B200/mpemu/mpemu.h"
INC_REF="-I$REF/kmeans/include -I$REF/gemm-emulation/include"

# build NAME SOURCE: NAME_ref and NAME_b200 from one reference source file
build() {
  local name="$1" src="$REF/$2"
  "$NVCC" $FLAGS $INC_REF -c "$src" -o "$OUT/$name.ref.o"
  "$NVCC" $ARCH -o "$OUT/${name}_ref" "$OUT/$name.ref.o" \
    -L"$OUT" -lmpkref -lcublas -Xlinker -rpath -Xlinker '$ORIGIN'
  "$NVCC" $FLAGS -I"$INC_B200" -c "$src" -o "$OUT/$name.b200.o"
  "$NVCC" $ARCH -o "$OUT/${name}_b200" "$OUT/$name.b200.o" \
    -L"$ROOT/mpkmeans_b200" -lmpkmeans_b200 -lcublas -Xlinker -rpath -Xlinker '$ORIGIN/../../mpkmeans_b200'
  rm -f "$OUT/$name.ref.o" "$OUT/$name.b200.o"
}

build mpkmeans_bench kmeans/bench/main.cu
build mpemu_test_split gemm-emulation/bench/test_split.cu
build mpemu_test_split_fp16 gemm-emulation/bench/test_split_fp16.cu
build mpemu_test_refine gemm-emulation/bench/test_refine.cu
build mpemu_test_concat gemm-emulation/bench/test_concat.cu
build mpemu_bench gemm-emulation/bench/bench.cu
build mpemu_bench_mw gemm-emulation/bench/bench_mw.cu
build mpemu_accum_probe gemm-emulation/bench/accum_probe.cu
echo "built the reference's driver programs into $OUT (*_ref, *_b200)"

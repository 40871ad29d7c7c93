#!/usr/bin/env bash
# Build the reference's own k-means and split-GEMM code from its sources, as
# they lie in the read-only reference tree, into oracle/_ref/libmpkref.so.
# The libraries' own source lists are compiled directly (no CMake, no cuVS):
#   kmeans/src/{mpkmeans,kernels,data,multiword,baseline,cuvs_baseline}.cu
#   (multiword with its mpemu path on, -DMPK_MULTIWORD, as the reference's
#   CMake option does; cuvs_baseline without MPK_CUVS, i.e. its stub)
#   gemm-emulation/src/{split,gemm,util,split_fp16,gemm_fp16,context,batched,
#   concat,ozaki1,ozaki1_gemm}.cu (the whole libmpemu source list)
# MPK_STATS is on so that mpkMeansMixed's per-iteration FP32 verification
# (mpkmeans.cu:555-582) is available.  The output is git-ignored; it travels to
# the GPU box with the working tree.  Usage: oracle/build_ref.sh [REF_ROOT]
set -euo pipefail
REF="${1:-${MPK_REFERENCE_ROOT:-}}"
if [ -z "$REF" ]; then
  echo "$(basename "$0"): give the reference checkout as the first argument or in MPK_REFERENCE_ROOT" >&2
  exit 2
fi
HERE="$(cd "$(dirname "$0")" && pwd)"
OUT="$HERE/_ref"
if [ ! -d "$REF/kmeans/src" ]; then
  echo "build_ref.sh: reference tree not found at $REF" >&2
  exit 1
fi
mkdir -p "$OUT"
NVCC="${NVCC:-nvcc}"
FLAGS="-O3 -std=c++17 -Xcompiler -fPIC -gencode arch=compute_100a,code=sm_100a -lineinfo -DMPK_STATS"
INC="-I$REF/kmeans/include -I$REF/kmeans/src -I$REF/gemm-emulation/include -I$REF/gemm-emulation/src"
OBJS=()
for f in kmeans/src/mpkmeans.cu kmeans/src/kernels.cu kmeans/src/data.cu kmeans/src/multiword.cu \
         kmeans/src/baseline.cu kmeans/src/cuvs_baseline.cu \
         gemm-emulation/src/split.cu gemm-emulation/src/gemm.cu gemm-emulation/src/util.cu \
         gemm-emulation/src/split_fp16.cu gemm-emulation/src/gemm_fp16.cu \
         gemm-emulation/src/context.cu gemm-emulation/src/batched.cu gemm-emulation/src/concat.cu \
         gemm-emulation/src/ozaki1.cu gemm-emulation/src/ozaki1_gemm.cu; do
  o="$OUT/$(echo "$f" | tr '/' '_' ).o"
  EXTRA=""
  [ "$f" = kmeans/src/multiword.cu ] && EXTRA="-DMPK_MULTIWORD"
  "$NVCC" $FLAGS $EXTRA $INC -c "$REF/$f" -o "$o"
  OBJS+=("$o")
done
"$NVCC" -shared -gencode arch=compute_100a,code=sm_100a -o "$OUT/libmpkref.so" "${OBJS[@]}" -lcublas
rm -f "${OBJS[@]}"
echo "built $OUT/libmpkref.so"

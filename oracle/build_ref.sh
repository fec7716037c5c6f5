#!/usr/bin/env bash
# Compiles the reference's own hot-path CUDA sources, where they lie, into
# oracle/_ref/libkcref.so (git-ignored; shipped with the tree as a built file).
# TEST INFRASTRUCTURE ONLY: the parity tests load it as a second, independent
# oracle on the B200.  Nothing is copied out of the reference tree.
#
#   KC_REF_DIR  kernel-craft checkout (default: a checkout named "reference"
#               beside this repository); the step is skipped where none exists.
set -euo pipefail
HERE="$(cd "$(dirname "${BASH_SOURCE[0]}")" && pwd)"
REF="${KC_REF_DIR:-$HERE/../../reference}"
SRC="$REF/src/kernels/transformer"
OUT="$HERE/_ref"
if [ ! -f "$SRC/quant_int4.cu" ]; then
  echo "build_ref: reference sources not found under $REF; keeping prebuilt $OUT (if any)"
  exit 0
fi
mkdir -p "$OUT/obj"
NVCC="${NVCC:-nvcc}"
FLAGS=(-gencode arch=compute_100a,code=sm_100a -O3 -Xcompiler -fPIC -std=c++17)
for f in quant_int4 fp8_quant tensor_parallel; do
  "$NVCC" "${FLAGS[@]}" -c "$SRC/$f.cu" -o "$OUT/obj/$f.o"
done
"$NVCC" "${FLAGS[@]}" -DHAVE_NCCL -c "$SRC/tensor_parallel_nccl.cu" -o "$OUT/obj/tensor_parallel_nccl.o"
"$NVCC" -shared -gencode arch=compute_100a,code=sm_100a -o "$OUT/libkcref.so" "$OUT"/obj/*.o -lnccl
rm -rf "$OUT/obj"
echo "build_ref: wrote $OUT/libkcref.so"

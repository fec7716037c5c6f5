#!/usr/bin/env bash
# Compiles the reference's own CALLERS of this path -- its C++ unit tests, its
# quantization benchmark and its pybind11 module -- unchanged, from the
# sources where they lie, against THIS library's libkernels.so, into
# oracle/_ref/callers/ (git-ignored; shipped with the tree as built files).
# TEST INFRASTRUCTURE ONLY: tests/test_ref_callers_gpu.py runs them on the
# B200 to show the drop-in boundary holds for the reference's own code.
# Nothing is copied out of the reference tree.
#
#   tests/test_quant_int4.cpp       launch_dequantize_int4, launch_gemv_int4
#   tests/test_fp8_quant.cpp        launch_quantize_fp8, launch_dequantize_fp8,
#                                   launch_smoothquant_scale
#   tests/test_tensor_parallel.cpp  launch_ring_allreduce, launch_allgather,
#                                   launch_col/row_parallel_linear, nccl_* (-DHAVE_NCCL)
#   benchmarks/benchmark_quant.cpp  the four quantization launchers
#   benchmarks/benchmark_tensor_parallel.cpp  launch_ring_allreduce, launch_allgather,
#                                   launch_col/row_parallel_linear, nccl_* (-DHAVE_NCCL)
#   src/python/pybind_transformer.cpp -> kernel_craft_transformer<ext>
#
# Each links -lkernels from kernel-craft_b200/lib with an $ORIGIN-relative
# rpath, so the binaries find the library wherever the tree is unpacked.
#
#   KC_REF_DIR  kernel-craft checkout (default: a checkout named "reference"
#               beside this repository); the step is skipped where none exists.
set -euo pipefail
HERE="$(cd "$(dirname "${BASH_SOURCE[0]}")" && pwd)"
ROOT="$(cd "$HERE/.." && pwd)"
REF="${KC_REF_DIR:-$HERE/../../reference}"
OUT="$HERE/_ref/callers"
LIBDIR="$ROOT/kernel-craft_b200/lib"
if [ ! -f "$REF/tests/test_quant_int4.cpp" ]; then
  echo "build_ref_callers: reference sources not found under $REF; keeping prebuilt $OUT (if any)"
  exit 0
fi
if [ ! -f "$LIBDIR/libkernels.so" ]; then
  echo "build_ref_callers: $LIBDIR/libkernels.so missing (python kernel-craft_b200/build.py)" >&2
  exit 1
fi
mkdir -p "$OUT"
CUDA_HOME="${CUDA_HOME:-/usr/local/cuda}"
CXX="${CXX:-g++}"
PY="${PYTHON:-python3}"
# from oracle/_ref/callers/ back to the repository root
RPATH='-Wl,-rpath,$ORIGIN/../../../kernel-craft_b200/lib'
COMMON=(-O2 -std=c++17 -I "$CUDA_HOME/include")
LINK=(-L "$LIBDIR" -lkernels -L "$CUDA_HOME/lib64" -lcudart "$RPATH")

"$CXX" "${COMMON[@]}" "$REF/tests/test_quant_int4.cpp" -o "$OUT/test_quant_int4" "${LINK[@]}"
"$CXX" "${COMMON[@]}" "$REF/tests/test_fp8_quant.cpp" -o "$OUT/test_fp8_quant" "${LINK[@]}"
"$CXX" "${COMMON[@]}" -DHAVE_NCCL "$REF/tests/test_tensor_parallel.cpp" -o "$OUT/test_tensor_parallel" \
  "${LINK[@]}" -lnccl
"$CXX" "${COMMON[@]}" "$REF/benchmarks/benchmark_quant.cpp" -o "$OUT/benchmark_quant" "${LINK[@]}"
"$CXX" "${COMMON[@]}" -DHAVE_NCCL "$REF/benchmarks/benchmark_tensor_parallel.cpp" \
  -o "$OUT/benchmark_tensor_parallel" "${LINK[@]}" -lnccl

PYBIND_INC="$("$PY" -c 'import pybind11; print(pybind11.get_include())')"
PY_INC="$("$PY" -c 'import sysconfig; print(sysconfig.get_paths()["include"])')"
EXT="$("$PY" -c 'import sysconfig; print(sysconfig.get_config_var("EXT_SUFFIX"))')"
"$CXX" "${COMMON[@]}" -shared -fPIC -fvisibility=hidden -I "$PYBIND_INC" -I "$PY_INC" \
  "$REF/src/python/pybind_transformer.cpp" -o "$OUT/kernel_craft_transformer$EXT" "${LINK[@]}"
echo "build_ref_callers: wrote $OUT"

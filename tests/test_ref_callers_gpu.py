"""GPU: the reference's own callers of this path, compiled unchanged against
this library (oracle/build_ref_callers.sh), run on the B200.

* tests/test_quant_int4.cpp, tests/test_fp8_quant.cpp and
  tests/test_tensor_parallel.cpp (with -DHAVE_NCCL) -- the reference's C++
  unit tests for the launchers this library replaces: exit status 0 and no
  "[FAIL]" line, with their own tolerances;
* benchmarks/benchmark_quant.cpp and benchmarks/benchmark_tensor_parallel.cpp
  -- run to completion;
* src/python/pybind_transformer.cpp (module kernel_craft_transformer) --
  imports against libkernels.so, and its quantization and tensor-parallel
  functions agree with the oracle: dequantized INT4 weights, FP8 codes and
  scales bit-exact, the fp32 shard GEMMs within 1e-5 normwise.

Skipped where the binaries were not built (no reference checkout when the
tree was built).
"""
import os
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

import oracle as O
from kc_testutil import normwise_err

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parent.parent
CALLERS = ROOT / "oracle" / "_ref" / "callers"


def _binary(name):
    p = CALLERS / name
    if not p.exists():
        pytest.skip(f"{name} not built (oracle/build_ref_callers.sh needs the reference checkout)")
    return p


@pytest.mark.parametrize("name", ["test_quant_int4", "test_fp8_quant", "test_tensor_parallel"])
def test_reference_cpp_test_passes(cuda, name):
    out = subprocess.run([str(_binary(name))], capture_output=True, text=True, timeout=300,
                         cwd=CALLERS)
    log = out.stdout + out.stderr
    print(log[-4000:])
    assert out.returncode == 0, log[-4000:]
    assert "[FAIL]" not in log
    assert "[PASS]" in log


def test_reference_quant_benchmark_runs(cuda):
    out = subprocess.run([str(_binary("benchmark_quant"))], capture_output=True, text=True,
                         timeout=300, cwd=CALLERS)
    print(out.stdout[-4000:])
    assert out.returncode == 0, (out.stdout + out.stderr)[-4000:]
    assert "GB/s" in out.stdout


def test_reference_tensor_parallel_benchmark_runs(cuda, tmp_path):
    """benchmarks/benchmark_tensor_parallel.cpp: the simulated collectives and
    the parallel linears at its own sizes (it appends a report file in its
    working directory, here a temporary one); its same-device NCCL case
    reports that NCCL refused and skips, as the reference handles it."""
    out = subprocess.run([str(_binary("benchmark_tensor_parallel"))], capture_output=True, text=True,
                         timeout=300, cwd=tmp_path)
    print(out.stdout[-4000:])
    assert out.returncode == 0, (out.stdout + out.stderr)[-4000:]
    assert "Benchmark complete" in out.stdout and "GB/s" in out.stdout


@pytest.fixture(scope="module")
def ktr():
    if not any(CALLERS.glob("kernel_craft_transformer*.so")):
        pytest.skip("pybind module not built (oracle/build_ref_callers.sh)")
    sys.path.insert(0, str(CALLERS))
    try:
        import kernel_craft_transformer as m
    finally:
        sys.path.remove(str(CALLERS))
    return m


def test_pybind_int4_dequant_bitexact(cuda, ktr):
    rng = np.random.default_rng(31)
    rows, cols, gs = 96, 1024, 128
    packed = rng.integers(0, 256, (rows, cols // 2), dtype=np.uint8)
    scales = rng.uniform(0.002, 0.02, (rows, cols // gs)).astype(np.float32)
    zeros = rng.integers(0, 256, (rows, cols // gs // 2), dtype=np.uint8)
    out = ktr.quant_int4_dequant(packed, scales, zeros, rows, cols, gs)
    np.testing.assert_array_equal(out, O.dequantize_int4(packed, scales, zeros, rows, cols, gs))


def test_pybind_fp8_quantize_bitexact(cuda, ktr):
    x = O.make_outlier_activations(64, 2048, seed=32)
    q, s = ktr.fp8_quantize(x, per_token=True)
    qr, sr = O.quantize_fp8_per_token(x)
    np.testing.assert_array_equal(np.asarray(q).view(np.uint8), qr)
    np.testing.assert_array_equal(s, sr)
    # per tensor: the module computes the scale on the host, the library quantizes
    qt, st = ktr.fp8_quantize(x, per_token=False)
    assert st[0] == O.per_tensor_scale(x)
    np.testing.assert_array_equal(np.asarray(qt).view(np.uint8), O.quantize_fp8_per_tensor(x, st[0]))
    back = ktr.fp8_dequantize(q, s, 64, 2048, True)
    np.testing.assert_array_equal(back, O.dequantize_fp8(qr, sr, 64, 2048, True))


def test_pybind_parallel_linears(cuda, ktr):
    rng = np.random.default_rng(33)
    M, N, K, R = 48, 96, 256, 2
    x = rng.standard_normal((M, K)).astype(np.float32)
    W = rng.standard_normal((N, K)).astype(np.float32)
    ref = O.gemm_nt_f32(x, W)
    # column parallel: each rank's weight rows, outputs side by side
    cols = [ktr.col_parallel_linear(x, np.ascontiguousarray(W[r * N // R:(r + 1) * N // R]))
            for r in range(R)]
    assert normwise_err(np.concatenate(cols, axis=1), ref) <= 1e-5
    # row parallel: K shards, partials summed by the module's simulated all-reduce
    parts = [ktr.row_parallel_linear(np.ascontiguousarray(x[:, r * K // R:(r + 1) * K // R]),
                                     np.ascontiguousarray(W[:, r * K // R:(r + 1) * K // R]))
             for r in range(R)]
    summed = ktr.ring_allreduce([p.reshape(-1).copy() for p in parts])
    assert normwise_err(np.asarray(summed[0]).reshape(M, N), ref) <= 1e-5

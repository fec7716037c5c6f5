"""Regenerates tests/golden/kat_*.npz from the reference's own known-answer tests.

    python tests/golden/make_golden.py      # needs the reference checkout (KC_REF_DIR)

Each fixture re-creates one reference test's inputs and expected outputs with
the reference's own generators, so the oracle can be pinned against them on
any machine:
  * C++ tests (tests/test_quant_int4.cpp, tests/test_fp8_quant.cpp,
    tests/test_tensor_parallel.cpp) seed glibc srand()/rand(); glibc's
    generator is called through ctypes to reproduce the exact sequences, and
    the tests' fp32 CPU reference loops are replayed in float32.
  * pytest tests (src/python/tests/test_transformer_bindings.py) use
    numpy default_rng(42).
  * src/python/tests/test_triton_kernels.py holds a numpy INT4 dequant+GEMV
    reference (_int4_dequant_gemv_ref) and data generator (_make_int4_data);
    both are loaded from the reference file's source (its module-level code
    needs a GPU, so the two functions are extracted with ast) and executed.
Nothing here runs on the GPU; the bit-exact FP8 pins come from
make_golden_ref.py, which runs the reference's CUDA kernels on a B200.
"""
from __future__ import annotations

import ast
import ctypes
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
# the kernel-craft checkout: $KC_REF_DIR, else one named "reference" beside this repository
REF = Path(os.environ.get("KC_REF_DIR", HERE.parent.parent.parent / "reference"))
RAND_MAX = 2147483647
f32 = np.float32

libc = ctypes.CDLL("libc.so.6")
libc.rand.restype = ctypes.c_int
libc.srand.argtypes = [ctypes.c_uint]


def c_rand_uniform():
    """((float)rand() / RAND_MAX) as the reference C++ tests compute it."""
    return f32(libc.rand()) / f32(RAND_MAX)


def pack_nibbles(w: np.ndarray) -> np.ndarray:
    """test_quant_int4.cpp:31-33: low nibble = first value."""
    lo = (w[:, 0::2].astype(np.int32) & 0x0F)
    hi = (w[:, 1::2].astype(np.int32) & 0x0F) << 4
    return (lo | hi).astype(np.uint8)


def kat_quant_int4() -> dict:
    out = {}
    # test_dequantize_correctness, test_quant_int4.cpp:35-88
    rows, cols, gs = 4, 8, 8
    w = np.array([(i % 16) - 8 for i in range(rows * cols)], np.int8).reshape(rows, cols)
    sc = cols // gs
    zc = sc // 2 + sc % 2
    out["deq4x8_packed"] = pack_nibbles(w)
    out["deq4x8_scales"] = np.full((rows, sc), f32(0.125), np.float32)
    out["deq4x8_zeros"] = np.zeros((rows, zc), np.uint8)
    out["deq4x8_expected"] = (w.astype(np.float32) * f32(0.125)).astype(np.float32)

    # test_gemv_correctness, :90-146 (srand(42))
    rows, cols, gs = 16, 16, 8
    libc.srand(42)
    w = np.array([(libc.rand() % 15) - 7 for _ in range(rows * cols)], np.int8).reshape(rows, cols)
    x = np.array([c_rand_uniform() * f32(2) - f32(1) for _ in range(cols)], np.float32)
    sc = cols // gs
    zc = sc // 2 + sc % 2
    y = np.zeros(rows, np.float32)
    for r in range(rows):
        for c in range(cols):  # y_ref[r] += (float)w * scale_val * x[c]   (:117-121)
            y[r] = f32(y[r] + f32(f32(f32(w[r, c]) * f32(0.1)) * x[c]))
    out["gemv16_packed"] = pack_nibbles(w)
    out["gemv16_scales"] = np.full((rows, sc), f32(0.1), np.float32)
    out["gemv16_zeros"] = np.zeros((rows, zc), np.uint8)
    out["gemv16_x"] = x
    out["gemv16_expected"] = y

    # test_multi_group, :148-199 (srand(13))
    rows, cols, gs = 4, 128, 64
    libc.srand(13)
    w = np.array([(libc.rand() % 15) - 7 for _ in range(rows * cols)], np.int8).reshape(rows, cols)
    sc = cols // gs
    zc = sc // 2 + sc % 2
    scales = np.array([f32(0.05) + f32(0.01) * f32(i) for i in range(rows * sc)],
                      np.float32).reshape(rows, sc)
    exp = np.empty((rows, cols), np.float32)
    for r in range(rows):
        for c in range(cols):
            exp[r, c] = f32(f32(w[r, c]) * scales[r, c // gs])
    out["mg_packed"] = pack_nibbles(w)
    out["mg_scales"] = scales
    out["mg_zeros"] = np.zeros((rows, zc), np.uint8)
    out["mg_expected"] = exp
    return out


def kat_bindings() -> dict:
    # src/python/tests/test_transformer_bindings.py:185-196 (TestQuantInt4.test_dequant_roundtrip)
    rows, cols, gs = 4, 16, 8
    rng = np.random.default_rng(42)
    w = rng.integers(-7, 8, (rows, cols), dtype=np.int8)
    sc = cols // gs
    out = {
        "bind_packed": pack_nibbles(w),
        "bind_scales": np.full((rows, sc), f32(0.125), np.float32),
        "bind_zeros": np.zeros((rows, sc // 2 + sc % 2), np.uint8),
        "bind_expected": w.astype(np.float32) * f32(0.125),
    }
    # TestFP8Quant.test_per_token_roundtrip (:213-221): rng(42) uniform(-1,1) (8, 64)
    rng = np.random.default_rng(42)
    out["bind_fp8_in"] = rng.uniform(-1, 1, (8, 64)).astype(np.float32)
    return out


def _load_triton_ref():
    src = (REF / "src/python/tests/test_triton_kernels.py").read_text()
    tree = ast.parse(src)
    keep = [n for n in tree.body if isinstance(n, ast.FunctionDef)
            and n.name in ("_int4_dequant_gemv_ref", "_make_int4_data")]
    mod = ast.Module(body=keep, type_ignores=[])
    ns = {"np": np}
    exec(compile(mod, str(REF / "src/python/tests/test_triton_kernels.py"), "exec"), ns)
    return ns["_make_int4_data"], ns["_int4_dequant_gemv_ref"]


def kat_triton() -> dict:
    make, ref = _load_triton_ref()
    out = {}
    # TestInt4GemvTriton cases (:230-257): (rows, cols, gs, seed)
    for tag, (rows, cols, gs, seed) in {"small": (4, 256, 128, 0), "medium": (64, 1024, 128, 7),
                                        "gs64": (8, 512, 64, 3)}.items():
        packed, scales, zeros, x = make(rows, cols, gs, seed)
        y = ref(packed, scales, zeros, x, rows, cols, gs)
        out[f"tri_{tag}_packed"] = packed
        out[f"tri_{tag}_scales"] = scales
        out[f"tri_{tag}_zeros"] = zeros
        out[f"tri_{tag}_x"] = x
        out[f"tri_{tag}_expected"] = y
        out[f"tri_{tag}_shape"] = np.array([rows, cols, gs], np.int32)
    return out


def kat_fp8() -> dict:
    out = {}
    # test_per_token_roundtrip, tests/test_fp8_quant.cpp:34-71 (srand(42), 8x64)
    libc.srand(42)
    out["pt_in"] = np.array([c_rand_uniform() * f32(2) - f32(1) for _ in range(8 * 64)],
                            np.float32).reshape(8, 64)
    # test_smoothquant_scaling, :99-135 (exact expected: all ones)
    x = np.ones((4, 16), np.float32)
    x[:, 0] = 100.0
    s = np.ones(16, np.float32)
    s[0] = 100.0
    out["sq_in"], out["sq_smooth"], out["sq_expected"] = x, s, np.ones((4, 16), np.float32)
    # test_per_tensor_roundtrip, :137-174 (srand(7), 4x32, scale = max_abs / 448.f)
    libc.srand(7)
    vals, max_abs = [], f32(0)
    for _ in range(4 * 32):
        v = c_rand_uniform() * f32(4) - f32(2)
        vals.append(v)
        max_abs = max(max_abs, abs(v))
    out["tensor_in"] = np.array(vals, np.float32).reshape(4, 32)
    out["tensor_scale"] = np.array([f32(max_abs) / f32(448)], np.float32)
    return out


def kat_tensor_parallel() -> dict:
    out = {}

    def cpu_gemm_nt(A, B):  # tests/test_tensor_parallel.cpp:67-78, fp32 in k order
        M, K = A.shape
        N = B.shape[0]
        C = np.zeros((M, N), np.float32)
        for m in range(M):
            for n in range(N):
                acc = f32(0)
                for k in range(K):
                    acc = f32(acc + f32(A[m, k] * B[n, k]))
                C[m, n] = acc
        return C

    # test_col_parallel_linear_2ranks (:209-259)
    M, N, K = 4, 6, 8
    x = np.array([f32(i % 7) * f32(0.1) + f32(0.05) for i in range(M * K)], np.float32).reshape(M, K)
    W = np.array([f32((i * 3 + 1) % 11) * f32(0.1) - f32(0.5) for i in range(N * K)],
                 np.float32).reshape(N, K)
    out["col_x"], out["col_W"], out["col_ref"] = x, W, cpu_gemm_nt(x, W)
    # test_row_parallel_linear_2ranks (:272-330)
    x = np.array([f32(i % 5) * f32(0.2) + f32(0.1) for i in range(M * K)], np.float32).reshape(M, K)
    W = np.array([f32((i * 7 + 3) % 13) * f32(0.1) - f32(0.6) for i in range(N * K)],
                 np.float32).reshape(N, K)
    out["row_x"], out["row_W"], out["row_ref"] = x, W, cpu_gemm_nt(x, W)
    # test_col_then_row_parallel_identity (:339-376)
    M, K, H, N = 3, 8, 6, 4
    x = np.array([f32(i % 7 + 1) * f32(0.1) for i in range(M * K)], np.float32).reshape(M, K)
    W1 = np.array([f32(i % 5 - 2) * f32(0.1) for i in range(H * K)], np.float32).reshape(H, K)
    W2 = np.array([f32(i % 3 - 1) * f32(0.15) for i in range(N * H)], np.float32).reshape(N, H)
    mid = cpu_gemm_nt(x, W1)
    out["chain_x"], out["chain_W1"], out["chain_W2"] = x, W1, W2
    out["chain_ref"] = cpu_gemm_nt(mid, W2)
    # simulated collectives (:84-196)
    out["ar2_in"] = np.array([[1, 2, 3, 4], [1, 2, 3, 4]], np.float32)
    out["ar2_expected"] = np.array([2, 4, 6, 8], np.float32)
    out["ar4_in"] = np.tile(np.arange(1, 9, dtype=np.float32), (4, 1))
    out["ar4_expected"] = 4 * np.arange(1, 9, dtype=np.float32)
    out["ag_chunks"] = np.array([[r * 10 + i for i in range(3)] for r in range(4)], np.float32)
    out["ag_expected"] = out["ag_chunks"].reshape(-1)
    return out


def main() -> int:
    if not (REF / "src/kernels/transformer/quant_int4.cu").exists():
        print(f"reference checkout not found at {REF}", file=sys.stderr)
        return 1
    np.savez_compressed(HERE / "kat_quant_int4.npz", **kat_quant_int4())
    np.savez_compressed(HERE / "kat_bindings.npz", **kat_bindings())
    np.savez_compressed(HERE / "kat_triton_int4.npz", **kat_triton())
    np.savez_compressed(HERE / "kat_fp8.npz", **kat_fp8())
    np.savez_compressed(HERE / "kat_tensor_parallel.npz", **kat_tensor_parallel())
    print("wrote", sorted(p.name for p in HERE.glob("kat_*.npz")))
    return 0


if __name__ == "__main__":
    sys.exit(main())

"""numpy front end of the CPU oracle (oracle/kc_oracle.c -> oracle/lib/liboracle.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
CPU-baseline leg of bench.py, always as the checker, never as the measured or
shipped path.  Build with ``make -C oracle``.

Also generates the seeded synthetic inputs shared by the oracle, the CPU
baseline and the GPU runs (numpy PCG64, seed 0 by default), with the value
distributions of the benchmark configurations (uniform nibbles, scales in
[0.002, 0.02], N(0, 1) activations, 1 % outlier channels, N(0, 0.02) weights).
"""
from __future__ import annotations

import ctypes
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "lib" / "liboracle.so"

_vp = ctypes.c_void_p
_ci = ctypes.c_int
_cl = ctypes.c_long
_lib = None


def _p(a: np.ndarray) -> ctypes.c_void_p:
    assert a.flags["C_CONTIGUOUS"], "oracle arrays must be C-contiguous"
    return ctypes.c_void_p(a.ctypes.data)


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise FileNotFoundError(f"{LIB_PATH} missing: run `make -C oracle`")
        l = ctypes.CDLL(str(LIB_PATH))
        protos = {
            "ora_unpack_nibble": (_ci, [ctypes.c_uint8, _ci]),
            "ora_dequantize_int4": (None, [_vp] * 4 + [_ci] * 3),
            "ora_gemv_int4": (None, [_vp] * 5 + [_ci] * 3),
            "ora_float_to_bf16": (ctypes.c_uint16, [ctypes.c_float]),
            "ora_dequantize_w4_bf16": (None, [_vp] * 3 + [_ci] * 3),
            "ora_dequantize_w4_bf16_zp": (None, [_vp] * 4 + [_ci] * 3),
            "ora_gemv_w4a16": (None, [_vp] * 4 + [_ci] * 4),
            "ora_gemv_w4a16_zp": (None, [_vp] * 5 + [_ci] * 4),
            "ora_e4m3_encode": (ctypes.c_uint8, [ctypes.c_float]),
            "ora_e4m3_decode": (ctypes.c_float, [ctypes.c_uint8]),
            "ora_e4m3_encode_array": (None, [_vp, _vp, _cl, _ci]),
            "ora_quantize_fp8_per_token": (None, [_vp] * 3 + [_ci] * 2),
            "ora_quantize_fp8_per_tensor": (None, [_vp, _vp, ctypes.c_float, _cl]),
            "ora_dequantize_fp8": (None, [_vp] * 3 + [_ci] * 3),
            "ora_smoothquant_scale": (None, [_vp] * 3 + [_ci] * 2),
            "ora_gemm_nt_f32": (None, [_vp] * 3 + [_ci] * 3),
            "ora_gemm_fp8_rowcol": (None, [_vp] * 5 + [_ci] * 3),
            "ora_gemm_w4a16": (None, [_vp] * 4 + [_ci] * 4),
            "ora_gemm_w4a16_zp": (None, [_vp] * 5 + [_ci] * 4),
            "ora_ring_allreduce": (None, [_vp, _ci, _ci]),
            "ora_allgather": (None, [_vp, _vp, _ci, _ci]),
            "ora_num_threads": (_ci, []),
            "ora_set_num_threads": (None, [_ci]),
        }
        for name, (res, args) in protos.items():
            fn = getattr(l, name)
            fn.restype, fn.argtypes = res, args
        _lib = l
    return _lib


def _c(a, dtype) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=dtype)


# --------------------------------------------------------------------------
# INT4 (reference semantics)
# --------------------------------------------------------------------------

def dequantize_int4(packed, scales, zeros, rows, cols, gs) -> np.ndarray:
    packed, scales, zeros = _c(packed, np.uint8), _c(scales, np.float32), _c(zeros, np.uint8)
    out = np.empty((rows, cols), np.float32)
    lib().ora_dequantize_int4(_p(packed), _p(scales), _p(zeros), _p(out), rows, cols, gs)
    return out


def gemv_int4(packed, scales, zeros, x, rows, cols, gs) -> np.ndarray:
    packed, scales, zeros = _c(packed, np.uint8), _c(scales, np.float32), _c(zeros, np.uint8)
    x = _c(x, np.float32)
    y = np.empty(rows, np.float32)
    lib().ora_gemv_int4(_p(packed), _p(scales), _p(zeros), _p(x), _p(y), rows, cols, gs)
    return y


# --------------------------------------------------------------------------
# GPTQ W4A16 (implicit zero-point 8, fp16 scales, bf16 activations)
# --------------------------------------------------------------------------

def _zeros(zeros, N, K, gs):
    """Per-group zero points as a contiguous u8 [N, K/gs] array, or None (symmetric, 8)."""
    if zeros is None:
        return None
    z = _c(zeros, np.uint8)
    assert z.shape == (N, K // gs), z.shape
    return z


def dequantize_w4_bf16(packed, scales_f16, N, K, gs, zeros=None) -> np.ndarray:
    """Returns the bf16 bit patterns (uint16) of the dequantized weights
    bf16((u - z) * s); zeros None means z = 8 (symmetric GPTQ)."""
    packed = _c(packed, np.uint8)
    s = _c(np.asarray(scales_f16).view(np.uint16), np.uint16)
    z = _zeros(zeros, N, K, gs)
    out = np.empty((N, K), np.uint16)
    lib().ora_dequantize_w4_bf16_zp(_p(packed), _p(s), _p(z) if z is not None else None, _p(out),
                                    N, K, gs)
    return out


def gemv_w4a16(packed, scales_f16, x_bf16_bits, M, N, K, gs, zeros=None) -> np.ndarray:
    packed = _c(packed, np.uint8)
    s = _c(np.asarray(scales_f16).view(np.uint16), np.uint16)
    x = _c(x_bf16_bits, np.uint16)
    z = _zeros(zeros, N, K, gs)
    y = np.empty((M, N), np.float32)
    lib().ora_gemv_w4a16_zp(_p(packed), _p(s), _p(z) if z is not None else None, _p(x), _p(y),
                            M, N, K, gs)
    return y


def gemm_w4a16(a_bf16_bits, packed, scales_f16, M, N, K, gs, zeros=None) -> np.ndarray:
    a = _c(a_bf16_bits, np.uint16)
    packed = _c(packed, np.uint8)
    s = _c(np.asarray(scales_f16).view(np.uint16), np.uint16)
    z = _zeros(zeros, N, K, gs)
    c = np.empty((M, N), np.float32)
    lib().ora_gemm_w4a16_zp(_p(a), _p(packed), _p(s), _p(z) if z is not None else None, _p(c),
                            M, N, K, gs)
    return c


def gelu_quick(h) -> np.ndarray:
    """x * sigmoid(1.702 x) in fp32, the activation of the reference's MLP block
    (examples/python/transformer/tensor_parallel.py:162)."""
    h = np.asarray(h, np.float32)
    with np.errstate(over="ignore"):
        return (h * (np.float32(1) / (np.float32(1) + np.exp(np.float32(-1.702) * h)))).astype(np.float32)


def mlp_block_w4a16(x_bf16_bits, w1_packed, w1_scales_f16, w2_packed, w2_scales_f16, M, H, I, gs,
                    act: str = "gelu_quick") -> np.ndarray:
    """The reference's MLP block (col-parallel linear -> GELU -> row-parallel
    linear -> all-reduce, examples/python/transformer/tensor_parallel.py:150-172;
    without the activation, test_tensor_parallel.cpp:339-376) on W4A16 weights:
    h = act(x . W1^T) in fp32 (W1 [I, H]), rounded to bf16 as the input of the
    second GEMM, y = h . W2^T in fp32 (W2 [H, I]).  A sharded run computes the
    same y as the sum over ranks of h[:, shard] . W2[:, shard]^T."""
    h = gemm_w4a16(x_bf16_bits, w1_packed, w1_scales_f16, M, I, H, gs)
    if act == "gelu_quick":
        h = gelu_quick(h)
    elif act != "none":
        raise ValueError(act)
    return gemm_w4a16(f32_to_bf16_bits(h), w2_packed, w2_scales_f16, M, H, I, gs)


# --------------------------------------------------------------------------
# FP8
# --------------------------------------------------------------------------

def e4m3_encode(x, clamp: bool = True) -> np.ndarray:
    x = _c(x, np.float32)
    out = np.empty(x.shape, np.uint8)
    lib().ora_e4m3_encode_array(_p(x), _p(out), x.size, 1 if clamp else 0)
    return out


def e4m3_decode_table() -> np.ndarray:
    return np.array([lib().ora_e4m3_decode(i) for i in range(256)], np.float32)


def quantize_fp8_per_token(x):
    x = _c(x, np.float32)
    rows, cols = x.shape
    q = np.empty((rows, cols), np.uint8)
    s = np.empty(rows, np.float32)
    lib().ora_quantize_fp8_per_token(_p(x), _p(q), _p(s), rows, cols)
    return q, s


def quantize_fp8_per_tensor(x, scale: float) -> np.ndarray:
    x = _c(x, np.float32)
    q = np.empty(x.shape, np.uint8)
    lib().ora_quantize_fp8_per_tensor(_p(x), _p(q), float(scale), x.size)
    return q


def per_tensor_scale(x) -> np.float32:
    """amax/448 (1 if amax == 0), amax ignoring NaN -- pybind_transformer.cpp:305-311."""
    a = np.abs(np.asarray(x, np.float32).ravel())
    a = a[~np.isnan(a)]
    amax = np.float32(a.max()) if a.size else np.float32(0)
    return np.float32(amax / np.float32(448.0)) if amax > 0 else np.float32(1.0)


def dequantize_fp8(q, scales, rows, cols, per_token: bool) -> np.ndarray:
    q = _c(np.asarray(q).view(np.uint8), np.uint8)
    scales = _c(scales, np.float32)
    out = np.empty((rows, cols), np.float32)
    lib().ora_dequantize_fp8(_p(q), _p(scales), _p(out), rows, cols, 1 if per_token else 0)
    return out


def smoothquant_scale(x, s) -> np.ndarray:
    x, s = _c(x, np.float32), _c(s, np.float32)
    rows, cols = x.shape
    out = np.empty_like(x)
    lib().ora_smoothquant_scale(_p(x), _p(s), _p(out), rows, cols)
    return out


# --------------------------------------------------------------------------
# GEMMs and simulated collectives
# --------------------------------------------------------------------------

def gemm_nt_f32(A, B) -> np.ndarray:
    A, B = _c(A, np.float32), _c(B, np.float32)
    M, K = A.shape
    N = B.shape[0]
    C = np.empty((M, N), np.float32)
    lib().ora_gemm_nt_f32(_p(A), _p(B), _p(C), M, N, K)
    return C


def gemm_fp8_rowcol(a_codes, sa, w_codes, sw) -> np.ndarray:
    a = _c(np.asarray(a_codes).view(np.uint8), np.uint8)
    w = _c(np.asarray(w_codes).view(np.uint8), np.uint8)
    sa, sw = _c(sa, np.float32), _c(sw, np.float32)
    M, K = a.shape
    N = w.shape[0]
    C = np.empty((M, N), np.float32)
    lib().ora_gemm_fp8_rowcol(_p(a), _p(sa), _p(w), _p(sw), _p(C), M, N, K)
    return C


def ring_allreduce(bufs) -> np.ndarray:
    b = _c(bufs, np.float32).copy()
    R, count = b.shape
    lib().ora_ring_allreduce(_p(b), count, R)
    return b


def allgather(chunks) -> np.ndarray:
    c = _c(chunks, np.float32)
    R, n = c.shape
    out = np.empty(R * n, np.float32)
    lib().ora_allgather(_p(c), _p(out), n, R)
    return out


def num_threads() -> int:
    return lib().ora_num_threads()


def set_num_threads(n: int) -> None:
    lib().ora_set_num_threads(n)


# --------------------------------------------------------------------------
# bf16 / fp16 helpers and seeded synthetic inputs
# --------------------------------------------------------------------------

def f32_to_bf16_bits(x) -> np.ndarray:
    """Round-to-nearest-even fp32 -> bf16 bit patterns (uint16)."""
    b = _c(x, np.float32).view(np.uint32)
    nan = (b & 0x7F800000) == 0x7F800000
    nan &= (b & 0x007FFFFF) != 0
    r = ((b + 0x7FFF + ((b >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = ((b[nan] >> 16) | 0x40).astype(np.uint16)
    return r


def bf16_bits_to_f32(b) -> np.ndarray:
    return (np.asarray(b, np.uint16).astype(np.uint32) << 16).view(np.float32)


def make_w4_gptq(N: int, K: int, gs: int = 128, seed: int = 0):
    """Configs 0/2/3: uniform nibbles 0..15 (two per byte, low = even k),
    fp16 per-group scales U[0.002, 0.02] (fp16-rounded)."""
    rng = np.random.default_rng(seed)
    packed = rng.integers(0, 256, size=(N, K // 2), dtype=np.uint8)
    scales = rng.uniform(0.002, 0.02, size=(N, K // gs)).astype(np.float16)
    return packed, scales


def make_activations_bf16(M: int, K: int, seed: int = 1) -> np.ndarray:
    """bf16 N(0,1) activations as bit patterns."""
    rng = np.random.default_rng(seed)
    return f32_to_bf16_bits(rng.standard_normal((M, K), dtype=np.float32))


def make_outlier_activations(T: int, D: int, seed: int = 0, frac: float = 0.01,
                             factor: float = 20.0) -> np.ndarray:
    """Config 1: N(0,1) [T, D] with a seeded 1% of channels scaled x20."""
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((T, D), dtype=np.float32)
    n_out = max(1, int(round(frac * D)))
    ch = rng.permutation(D)[:n_out]
    x[:, ch] *= np.float32(factor)
    return x


def make_weight_f32(N: int, K: int, seed: int = 2, std: float = 0.02) -> np.ndarray:
    rng = np.random.default_rng(seed)
    return (rng.standard_normal((N, K), dtype=np.float32) * np.float32(std)).astype(np.float32)

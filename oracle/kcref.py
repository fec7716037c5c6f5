"""Loader for oracle/_ref/libkcref.so: the reference's own hot-path CUDA kernels
(quant_int4.cu, fp8_quant.cu, tensor_parallel.cu, tensor_parallel_nccl.cu),
compiled from the reference sources by oracle/build_ref.sh.

TEST INFRASTRUCTURE ONLY: the GPU parity tests and tests/golden/make_golden_ref.py
run it beside the product library on identical inputs, as a second oracle.
It is loaded RTLD_LOCAL so its launch_* symbols never shadow libkernels.so's.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "_ref" / "libkcref.so"
_lib = None

vp, ci, cb = ctypes.c_void_p, ctypes.c_int, ctypes.c_bool


def available() -> bool:
    return LIB_PATH.exists()


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        try:
            import torch  # noqa: F401  (torch's NCCL must be resolved first)
        except ImportError:  # pragma: no cover
            pass
        l = ctypes.CDLL(str(LIB_PATH), mode=ctypes.RTLD_LOCAL)
        for name, args in {
            "launch_dequantize_int4": [vp, vp, vp, vp, ci, ci, ci, vp],
            "launch_gemv_int4": [vp, vp, vp, vp, vp, ci, ci, ci, vp],
            "launch_quantize_fp8": [vp, vp, vp, ci, ci, cb, vp],
            "launch_dequantize_fp8": [vp, vp, vp, ci, ci, cb, vp],
            "launch_smoothquant_scale": [vp, vp, vp, ci, ci, vp],
            "launch_col_parallel_linear": [vp, vp, vp, ci, ci, ci, vp],
            "launch_row_parallel_linear": [vp, vp, vp, ci, ci, ci, vp],
            "launch_ring_allreduce": [vp, ci, ci, vp],
            "launch_allgather": [vp, vp, ci, ci, vp],
        }.items():
            fn = getattr(l, name)
            fn.restype, fn.argtypes = None, args
        _lib = l
    return _lib


def _ptr(t) -> ctypes.c_void_p:
    return ctypes.c_void_p(t.data_ptr())


def _stream():
    import torch
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def dequantize_int4(packed, scales, zeros, rows, cols, gs):
    import torch
    out = torch.zeros(rows, cols, dtype=torch.float32, device=packed.device)
    lib().launch_dequantize_int4(_ptr(packed), _ptr(scales), _ptr(zeros), _ptr(out), rows, cols,
                                 gs, _stream())
    return out


def gemv_int4(packed, scales, zeros, x, rows, cols, gs):
    import torch
    y = torch.zeros(rows, dtype=torch.float32, device=packed.device)
    lib().launch_gemv_int4(_ptr(packed), _ptr(scales), _ptr(zeros), _ptr(x), _ptr(y), rows, cols,
                           gs, _stream())
    return y


def quantize_fp8(x, per_token: bool, scale=None):
    """Reference launch_quantize_fp8.  Per-tensor mode needs `scale` (a float);
    the reference reads it from d_scales[0]."""
    import torch
    rows, cols = x.shape
    q = torch.zeros(rows, cols, dtype=torch.int8, device=x.device)
    s = torch.zeros(rows if per_token else 1, dtype=torch.float32, device=x.device)
    if not per_token:
        s.fill_(float(scale))
    lib().launch_quantize_fp8(_ptr(x), _ptr(q), _ptr(s), rows, cols, per_token, _stream())
    return q, s


def dequantize_fp8(q, scales, rows, cols, per_token: bool):
    import torch
    out = torch.zeros(rows, cols, dtype=torch.float32, device=q.device)
    lib().launch_dequantize_fp8(_ptr(q), _ptr(scales), _ptr(out), rows, cols, per_token,
                                _stream())
    return out


def smoothquant_scale(x, s):
    import torch
    rows, cols = x.shape
    out = torch.zeros_like(x)
    lib().launch_smoothquant_scale(_ptr(x), _ptr(s), _ptr(out), rows, cols, _stream())
    return out


def sgemm_nt(A, B):
    import torch
    M, K = A.shape
    N = B.shape[0]
    C = torch.zeros(M, N, dtype=torch.float32, device=A.device)
    lib().launch_col_parallel_linear(_ptr(A), _ptr(B), _ptr(C), M, N, K, _stream())
    torch.cuda.synchronize()
    return C


def ring_allreduce(bufs):
    """bufs: list of CUDA float tensors (updated in place)."""
    arr = (ctypes.c_void_p * len(bufs))(*[b.data_ptr() for b in bufs])
    lib().launch_ring_allreduce(arr, bufs[0].numel(), len(bufs), _stream())


def allgather(chunks, out):
    arr = (ctypes.c_void_p * len(chunks))(*[c.data_ptr() for c in chunks])
    lib().launch_allgather(arr, _ptr(out), chunks[0].numel(), len(chunks), _stream())

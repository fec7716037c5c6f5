"""Shared helpers for the GPU parity tests."""
import ctypes

import numpy as np
import torch

import kc_lib


def stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def ptr(t: torch.Tensor):
    return ctypes.c_void_p(t.data_ptr())


def dev(a: np.ndarray, device="cuda:0") -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a)).to(device)


def host(t: torch.Tensor) -> np.ndarray:
    torch.cuda.synchronize()
    return t.cpu().numpy()


def normwise_err(y: np.ndarray, ref: np.ndarray) -> float:
    """max |y - ref| / max |ref| -- the GEMV/GEMM parity metric (elementwise
    relative error is unbounded where sums cancel)."""
    y = np.asarray(y, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.max(np.abs(y - ref)) / max(np.max(np.abs(ref)), 1e-30))


def misaligned(t: torch.Tensor, offset_bytes: int = 4) -> torch.Tensor:
    """A copy of t whose data pointer is `offset_bytes` past a 16-byte boundary
    (drives the scalar, any-alignment kernels)."""
    flat = t.contiguous().view(torch.uint8).reshape(-1)
    buf = torch.empty(flat.numel() + 64, dtype=torch.uint8, device=t.device)
    base = (-buf.data_ptr()) % 16
    v = buf[base + offset_bytes: base + offset_bytes + flat.numel()]
    v.copy_(flat)
    return v.view(t.dtype).reshape(t.shape)


def last_error():
    l = kc_lib.lib()
    return l.kc_get_last_error(), (l.kc_get_last_error_string() or b"").decode()

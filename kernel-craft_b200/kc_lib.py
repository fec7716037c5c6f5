"""ctypes binding of libkernels.so (the sm_100a quantized-linear library).

The library is the product: there is no Python or CPU fallback.  ``lib()``
raises if libkernels.so cannot be found or loaded, and ``check()`` turns a
non-zero kc_* status into a ``KcError`` carrying the library's message.

Search order for the library: ``$KERNEL_CRAFT_LIB``, then the in-tree build
``kernel-craft_b200/lib/libkernels.so`` (``python kernel-craft_b200/build.py``).
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path
from typing import Optional

HERE = Path(__file__).resolve().parent
DEFAULT_LIB = HERE / "lib" / "libkernels.so"

vp = ctypes.c_void_p
ci = ctypes.c_int
cl = ctypes.c_long
cb = ctypes.c_bool

KC_OK = 0
KC_ERR_INVALID_ARG = 1
KC_ERR_ALIGNMENT = 2
KC_ERR_CUDA = 3
KC_ERR_NCCL = 4
KC_ERR_UNSUPPORTED = 5
KC_ERR_TIMEOUT = 6
KC_W4A16_MAX_PROBLEMS = 8
KC_MAX_RANKS = 8
KC_ACT_NONE = 0
KC_ACT_GELU_QUICK = 1


class KcError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"kernel-craft status {status}: {message}")
        self.status = status


class W4A16Problem(ctypes.Structure):
    """Mirror of ``kc_w4a16_problem`` (include/kernel_craft.h)."""
    _fields_ = [("packed", vp), ("scales_f16", vp), ("x_bf16", vp), ("y", vp),
                ("N", ci), ("K", ci)]


# (name, restype, argtypes) for every exported entry point.
_PROTOS = [
    ("kc_get_last_error", ci, []),
    ("kc_get_last_error_string", ctypes.c_char_p, []),
    ("kc_version", ctypes.c_char_p, []),
    ("kc_get_device_status", ci, []),
    ("kc_selftest_bounded_wait", ci, [ctypes.c_uint64, vp, vp]),
    ("kc_selftest_stream_read", ci, [vp, ctypes.c_size_t, ctypes.c_uint32, vp, vp]),
    # reference ABI
    ("launch_dequantize_int4", None, [vp, vp, vp, vp, ci, ci, ci, vp]),
    ("launch_gemv_int4", None, [vp, vp, vp, vp, vp, ci, ci, ci, vp]),
    ("launch_quantize_fp8", None, [vp, vp, vp, ci, ci, cb, vp]),
    ("launch_dequantize_fp8", None, [vp, vp, vp, ci, ci, cb, vp]),
    ("launch_smoothquant_scale", None, [vp, vp, vp, ci, ci, vp]),
    ("launch_col_parallel_linear", None, [vp, vp, vp, ci, ci, ci, vp]),
    ("launch_row_parallel_linear", None, [vp, vp, vp, ci, ci, ci, vp]),
    ("launch_ring_allreduce", None, [vp, ci, ci, vp]),
    ("launch_allgather", None, [vp, vp, ci, ci, vp]),
    ("nccl_comm_init_all", None, [vp, ci, vp]),
    ("nccl_comm_destroy", None, [vp]),
    ("nccl_group_start", None, []),
    ("nccl_group_end", None, []),
    ("launch_ring_allreduce_nccl", None, [vp, vp, ci, vp]),
    ("launch_allgather_nccl", None, [vp, vp, vp, ci, vp]),
    ("nccl_comm_count", ci, [vp]),
    ("nccl_comm_user_rank", ci, [vp]),
    ("launch_flash_attention", None, [vp, vp, vp, vp, ci, ci, ci, ci, ci, cb, vp]),
    ("launch_paged_attention", None, [vp, vp, vp, vp, vp, vp, ci, ci, ci, ci, ci, ci, vp]),
    ("launch_verify_draft_tokens", None, [vp, vp, vp, vp, vp, vp, vp, ci, ci, vp]),
    ("launch_compute_prefix_length", None, [vp, vp, ci, vp]),
    ("launch_selective_scan", None, [vp, vp, vp, vp, vp, vp, ci, ci, ci, ci, vp]),
    ("launch_depthwise_conv1d", None, [vp, vp, vp, vp, ci, ci, ci, ci, vp]),
    ("launch_rmsnorm", None, [vp, vp, vp, ci, ci, ctypes.c_float, vp]),
    # kc_* API
    ("kc_dequantize_int4_f32", ci, [vp, vp, vp, vp, ci, ci, ci, vp]),
    ("kc_gemv_int4_f32", ci, [vp, vp, vp, vp, vp, ci, ci, ci, vp]),
    ("kc_dequantize_w4_bf16", ci, [vp, vp, vp, ci, ci, ci, vp]),
    ("kc_dequantize_w4_bf16_zp", ci, [vp, vp, vp, vp, ci, ci, ci, vp]),
    ("kc_gemv_w4a16", ci, [vp, vp, vp, vp, ci, ci, ci, ci, vp]),
    ("kc_gemv_w4a16_grouped", ci, [ctypes.POINTER(W4A16Problem), ci, ci, ci, vp]),
    ("kc_gemv_w4a16_zp", ci, [vp, vp, vp, vp, vp, ci, ci, ci, ci, vp]),
    ("kc_gemv_w4a16_grouped_zp", ci, [ctypes.POINTER(W4A16Problem), ctypes.POINTER(vp), ci, ci, ci, vp]),
    ("kc_w4a16_tile_weights", ci, [vp, vp, ci, ci, vp]),
    ("kc_gemv_w4a16_grouped_tiled", ci, [ctypes.POINTER(W4A16Problem), ctypes.POINTER(vp), ctypes.POINTER(vp), ci, ci, ci, vp]),
    ("kc_quantize_fp8_per_token", ci, [vp, vp, vp, ci, ci, vp]),
    ("kc_quantize_fp8_per_channel", ci, [vp, vp, vp, ci, ci, vp]),
    ("kc_quantize_fp8_per_tensor", ci, [vp, vp, vp, cl, vp]),
    ("kc_quantize_fp8_per_tensor_dynamic", ci, [vp, vp, vp, cl, vp, ctypes.c_size_t, vp]),
    ("kc_quantize_fp8_per_tensor_dynamic_noalloc", ci, [vp, vp, vp, cl, vp]),
    ("kc_smoothquant_quantize_fp8", ci, [vp, vp, vp, vp, ci, ci, vp]),
    ("kc_dequantize_fp8", ci, [vp, vp, vp, ci, ci, cb, vp]),
    ("kc_smoothquant_scale", ci, [vp, vp, vp, ci, ci, vp]),
    ("kc_sgemm_nt", ci, [vp, vp, vp, ci, ci, ci, vp]),
    ("kc_gemm_fp8", ci, [vp, vp, vp, vp, vp, ci, ci, ci, ci, ci, vp]),
    ("kc_gemm_fp8_ctas", ci, [vp, vp, vp, vp, vp, ci, ci, ci, ci, ci, ci, vp]),
    ("kc_gemm_w4a16", ci, [vp, vp, vp, vp, ci, ci, ci, ci, ci, ci, vp]),
    ("kc_gemm_w4a16_act", ci, [vp, vp, vp, vp, ci, ci, ci, ci, ci, ci, ci, vp]),
    ("kc_gemm_w4a16_zp", ci, [vp, vp, vp, vp, vp, ci, ci, ci, ci, ci, ci, ci, vp]),
    ("kc_gemm_w4a16_allgather", ci, [vp, vp, vp, ctypes.POINTER(vp), ci, ci, ci, ci, ci, ci, vp]),
    ("kc_gemm_w4a16_allgather_mc", ci, [vp, vp, vp, vp, ci, ci, ci, ci, ci, ci, vp]),
    ("kc_allreduce_bf16_peer", ci, [ctypes.POINTER(vp), ctypes.POINTER(vp), ci, ci, cl, vp]),
    ("kc_allreduce_bf16_nvls", ci, [vp, ci, ci, cl, ci, vp]),
    ("kc_gemm_fp8_allreduce_mc", ci, [vp, vp, vp, vp, vp, vp, ctypes.POINTER(vp), ci, ci, ci, ci, ci, ci, ctypes.c_uint64, vp]),
    ("kc_gemm_fp8_allreduce", ci, [vp, vp, vp, vp, ctypes.POINTER(vp), ctypes.POINTER(vp), ctypes.POINTER(vp), ci, ci, ci, ci, ci, ci, ctypes.c_uint64, vp]),
    ("kc_peer_barrier", ci, [ctypes.POINTER(vp), ci, ci, ci, ctypes.c_uint64, vp, vp]),
    ("kc_ipc_handle_bytes", ci, []),
    ("kc_ipc_alloc", ci, [ctypes.POINTER(vp), ctypes.c_size_t]),
    ("kc_ipc_free", ci, [vp]),
    ("kc_ipc_get_handle", ci, [vp, vp]),
    ("kc_ipc_open", ci, [vp, ctypes.POINTER(vp)]),
    ("kc_ipc_close", ci, [vp]),
    ("kc_nccl_unique_id_bytes", ci, []),
    ("kc_nccl_get_unique_id", ci, [vp]),
    ("kc_nccl_comm_init_rank", ci, [vp, ci, vp, ci]),
    ("kc_nccl_comm_destroy", ci, [vp]),
    ("kc_nccl_comm_abort", ci, [vp]),
    ("kc_nccl_comm_check", ci, [vp]),
    ("kc_allgather_bf16", ci, [vp, vp, vp, cl, vp]),
    ("kc_allreduce_bf16", ci, [vp, vp, vp, cl, vp]),
    ("kc_allreduce_f32", ci, [vp, vp, vp, cl, vp]),
]

_LIB: Optional[ctypes.CDLL] = None


def lib_path() -> Path:
    env = os.environ.get("KERNEL_CRAFT_LIB")
    p = Path(env) if env else DEFAULT_LIB
    if not p.exists():
        raise FileNotFoundError(
            f"libkernels.so not found at {p}; build it with `python kernel-craft_b200/build.py`")
    return p


def lib() -> ctypes.CDLL:
    """The loaded library with prototypes set (loaded once per process).

    torch is imported first when it is installed: libkernels.so links
    ``libnccl.so.2`` by soname, and torch's bundled NCCL must be the copy that
    is resolved first, or torch's own NCCL symbols go missing.
    """
    global _LIB
    if _LIB is None:
        try:
            import torch  # noqa: F401
        except ImportError:  # pragma: no cover
            pass
        handle = ctypes.CDLL(str(lib_path()), mode=ctypes.RTLD_GLOBAL)
        for name, res, args in _PROTOS:
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _LIB = handle
    return _LIB


def exported_names() -> list[str]:
    return [n for n, _, _ in _PROTOS]


def check(status: int) -> None:
    """Raise KcError for a non-zero kc_* status."""
    if status != KC_OK:
        l = lib()
        msg = (l.kc_get_last_error_string() or b"").decode(errors="replace")
        l.kc_get_last_error()
        raise KcError(status, msg)


def check_last() -> None:
    """Raise KcError if a void (reference-ABI) launcher recorded an error."""
    l = lib()
    st = l.kc_get_last_error()
    if st != KC_OK:
        raise KcError(st, (l.kc_get_last_error_string() or b"").decode(errors="replace"))

"""
kernel_craft_torch_ops -- torch-facing operators of the B200 quantized-linear library.

Mirrors the quantized-linear part of kernel-craft's ctypes bridge
(src/python/kernel_craft_torch_ops.py:265-381): same function names, argument
meaning, return shapes and dtypes, and the same ``torch.ops.kernel_craft.*``
registration (:428-471).  Each call hands ``data_ptr()``s and torch's current
CUDA stream to the C ABI of libkernels.so (include/kernel_craft.h); there is no
CPU path: the library must be built and the tensors must live on a CUDA device.

Differences from the reference bridge, all on inputs the reference mishandles:
  * ``fp8_quantize(x, per_token=False)`` computes the per-tensor scale
    (amax/448) on the device, as the reference's pybind path does on the host
    (src/python/pybind_transformer.cpp:305-311); the reference ctypes bridge
    passes a zero scale (kernel_craft_torch_ops.py:347), which saturates
    every code.
  * invalid shapes raise ``KcError`` instead of launching.
  * the reference's launchers synchronize the stream; these ops call the
    non-synchronizing ``kc_*`` twins (results are ordered on the stream).

New operators (no reference counterpart): ``w4a16_dequantize``,
``w4a16_gemv``, ``w4a16_gemv_grouped``, ``w4a16_gemm``, ``fp8_gemm``,
``fp8_quantize_per_channel``, ``smoothquant_fp8_quantize``,
``smoothquant_scale``.
"""
from __future__ import annotations

import ctypes
from typing import List, Sequence, Tuple

import torch

try:  # the reference's OTEL span helper, when it is on sys.path
    from kernel_craft_otel import kernel_span  # type: ignore
except ImportError:  # pragma: no cover
    from contextlib import nullcontext as _nullcontext

    def kernel_span(*_a, **_k):
        return _nullcontext()

import kc_lib
from kc_lib import check, lib


def _stream() -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _ptr(t: torch.Tensor) -> ctypes.c_void_p:
    return ctypes.c_void_p(t.data_ptr())


def _require_cuda(*ts: torch.Tensor) -> None:
    for t in ts:
        if not t.is_cuda:
            raise ValueError("kernel-craft ops take CUDA tensors only (no CPU path)")


def _expect(t: torch.Tensor, name: str, numel=None, shape=None, dtypes=None) -> None:
    """Raise ValueError unless t has the element count / shape / dtype the
    kernel will read: the library receives raw pointers and sizes, so a short
    or mistyped tensor would be read out of bounds instead of failing."""
    if shape is not None and tuple(t.shape) != tuple(shape):
        raise ValueError(f"{name}: shape {tuple(t.shape)}, expected {tuple(shape)}")
    if numel is not None and t.numel() < numel:
        raise ValueError(f"{name}: {t.numel()} elements, the kernel reads {numel}")
    if dtypes is not None and t.dtype not in dtypes:
        raise ValueError(f"{name}: dtype {t.dtype}, expected one of {[str(d) for d in dtypes]}")


_F32 = (torch.float32,)
_F16 = (torch.float16, torch.int16)      # fp16 bits may arrive as int16
_BF16 = (torch.bfloat16, torch.int16)
_U8 = (torch.uint8, torch.int8)
_I8 = (torch.int8, torch.uint8)


def _check_int4_ref(packed, scales, zeros, rows, cols, group_size):
    if rows < 0 or cols < 0 or group_size <= 0:
        raise ValueError("rows, cols must be >= 0 and group_size > 0")
    g = -(-cols // group_size)
    _expect(packed, "packed", numel=rows * ((cols + 1) // 2), dtypes=_U8)
    _expect(scales, "scales", numel=rows * g, dtypes=_F32)
    # the reference kernel's zero-point row stride is floor(G/2) bytes
    # (quant_int4.cu:93); an odd group count reads one byte past the last row
    _expect(zeros, "zeros", numel=(rows * (g // 2) + g % 2) if rows else 0, dtypes=_U8)


def _check_w4(packed, scales, group_size, name=""):
    if packed.dim() != 2 or group_size <= 0 or (packed.shape[1] * 2) % group_size:
        raise ValueError(f"{name}packed must be [N, K/2] with group_size dividing K")
    n, k = packed.shape[0], packed.shape[1] * 2
    _expect(packed, name + "packed", dtypes=_U8)
    _expect(scales, name + "scales_f16", shape=(n, k // group_size), dtypes=_F16)
    return n, k


# ---------------------------------------------------------------------------
# Reference operators (kernel_craft_torch_ops.py:265-381)
# ---------------------------------------------------------------------------

def int4_dequantize(packed, scales, zeros, rows: int, cols: int, group_size: int = 128):
    """INT4 -> fp32 [rows, cols]; reference semantics (sign-extended nibbles,
    unsigned zero points)."""
    packed, scales, zeros = packed.contiguous(), scales.contiguous(), zeros.contiguous()
    _check_int4_ref(packed, scales, zeros, rows, cols, group_size)
    _require_cuda(packed, scales, zeros)
    out = torch.empty(rows, cols, dtype=torch.float32, device=packed.device)
    check(lib().kc_dequantize_int4_f32(_ptr(packed), _ptr(scales), _ptr(zeros), _ptr(out),
                                       rows, cols, group_size, _stream()))
    return out


def int4_gemv(packed, scales, zeros, x, rows: int, cols: int, group_size: int = 128):
    """y[rows] = W_int4 . x in fp32 (on-the-fly dequant)."""
    packed, scales, zeros, x = (t.contiguous() for t in (packed, scales, zeros, x))
    _check_int4_ref(packed, scales, zeros, rows, cols, group_size)
    _expect(x, "x", numel=cols, dtypes=_F32)
    _require_cuda(packed, scales, zeros, x)
    y = torch.empty(rows, dtype=torch.float32, device=packed.device)
    with kernel_span("int4_gemv", rows=rows, cols=cols, group_size=group_size):
        check(lib().kc_gemv_int4_f32(_ptr(packed), _ptr(scales), _ptr(zeros), _ptr(x), _ptr(y),
                                     rows, cols, group_size, _stream()))
    return y


def fp8_quantize(x, per_token: bool = True) -> Tuple[torch.Tensor, torch.Tensor]:
    """fp32 [rows, cols] -> (int8 E4M3 codes [rows, cols], fp32 scales [rows] or [1])."""
    x = x.contiguous()
    if x.dim() != 2:
        raise ValueError("x must be 2-D [rows, cols]")
    _expect(x, "x", dtypes=_F32)
    _require_cuda(x)
    rows, cols = x.shape
    q = torch.empty(rows, cols, dtype=torch.int8, device=x.device)
    with kernel_span("fp8_quantize", rows=rows, cols=cols, per_token=per_token):
        if per_token:
            scales = torch.empty(rows, dtype=torch.float32, device=x.device)
            check(lib().kc_quantize_fp8_per_token(_ptr(x), _ptr(q), _ptr(scales), rows, cols,
                                                  _stream()))
        else:
            scales = torch.empty(1, dtype=torch.float32, device=x.device)
            ws = torch.empty(1, dtype=torch.int32, device=x.device)
            check(lib().kc_quantize_fp8_per_tensor_dynamic(_ptr(x), _ptr(q), _ptr(scales),
                                                           rows * cols, _ptr(ws), 4, _stream()))
    return q, scales


def fp8_dequantize(q, scales, rows: int, cols: int, per_token: bool = True):
    """int8 E4M3 codes -> fp32 [rows, cols]."""
    q, scales = q.contiguous(), scales.contiguous()
    _expect(q, "q", numel=rows * cols, dtypes=_I8)
    _expect(scales, "scales", numel=rows if per_token else 1, dtypes=_F32)
    _require_cuda(q, scales)
    out = torch.empty(rows, cols, dtype=torch.float32, device=q.device)
    check(lib().kc_dequantize_fp8(_ptr(q), _ptr(scales), _ptr(out), rows, cols, per_token,
                                  _stream()))
    return out


# ---------------------------------------------------------------------------
# New operators
# ---------------------------------------------------------------------------

def smoothquant_scale(x, smooth):
    """x[r, c] / smooth[c] (fp8_quant.cu:174-184 semantics)."""
    x, smooth = x.contiguous(), smooth.contiguous()
    if x.dim() != 2:
        raise ValueError("x must be 2-D [rows, cols]")
    _expect(x, "x", dtypes=_F32)
    _expect(smooth, "smooth", numel=x.shape[1], dtypes=_F32)
    _require_cuda(x, smooth)
    rows, cols = x.shape
    out = torch.empty_like(x)
    check(lib().kc_smoothquant_scale(_ptr(x), _ptr(smooth), _ptr(out), rows, cols, _stream()))
    return out


def smoothquant_fp8_quantize(x, smooth) -> Tuple[torch.Tensor, torch.Tensor]:
    """Fused SmoothQuant divide + per-token FP8 quantization."""
    x, smooth = x.contiguous(), smooth.contiguous()
    if x.dim() != 2:
        raise ValueError("x must be 2-D [rows, cols]")
    _expect(x, "x", dtypes=_F32)
    _expect(smooth, "smooth", numel=x.shape[1], dtypes=_F32)
    _require_cuda(x, smooth)
    rows, cols = x.shape
    q = torch.empty(rows, cols, dtype=torch.int8, device=x.device)
    scales = torch.empty(rows, dtype=torch.float32, device=x.device)
    check(lib().kc_smoothquant_quantize_fp8(_ptr(x), _ptr(smooth), _ptr(q), _ptr(scales), rows,
                                            cols, _stream()))
    return q, scales


def fp8_quantize_per_channel(w) -> Tuple[torch.Tensor, torch.Tensor]:
    """Per-output-channel weight quantization of W[N, K]: one scale per row."""
    w = w.contiguous()
    if w.dim() != 2:
        raise ValueError("w must be 2-D [N, K]")
    _expect(w, "w", dtypes=_F32)
    _require_cuda(w)
    n, k = w.shape
    q = torch.empty(n, k, dtype=torch.int8, device=w.device)
    scales = torch.empty(n, dtype=torch.float32, device=w.device)
    check(lib().kc_quantize_fp8_per_channel(_ptr(w), _ptr(q), _ptr(scales), n, k, _stream()))
    return q, scales


def _check_zeros(zeros, n, k, group_size, name=""):
    """Per-group zero points: u8 [N, K/gs] (one 0..15 value per byte), or None."""
    if zeros is None:
        return None
    zeros = zeros.contiguous()
    _expect(zeros, f"{name}zeros", shape=(n, k // group_size), dtypes=(torch.uint8,))
    return zeros


def w4a16_dequantize(packed, scales_f16, group_size: int = 128, zeros=None):
    """W4 -> bf16 [N, K]: bf16((u - z) * s), z = 8 (GPTQ symmetric) unless
    per-group zero points zeros u8 [N, K/gs] are given (AWQ, asymmetric GPTQ)."""
    packed, scales_f16 = packed.contiguous(), scales_f16.contiguous()
    n, k = _check_w4(packed, scales_f16, group_size)
    zeros = _check_zeros(zeros, n, k, group_size)
    _require_cuda(packed, scales_f16, *([zeros] if zeros is not None else []))
    out = torch.empty(n, k, dtype=torch.bfloat16, device=packed.device)
    if zeros is None:
        check(lib().kc_dequantize_w4_bf16(_ptr(packed), _ptr(scales_f16), _ptr(out), n, k,
                                          group_size, _stream()))
    else:
        check(lib().kc_dequantize_w4_bf16_zp(_ptr(packed), _ptr(scales_f16), _ptr(zeros), _ptr(out),
                                             n, k, group_size, _stream()))
    return out


def w4a16_gemv(packed, scales_f16, x, group_size: int = 128, zeros=None):
    """y[M, N] (fp32) = x[M, K] (bf16, M <= 16) . W^T with W the W4 [N, K]
    (zero point 8, or per-group zero points zeros u8 [N, K/gs])."""
    packed, scales_f16, x = packed.contiguous(), scales_f16.contiguous(), x.contiguous()
    if x.dim() == 1:
        x = x.unsqueeze(0)
    n, k = _check_w4(packed, scales_f16, group_size)
    zeros = _check_zeros(zeros, n, k, group_size)
    _expect(x, "x", shape=(x.shape[0], k), dtypes=_BF16)
    _require_cuda(packed, scales_f16, x, *([zeros] if zeros is not None else []))
    m = x.shape[0]
    y = torch.empty(m, n, dtype=torch.float32, device=packed.device)
    with kernel_span("w4a16_gemv", rows=n, cols=k, batch=m, group_size=group_size):
        if zeros is None:
            check(lib().kc_gemv_w4a16(_ptr(packed), _ptr(scales_f16), _ptr(x), _ptr(y), m, n, k,
                                      group_size, _stream()))
        else:
            check(lib().kc_gemv_w4a16_zp(_ptr(packed), _ptr(scales_f16), _ptr(zeros), _ptr(x),
                                         _ptr(y), m, n, k, group_size, _stream()))
    return y


def w4a16_gemv_grouped(problems: Sequence[Tuple[torch.Tensor, torch.Tensor, torch.Tensor]],
                       group_size: int = 128) -> List[torch.Tensor]:
    """One launch over several (packed, scales_f16, x) problems sharing M."""
    if not 1 <= len(problems) <= kc_lib.KC_W4A16_MAX_PROBLEMS:
        raise ValueError("1..8 problems per grouped launch")
    # every problem is checked before any is handed to the library
    checked = []
    m = None
    for i, (packed, scales, x) in enumerate(problems):
        packed, scales, x = packed.contiguous(), scales.contiguous(), x.contiguous()
        if x.dim() == 1:
            x = x.unsqueeze(0)
        n, k = _check_w4(packed, scales, group_size, name=f"problem {i}: ")
        _expect(x, f"problem {i}: x", shape=(x.shape[0], k), dtypes=_BF16)
        m = x.shape[0] if m is None else m
        if x.shape[0] != m:
            raise ValueError("all problems of a grouped launch share M")
        checked.append((packed, scales, x, n, k))
    arr = (kc_lib.W4A16Problem * len(problems))()
    outs = []
    for i, (packed, scales, x, n, k) in enumerate(checked):
        _require_cuda(packed, scales, x)
        y = torch.empty(m, n, dtype=torch.float32, device=packed.device)
        arr[i] = kc_lib.W4A16Problem(packed.data_ptr(), scales.data_ptr(), x.data_ptr(),
                                     y.data_ptr(), n, k)
        outs.append(y)
    check(lib().kc_gemv_w4a16_grouped(arr, len(problems), m, group_size, _stream()))
    return outs


_ACTIVATIONS = {"none": kc_lib.KC_ACT_NONE, "gelu_quick": kc_lib.KC_ACT_GELU_QUICK}


def w4a16_gemm(x, packed, scales_f16, group_size: int = 128, out_dtype=torch.bfloat16,
               activation: str = "none", zeros=None):
    """C[M, N] = act(x[M, K] (bf16) . W^T) on the tcgen05 tensor cores, W the
    GPTQ W4 [N, K] (packed u8 [N, K/2], fp16 scales [N, K/gs]); fp32
    accumulation, bf16 (default) or fp32 output.  activation "gelu_quick"
    applies x * sigmoid(1.702 x), the reference MLP block's GELU
    (examples/python/transformer/tensor_parallel.py:162), in the epilogue.
    zeros: per-group zero points u8 [N, K/gs] (AWQ, asymmetric GPTQ)."""
    if activation not in _ACTIVATIONS:
        raise ValueError(f"activation must be one of {sorted(_ACTIVATIONS)}")
    x, packed, scales_f16 = x.contiguous(), packed.contiguous(), scales_f16.contiguous()
    n, k = _check_w4(packed, scales_f16, group_size)
    zeros = _check_zeros(zeros, n, k, group_size)
    if x.dim() != 2 or x.shape[1] != k:
        raise ValueError(f"x must be [M, {k}] (the packed weights' K), got {tuple(x.shape)}")
    _expect(x, "x", dtypes=_BF16)
    if out_dtype not in (torch.bfloat16, torch.float32):
        raise ValueError("out_dtype must be torch.bfloat16 or torch.float32")
    _require_cuda(x, packed, scales_f16)
    m = x.shape[0]
    out = torch.empty(m, n, dtype=out_dtype, device=x.device)
    with kernel_span("w4a16_gemm", rows=n, cols=k, batch=m, group_size=group_size):
        if zeros is None:
            check(lib().kc_gemm_w4a16_act(_ptr(x), _ptr(packed), _ptr(scales_f16), _ptr(out),
                                          1 if out_dtype == torch.float32 else 0, m, n, k,
                                          group_size, n, _ACTIVATIONS[activation], _stream()))
        else:
            _require_cuda(zeros)
            check(lib().kc_gemm_w4a16_zp(_ptr(x), _ptr(packed), _ptr(scales_f16), _ptr(zeros),
                                         _ptr(out), 1 if out_dtype == torch.float32 else 0, m, n,
                                         k, group_size, n, _ACTIVATIONS[activation], _stream()))
    return out


def fp8_gemm(a_codes, sa, w_codes, sw, out_dtype=torch.bfloat16):
    """out[M, N] = (e4m3(a) . e4m3(w)^T) * sa[m] * sw[n] on the tcgen05 tensor
    cores: a_codes [M, K] and w_codes [N, K] the int8 E4M3 bit patterns of
    fp8_quantize(per_token=True) / fp8_quantize_per_channel, fp32 accumulation,
    bf16 (default) or fp32 output."""
    a_codes, w_codes = a_codes.contiguous(), w_codes.contiguous()
    sa, sw = sa.contiguous(), sw.contiguous()
    if a_codes.dim() != 2 or w_codes.dim() != 2 or a_codes.shape[1] != w_codes.shape[1]:
        raise ValueError("a_codes [M, K] and w_codes [N, K] must share K")
    m, k = a_codes.shape
    n = w_codes.shape[0]
    _expect(a_codes, "a_codes", dtypes=_I8)
    _expect(w_codes, "w_codes", dtypes=_I8)
    _expect(sa, "sa", shape=(m,), dtypes=_F32)
    _expect(sw, "sw", shape=(n,), dtypes=_F32)
    if out_dtype not in (torch.bfloat16, torch.float32):
        raise ValueError("out_dtype must be torch.bfloat16 or torch.float32")
    _require_cuda(a_codes, sa, w_codes, sw)
    out = torch.empty(m, n, dtype=out_dtype, device=a_codes.device)
    with kernel_span("fp8_gemm", rows=n, cols=k, batch=m):
        check(lib().kc_gemm_fp8(_ptr(a_codes), _ptr(sa), _ptr(w_codes), _ptr(sw), _ptr(out),
                                1 if out_dtype == torch.float32 else 0, m, n, k, n, _stream()))
    return out


# ---------------------------------------------------------------------------
# torch.library registration (kernel_craft_torch_ops.py:428-471)
# ---------------------------------------------------------------------------

def _register_torch_library() -> None:
    libdef = torch.library.Library("kernel_craft", "DEF")
    libdef.define("int4_dequantize(Tensor packed, Tensor scales, Tensor zeros, "
                  "int rows, int cols, int group_size) -> Tensor")
    libdef.define("int4_gemv(Tensor packed, Tensor scales, Tensor zeros, "
                  "Tensor x, int rows, int cols, int group_size) -> Tensor")
    libdef.define("fp8_quantize(Tensor x, bool per_token) -> (Tensor, Tensor)")
    libdef.define("fp8_dequantize(Tensor q, Tensor scales, int rows, int cols, bool per_token) "
                  "-> Tensor")
    libdef.define("w4a16_gemv(Tensor packed, Tensor scales_f16, Tensor x, int group_size) -> Tensor")
    libdef.define("w4a16_dequantize(Tensor packed, Tensor scales_f16, int group_size) -> Tensor")
    libdef.define("fp8_quantize_per_channel(Tensor w) -> (Tensor, Tensor)")
    libdef.define("smoothquant_fp8_quantize(Tensor x, Tensor smooth) -> (Tensor, Tensor)")
    libdef.define("w4a16_gemm(Tensor x, Tensor packed, Tensor scales_f16, int group_size) -> Tensor")
    libdef.define("fp8_gemm(Tensor a_codes, Tensor sa, Tensor w_codes, Tensor sw) -> Tensor")
    impl = torch.library.Library("kernel_craft", "IMPL")
    for name, fn in (("int4_dequantize", int4_dequantize), ("int4_gemv", int4_gemv),
                     ("fp8_quantize", fp8_quantize), ("fp8_dequantize", fp8_dequantize),
                     ("w4a16_gemv", w4a16_gemv), ("w4a16_dequantize", w4a16_dequantize),
                     ("fp8_quantize_per_channel", fp8_quantize_per_channel),
                     ("smoothquant_fp8_quantize", smoothquant_fp8_quantize),
                     ("w4a16_gemm", lambda x, p, s, gs: w4a16_gemm(x, p, s, gs)),
                     ("fp8_gemm", lambda a, sa, w, sw: fp8_gemm(a, sa, w, sw))):
        impl.impl(name, fn, "CUDA")
    globals()["_torch_lib_def"] = libdef
    globals()["_torch_lib_impl"] = impl


try:
    _register_torch_library()
    TORCH_OPS_REGISTERED = True
except Exception:  # pragma: no cover - e.g. the namespace is already taken
    TORCH_OPS_REGISTERED = False

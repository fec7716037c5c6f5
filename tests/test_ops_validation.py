"""The torch-op wrappers (kernel_craft_torch_ops) check every operand's size
and dtype on the host before the library sees a pointer, so a short or
mistyped tensor raises ValueError instead of being read out of bounds.
CPU tensors: the checks come before the CUDA-device check, which then rejects
correctly shaped CPU tensors (there is no CPU path)."""
import pytest
import torch

import kernel_craft_torch_ops as ops

u8, f16, f32, bf16, i8 = torch.uint8, torch.float16, torch.float32, torch.bfloat16, torch.int8


def z(*shape, dtype=f32):
    return torch.zeros(*shape, dtype=dtype)


def _raises(fn, match):
    with pytest.raises(ValueError, match=match):
        fn()


def test_w4a16_gemv_and_gemm():
    N, K, gs = 32, 256, 128
    p, s, x = z(N, K // 2, dtype=u8), z(N, K // gs, dtype=f16), z(2, K, dtype=bf16)
    _raises(lambda: ops.w4a16_gemv(p, s, x, gs), "CUDA")
    _raises(lambda: ops.w4a16_gemv(p, z(N, 3, dtype=f16), x, gs), "scales_f16")
    _raises(lambda: ops.w4a16_gemv(p, s.float(), x, gs), "scales_f16")
    _raises(lambda: ops.w4a16_gemv(p, s, z(2, K // 2, dtype=bf16), gs), "x")
    _raises(lambda: ops.w4a16_gemv(p, s, x.float(), gs), "x")
    _raises(lambda: ops.w4a16_gemv(p, s, x, 96), "group_size")
    _raises(lambda: ops.w4a16_gemm(x, p, s, gs), "CUDA")
    _raises(lambda: ops.w4a16_gemm(z(2, K + 64, dtype=bf16), p, s, gs), "x must be")
    _raises(lambda: ops.w4a16_gemm(x, p, s, gs, out_dtype=torch.float16), "out_dtype")
    _raises(lambda: ops.w4a16_dequantize(p, z(N - 1, K // gs, dtype=f16), gs), "scales_f16")
    _raises(lambda: ops.w4a16_gemv_grouped([(p, s, x), (p, z(N, 1, dtype=f16), x)], gs), "problem 1")


def test_fp8_ops():
    _raises(lambda: ops.fp8_quantize(z(4, 32)), "CUDA")
    _raises(lambda: ops.fp8_quantize(z(4, 32, dtype=torch.float64)), "x")
    _raises(lambda: ops.fp8_quantize(z(128)), "2-D")
    _raises(lambda: ops.fp8_dequantize(z(4, 31, dtype=i8), z(4), 4, 32), "q")
    _raises(lambda: ops.fp8_dequantize(z(4, 32, dtype=i8), z(3), 4, 32), "scales")
    _raises(lambda: ops.smoothquant_scale(z(4, 32), z(31)), "smooth")
    _raises(lambda: ops.smoothquant_fp8_quantize(z(4, 32), z(32, dtype=f16)), "smooth")
    _raises(lambda: ops.fp8_quantize_per_channel(z(8, 32, dtype=bf16)), "w")
    a, w = z(16, 64, dtype=i8), z(8, 64, dtype=i8)
    _raises(lambda: ops.fp8_gemm(a, z(16), w, z(8)), "CUDA")
    _raises(lambda: ops.fp8_gemm(a, z(16), z(8, 32, dtype=i8), z(8)), "share K")
    _raises(lambda: ops.fp8_gemm(a, z(15), w, z(8)), "sa")
    _raises(lambda: ops.fp8_gemm(a, z(16), w, z(8, dtype=f16)), "sw")


def test_reference_int4_ops():
    rows, cols, gs = 8, 384, 128                       # 3 groups: odd count
    p, s = z(rows, cols // 2, dtype=u8), z(rows, cols // gs)
    zeros_ok = z(rows * 1 + 1, dtype=u8)               # floor(3/2) per row + the last row's byte
    _raises(lambda: ops.int4_dequantize(p, s, zeros_ok, rows, cols, gs), "CUDA")
    _raises(lambda: ops.int4_dequantize(p, s, z(rows, dtype=u8), rows, cols, gs), "zeros")
    _raises(lambda: ops.int4_dequantize(p[:4], s, zeros_ok, rows, cols, gs), "packed")
    _raises(lambda: ops.int4_dequantize(p, s.half(), zeros_ok, rows, cols, gs), "scales")
    _raises(lambda: ops.int4_gemv(p, s, zeros_ok, z(cols - 1), rows, cols, gs), "x")
    _raises(lambda: ops.int4_gemv(p, s, zeros_ok, z(cols), rows, cols, 0), "group_size")

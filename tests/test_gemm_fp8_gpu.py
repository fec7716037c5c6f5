"""GPU parity: tcgen05 FP8 W8A8 GEMM (kc_gemm_fp8) vs the oracle.

Bars (written here): fp32 output normwise <= 1e-4 (e4m3 products are exact in
fp32, only the accumulation order differs); bf16 output normwise <= 1e-2 (the
task's bound for bf16 / FP8 outputs), also against the reference's own chain
dequantize_fp8 -> fp32 GEMM (fp8_quant.cu:145-160, tensor_parallel.cu:164-192).
"""
import numpy as np
import pytest
import torch

import kc_lib
import oracle as O
from kc_testutil import dev, host, normwise_err, ptr, stream

pytestmark = pytest.mark.gpu


def _quantized_operands(M, N, K, seed):
    x = O.make_outlier_activations(M, K, seed=seed)
    w = O.make_weight_f32(N, K, seed=seed + 1)
    qa, sa = O.quantize_fp8_per_token(x)
    qw, sw = O.quantize_fp8_per_token(w)
    return qa, sa, qw, sw


def _run(qa, sa, qw, sw, M, N, K, out_f32):
    da, dsa, dw, dsw = dev(qa.view(np.int8)), dev(sa), dev(qw.view(np.int8)), dev(sw)
    out = torch.full((M, N), float("nan"), dtype=torch.float32 if out_f32 else torch.bfloat16,
                     device="cuda:0")
    kc_lib.check(kc_lib.lib().kc_gemm_fp8(ptr(da), ptr(dsa), ptr(dw), ptr(dsw), ptr(out),
                                          1 if out_f32 else 0, M, N, K, N, stream()))
    res = host(out.float())
    assert kc_lib.lib().kc_get_device_status() == kc_lib.KC_OK
    return res


@pytest.mark.parametrize("M,N,K", [(128, 256, 128), (256, 512, 1024), (300, 264, 4112),
                                   (1, 8, 16), (129, 520, 2048), (512, 1024, 512)])
def test_fp8_gemm_small(cuda, M, N, K):
    qa, sa, qw, sw = _quantized_operands(M, N, K, seed=M + N + K)
    ref = O.gemm_fp8_rowcol(qa, sa, qw, sw)
    got32 = _run(qa, sa, qw, sw, M, N, K, out_f32=True)
    assert normwise_err(got32, ref) <= 1e-4
    got16 = _run(qa, sa, qw, sw, M, N, K, out_f32=False)
    assert normwise_err(got16, ref) <= 1e-2
    # the reference's own chain: dequantize both operands, fp32 GEMM
    chain = O.gemm_nt_f32(O.dequantize_fp8(qa, sa, M, K, True), O.dequantize_fp8(qw, sw, N, K, True))
    assert normwise_err(got16, chain) <= 1e-2


def test_fp8_gemm_config4_sampled_rows(cuda):
    """Config 4 shape (M=4096, N=8192, K=8192); the oracle checks 24 seeded rows."""
    M, N, K = 4096, 8192, 8192
    qa, sa, qw, sw = _quantized_operands(M, N, K, seed=4)
    got = _run(qa, sa, qw, sw, M, N, K, out_f32=False)
    rows = np.sort(np.random.default_rng(1).choice(M, 24, replace=False))
    rows[0], rows[-1] = 0, M - 1
    ref = O.gemm_fp8_rowcol(qa[rows], sa[rows], qw, sw)
    assert normwise_err(got[rows], ref) <= 1e-2
    assert np.all(np.isfinite(got))


def test_fp8_gemm_rejects_bad_args(cuda):
    l = kc_lib.lib()
    b = torch.zeros(4096, dtype=torch.uint8, device=cuda)
    with pytest.raises(kc_lib.KcError):   # K not a multiple of 16
        kc_lib.check(l.kc_gemm_fp8(ptr(b), ptr(b), ptr(b), ptr(b), ptr(b), 0, 4, 8, 24, 8, stream()))
    with pytest.raises(kc_lib.KcError):   # N not a multiple of 8
        kc_lib.check(l.kc_gemm_fp8(ptr(b), ptr(b), ptr(b), ptr(b), ptr(b), 0, 4, 12, 32, 12, stream()))


def test_fp8_gemm_torch_op(cuda):
    """kernel_craft_torch_ops.fp8_gemm (and its torch.ops registration) on codes
    and scales from the library's own per-token / per-channel quantizers."""
    import kernel_craft_torch_ops as ops
    M, N, K = 200, 264, 2048
    x = O.make_outlier_activations(M, K, seed=31)
    w = O.make_weight_f32(N, K, seed=32)
    qa, sa = ops.fp8_quantize(dev(x), per_token=True)
    qw, sw = ops.fp8_quantize_per_channel(dev(w))
    y = ops.fp8_gemm(qa, sa, qw, sw, out_dtype=torch.float32)
    ref = O.gemm_fp8_rowcol(host(qa).view(np.uint8), host(sa), host(qw).view(np.uint8), host(sw))
    assert normwise_err(host(y), ref) <= 1e-4
    y2 = torch.ops.kernel_craft.fp8_gemm(qa, sa, qw, sw)
    assert y2.dtype == torch.bfloat16 and normwise_err(host(y2.float()), ref) <= 1e-2

"""GPU parity: tcgen05 W4A16 GEMM (kc_gemm_w4a16) vs the oracle.

Bars (written here): fp32 output normwise <= 1e-5 against the bf16-rounded
dequantized weights (ora_dequantize_w4_bf16, bit-identical to the kernel's
weights) times the bf16 activations in double -- only the accumulation order
differs; bf16 output normwise <= 1e-2 against the oracle's fp32-weight GEMM
(ora_gemm_w4a16, the reference's dequantize -> GEMM chain,
quant_int4.cu:99-104 and tensor_parallel.cu:164-192).
"""
import numpy as np
import pytest
import torch

import kc_lib
import oracle as O
from kc_testutil import dev, host, normwise_err, ptr, stream

pytestmark = pytest.mark.gpu


def _run(x_bits, packed, scales, M, N, K, gs, out_f32):
    dx, dp, ds = dev(x_bits.view(np.int16)), dev(packed), dev(scales.view(np.int16))
    out = torch.full((M, N), float("nan"), dtype=torch.float32 if out_f32 else torch.bfloat16,
                     device="cuda:0")
    kc_lib.check(kc_lib.lib().kc_gemm_w4a16(ptr(dx), ptr(dp), ptr(ds), ptr(out), 1 if out_f32 else 0,
                                            M, N, K, gs, N, stream()))
    res = host(out.float())
    assert kc_lib.lib().kc_get_device_status() == kc_lib.KC_OK
    return res


def _exact_weight_ref(x_bits, packed, scales, N, K, gs):
    w = O.bf16_bits_to_f32(O.dequantize_w4_bf16(packed, scales, N, K, gs)).astype(np.float64)
    return O.bf16_bits_to_f32(x_bits).astype(np.float64) @ w.T


@pytest.mark.parametrize("M,N,K,gs", [(1, 128, 64, 64), (256, 256, 512, 128), (300, 200, 1024, 128),
                                      (513, 384, 2048, 64), (128, 1000, 4096, 128),
                                      (257, 136, 256, 256), (64, 130, 128, 128)])
def test_w4a16_gemm_small(cuda, M, N, K, gs):
    packed, scales = O.make_w4_gptq(N, K, gs, seed=M + N)
    x = O.make_activations_bf16(M, K, seed=K)
    got32 = _run(x, packed, scales, M, N, K, gs, out_f32=True)
    assert normwise_err(got32, _exact_weight_ref(x, packed, scales, N, K, gs)) <= 1e-5
    got16 = _run(x, packed, scales, M, N, K, gs, out_f32=False)
    assert normwise_err(got16, O.gemm_w4a16(x, packed, scales, M, N, K, gs)) <= 1e-2


def test_w4a16_gemm_config3_sampled(cuda):
    """Config 3 shape (M=2048, K=8192, N=28672, group 128); the oracle checks
    16 seeded token rows against 1024 seeded weight rows."""
    M, N, K, gs = 2048, 28672, 8192, 128
    packed, scales = O.make_w4_gptq(N, K, gs, seed=3)
    x = O.make_activations_bf16(M, K, seed=4)
    got = _run(x, packed, scales, M, N, K, gs, out_f32=False)
    assert np.all(np.isfinite(got))
    rng = np.random.default_rng(5)
    rows = np.sort(rng.choice(M, 16, replace=False))
    cols = np.sort(rng.choice(N, 1024, replace=False))
    rows[0], rows[-1], cols[0], cols[-1] = 0, M - 1, 0, N - 1
    ref = O.gemm_w4a16(x[rows], packed[cols], scales[cols], len(rows), len(cols), K, gs)
    assert normwise_err(got[np.ix_(rows, cols)], ref) <= 1e-2


def test_w4a16_gemm_rejects_bad_args(cuda):
    l = kc_lib.lib()
    b = torch.zeros(1 << 16, dtype=torch.uint8, device=cuda)
    with pytest.raises(kc_lib.KcError):   # K not a multiple of 64
        kc_lib.check(l.kc_gemm_w4a16(ptr(b), ptr(b), ptr(b), ptr(b), 0, 4, 8, 96, 32, 8, stream()))
    with pytest.raises(kc_lib.KcError):   # group size not dividing K
        kc_lib.check(l.kc_gemm_w4a16(ptr(b), ptr(b), ptr(b), ptr(b), 0, 4, 8, 192, 128, 8, stream()))
    with pytest.raises(kc_lib.KcError):   # misaligned activations
        kc_lib.check(l.kc_gemm_w4a16(ptr(b[2:]), ptr(b), ptr(b), ptr(b), 0, 4, 8, 128, 64, 8, stream()))


def test_w4a16_gemm_torch_op(cuda):
    """kernel_craft_torch_ops.w4a16_gemm and torch.ops.kernel_craft.w4a16_gemm
    run the same kernel as the C ABI call."""
    import kernel_craft_torch_ops as ops
    M, N, K, gs = 300, 384, 1024, 128
    packed, scales = O.make_w4_gptq(N, K, gs, seed=21)
    x = O.make_activations_bf16(M, K, seed=22)
    dx = dev(x.view(np.int16)).view(torch.bfloat16)
    dp, ds = dev(packed), dev(scales)
    y = ops.w4a16_gemm(dx, dp, ds, gs)
    assert y.shape == (M, N) and y.dtype == torch.bfloat16
    ref = _run(x, packed, scales, M, N, K, gs, out_f32=False)
    np.testing.assert_array_equal(host(y.float()), ref)
    y2 = torch.ops.kernel_craft.w4a16_gemm(dx, dp, ds, gs)
    assert torch.equal(y2, y)

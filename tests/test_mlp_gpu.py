"""GPU parity: the W4A16 GEMM with the GELU in its epilogue (kc_gemm_w4a16_act)
and the MLP block built on it (tp.MLPBlockW4A16, one GPU), vs the oracle.

The block is the reference's column-parallel -> GELU -> row-parallel chain
(examples/python/transformer/tensor_parallel.py:150-172) with the GELU
x * sigmoid(1.702 x) of that file (:162).

Bars (written here): fp32 output normwise <= 1e-4 against the activation of
the exact-weight double GEMM (the kernel's __expf / __fdividef against
numpy's exp); bf16 output and the block normwise <= 1e-2 against the oracle
(ora_gemm_w4a16 with fp32 weights, then the activation, the bf16 rounding of
h and the second GEMM); KC_ACT_NONE and the torch op bit for bit against the
plain entry points.
"""
import numpy as np
import pytest
import torch

import kc_lib
import oracle as O
from kc_testutil import dev, host, normwise_err, ptr, stream

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _no_device_timeouts(cuda):
    yield
    assert kc_lib.lib().kc_get_device_status() == kc_lib.KC_OK


def _gemm(x_bits, packed, scales, M, N, K, gs, out_f32, act, ldc=None):
    ldc = ldc or N
    dx, dp, ds = dev(x_bits.view(np.int16)), dev(packed), dev(scales.view(np.int16))
    out = torch.full((M, ldc), float("nan"), dtype=torch.float32 if out_f32 else torch.bfloat16,
                     device="cuda:0")
    kc_lib.check(kc_lib.lib().kc_gemm_w4a16_act(ptr(dx), ptr(dp), ptr(ds), ptr(out), 1 if out_f32 else 0,
                                                M, N, K, gs, ldc, act, stream()))
    return host(out.float())[:, :N]


def _exact_weight_ref(x_bits, packed, scales, N, K, gs):
    w = O.bf16_bits_to_f32(O.dequantize_w4_bf16(packed, scales, N, K, gs)).astype(np.float64)
    return O.bf16_bits_to_f32(x_bits).astype(np.float64) @ w.T


def _gelu64(h):
    with np.errstate(over="ignore"):     # exp overflows to inf on the negative tail: h / inf = -0
        return h / (1.0 + np.exp(-1.702 * h))


# (256, 256, 512): TMA-store epilogue; (64, 130, 128): pitch the TMA cannot
# address, direct stores; (300, 200, 1024): partial tiles in both directions
@pytest.mark.parametrize("M,N,K,gs", [(256, 256, 512, 128), (64, 130, 128, 128), (300, 200, 1024, 128),
                                      (129, 384, 2048, 64)])
def test_gelu_epilogue(cuda, M, N, K, gs):
    packed, scales = O.make_w4_gptq(N, K, gs, seed=M + 3 * N)
    x = O.make_activations_bf16(M, K, seed=K + 1)
    got32 = _gemm(x, packed, scales, M, N, K, gs, True, kc_lib.KC_ACT_GELU_QUICK)
    assert normwise_err(got32, _gelu64(_exact_weight_ref(x, packed, scales, N, K, gs))) <= 1e-4
    got16 = _gemm(x, packed, scales, M, N, K, gs, False, kc_lib.KC_ACT_GELU_QUICK)
    assert normwise_err(got16, O.gelu_quick(O.gemm_w4a16(x, packed, scales, M, N, K, gs))) <= 1e-2
    # KC_ACT_NONE is the plain GEMM, bit for bit
    plain = _gemm(x, packed, scales, M, N, K, gs, False, kc_lib.KC_ACT_NONE)
    dx, dp, ds = dev(x.view(np.int16)), dev(packed), dev(scales.view(np.int16))
    ref = torch.empty(M, N, dtype=torch.bfloat16, device=cuda)
    kc_lib.check(kc_lib.lib().kc_gemm_w4a16(ptr(dx), ptr(dp), ptr(ds), ptr(ref), 0, M, N, K, gs, N,
                                            stream()))
    np.testing.assert_array_equal(plain, host(ref.float()))


def test_gelu_epilogue_extremes(cuda):
    """Outputs far out on both tails: the activation gives x and -0 there, no NaN."""
    M, N, K, gs = 128, 128, 4096, 128
    packed, scales = O.make_w4_gptq(N, K, gs, seed=9)
    scales = np.full_like(scales, 0.5)   # large outputs: |y| reaches several hundred
    x = O.make_activations_bf16(M, K, seed=10)
    got = _gemm(x, packed, scales, M, N, K, gs, True, kc_lib.KC_ACT_GELU_QUICK)
    pre = _exact_weight_ref(x, packed, scales, N, K, gs)
    assert np.all(np.isfinite(got))
    assert np.abs(pre).max() > 200          # the tails are reached
    assert normwise_err(got, _gelu64(pre)) <= 1e-4


def test_act_rejects_unknown(cuda):
    b = torch.zeros(1 << 16, dtype=torch.uint8, device=cuda)
    with pytest.raises(kc_lib.KcError):
        kc_lib.check(kc_lib.lib().kc_gemm_w4a16_act(ptr(b), ptr(b), ptr(b), ptr(b), 0, 4, 8, 128, 64, 8,
                                                    7, stream()))


def test_torch_op_activation(cuda):
    import kernel_craft_torch_ops as ops
    M, N, K, gs = 200, 256, 1024, 128
    packed, scales = O.make_w4_gptq(N, K, gs, seed=31)
    x = O.make_activations_bf16(M, K, seed=32)
    y = ops.w4a16_gemm(dev(x.view(np.int16)).view(torch.bfloat16), dev(packed), dev(scales), gs,
                       activation="gelu_quick")
    np.testing.assert_array_equal(host(y.float()),
                                  _gemm(x, packed, scales, M, N, K, gs, False, kc_lib.KC_ACT_GELU_QUICK))
    with pytest.raises(ValueError):
        ops.w4a16_gemm(dev(x.view(np.int16)).view(torch.bfloat16), dev(packed), dev(scales), gs,
                       activation="relu")


def _mlp_inputs(M, H, I, gs, seed):
    w1p, w1s = O.make_w4_gptq(I, H, gs, seed=seed)
    w2p, w2s = O.make_w4_gptq(H, I, gs, seed=seed + 1)
    x = O.make_activations_bf16(M, H, seed=seed + 2)
    return x, w1p, w1s, w2p, w2s


def _run_block(x, w1p, w1s, w2p, w2s, M, H, I, gs):
    import tp
    blk = tp.MLPBlockW4A16(M, H, I, gs)
    y = blk(dev(x.view(np.int16)).view(torch.bfloat16), dev(w1p), dev(w1s.view(np.int16)), dev(w2p),
            dev(w2s.view(np.int16)))
    return host(y)


@pytest.mark.parametrize("M,H,I", [(64, 512, 1024), (300, 256, 768)])
def test_mlp_block_one_gpu(cuda, M, H, I):
    gs = 128
    x, w1p, w1s, w2p, w2s = _mlp_inputs(M, H, I, gs, seed=M + H)
    got = _run_block(x, w1p, w1s, w2p, w2s, M, H, I, gs)
    assert normwise_err(got, O.mlp_block_w4a16(x, w1p, w1s, w2p, w2s, M, H, I, gs)) <= 1e-2


def test_mlp_block_bench_shape_sampled(cuda):
    """The bench's block (M=2048, H=4096, I=16384); the oracle runs 8 seeded
    token rows through the whole block."""
    M, H, I, gs = 2048, 4096, 16384, 128
    x, w1p, w1s, w2p, w2s = _mlp_inputs(M, H, I, gs, seed=40)
    got = _run_block(x, w1p, w1s, w2p, w2s, M, H, I, gs)
    assert np.all(np.isfinite(got))
    rows = np.sort(np.random.default_rng(6).choice(M, 8, replace=False))
    rows[0], rows[-1] = 0, M - 1
    ref = O.mlp_block_w4a16(x[rows], w1p, w1s, w2p, w2s, len(rows), H, I, gs)
    assert normwise_err(got[rows], ref) <= 1e-2

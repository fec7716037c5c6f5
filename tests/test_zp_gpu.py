"""GPU parity: W4A16 with per-group zero points (AWQ, asymmetric GPTQ).

w[n, k] = (u - z[n, k/gs]) * s[n, k/gs], zeros u8 [N, K/gs] (0..15).  Bars as
for the symmetric kernels: dequantized bf16 weights bit-exact; GEMV (fp32
accumulation) normwise <= 1e-3 against the oracle; GEMM fp32 output <= 1e-5
against the exact bf16 weights in double precision, bf16 output <= 1e-2.
The conversion of a real AWQ layout (checkpoint.from_awq) feeds the kernels
in the last test.
"""
import ctypes

import numpy as np
import pytest
import torch

import checkpoint as C
import kc_lib
import oracle as O
from kc_testutil import dev, host, misaligned, normwise_err, ptr, stream

pytestmark = pytest.mark.gpu
GEMV_TOL = 1e-3


@pytest.fixture(autouse=True)
def _no_device_timeouts(cuda):
    yield
    assert kc_lib.lib().kc_get_device_status() == kc_lib.KC_OK


def _inputs(N, K, gs, seed, M=1):
    packed, scales = O.make_w4_gptq(N, K, gs, seed=seed)
    zeros = np.random.default_rng(seed + 1).integers(0, 16, (N, K // gs), dtype=np.uint8)
    x = O.make_activations_bf16(M, K, seed=seed + 2)
    return packed, scales, zeros, x


def _gemv_zp(packed, scales, zeros, x, M, N, K, gs):
    y = torch.full((M, N), float("nan"), dtype=torch.float32, device="cuda:0")
    dp, ds, dz = dev(packed), dev(scales), dev(zeros)
    dx = dev(x).view(torch.bfloat16)
    kc_lib.check(kc_lib.lib().kc_gemv_w4a16_zp(ptr(dp), ptr(ds), ptr(dz), ptr(dx), ptr(y), M, N, K,
                                               gs, stream()))
    return host(y)


@pytest.mark.parametrize("N,K,gs", [(256, 512, 128), (40, 384, 128), (33, 96, 32), (64, 4096, 64)])
def test_dequant_bf16_zp_bitexact(cuda, N, K, gs):
    packed, scales, zeros, _ = _inputs(N, K, gs, seed=N + K)
    out = torch.empty(N, K, dtype=torch.bfloat16, device=cuda)
    dp, ds, dz = dev(packed), dev(scales), dev(zeros)
    kc_lib.check(kc_lib.lib().kc_dequantize_w4_bf16_zp(ptr(dp), ptr(ds), ptr(dz), ptr(out), N, K, gs,
                                                       stream()))
    got = host(out.view(torch.int16)).view(np.uint16)
    np.testing.assert_array_equal(got, O.dequantize_w4_bf16(packed, scales, N, K, gs, zeros=zeros))
    # the scalar path (misaligned packed bytes) gives the same bits
    out2 = torch.empty(N, K, dtype=torch.bfloat16, device=cuda)
    dpm = misaligned(dp, 4)
    kc_lib.check(kc_lib.lib().kc_dequantize_w4_bf16_zp(ptr(dpm), ptr(ds), ptr(dz), ptr(out2), N, K,
                                                       gs, stream()))
    np.testing.assert_array_equal(host(out2.view(torch.int16)).view(np.uint16), got)


@pytest.mark.parametrize("M", [1, 3, 8])
@pytest.mark.parametrize("N,K,gs", [(256, 1024, 128), (100, 384, 128), (48, 2048, 256), (24, 256, 64)])
def test_gemv_zp_vs_oracle(cuda, M, N, K, gs):
    packed, scales, zeros, x = _inputs(N, K, gs, seed=3 * M + N, M=M)
    y = _gemv_zp(packed, scales, zeros, x, M, N, K, gs)
    ref = O.gemv_w4a16(packed, scales, x, M, N, K, gs, zeros=zeros)
    assert normwise_err(y, ref) <= GEMV_TOL


@pytest.mark.parametrize("K,N", [(4096, 12288), (11008, 4096)])
def test_gemv_zp_7b_shapes_batch1(cuda, K, N):
    """Config-2 shapes at batch 1 (the integer tensor-core path), 96 seeded rows."""
    gs = 128
    packed, scales, zeros, x = _inputs(N, K, gs, seed=K + N)
    y = _gemv_zp(packed, scales, zeros, x, 1, N, K, gs)
    rows = np.sort(np.random.default_rng(1).choice(N, 96, replace=False))
    rows[0], rows[-1] = 0, N - 1
    ref = O.gemv_w4a16(packed[rows], scales[rows], x, 1, len(rows), K, gs, zeros=zeros[rows])
    assert normwise_err(y[:, rows], ref) <= GEMV_TOL


def test_gemv_zp_all_eight_equals_symmetric(cuda):
    """z = 8 everywhere through the zero-point path gives the symmetric result."""
    N, K, gs = 512, 4096, 128
    packed, scales, _, x = _inputs(N, K, gs, seed=21)
    z8 = np.full((N, K // gs), 8, np.uint8)
    y = _gemv_zp(packed, scales, z8, x, 1, N, K, gs)
    import kernel_craft_torch_ops as ops
    ys = host(ops.w4a16_gemv(dev(packed), dev(scales).view(torch.float16),
                             dev(x).view(torch.bfloat16), gs))
    assert normwise_err(y, ys) <= 1e-6


def test_gemv_grouped_zp_mixed(cuda):
    """One launch: two problems with zero points, one without (NULL: 8)."""
    gs, M = 128, 1
    shapes = [(4096, 1536), (4096, 512), (1024, 2752)]
    probs, keep, zps = [], [], []
    for i, (K, N) in enumerate(shapes):
        packed, scales, zeros, x = _inputs(N, K, gs, seed=60 + i)
        if i == 1:
            zeros = None
        dp, ds, dx = dev(packed), dev(scales), dev(x).view(torch.bfloat16)
        dz = dev(zeros) if zeros is not None else None
        y = torch.full((M, N), float("nan"), dtype=torch.float32, device=cuda)
        keep.append((packed, scales, zeros, x, y, dp, ds, dx, dz, N, K))
        probs.append(kc_lib.W4A16Problem(dp.data_ptr(), ds.data_ptr(), dx.data_ptr(), y.data_ptr(), N, K))
        zps.append(dz.data_ptr() if dz is not None else None)
    arr = (kc_lib.W4A16Problem * 3)(*probs)
    zarr = (ctypes.c_void_p * 3)(*zps)
    kc_lib.check(kc_lib.lib().kc_gemv_w4a16_grouped_zp(arr, zarr, 3, M, gs, stream()))
    for packed, scales, zeros, x, y, *_, N, K in keep:
        ref = O.gemv_w4a16(packed, scales, x, M, N, K, gs, zeros=zeros)
        assert normwise_err(host(y), ref) <= GEMV_TOL


@pytest.mark.parametrize("M,N,K,gs", [(256, 256, 512, 128), (130, 384, 1024, 64), (64, 128, 256, 256)])
def test_gemm_zp(cuda, M, N, K, gs):
    import kernel_craft_torch_ops as ops
    packed, scales, zeros, x = _inputs(N, K, gs, seed=M + N, M=M)
    dx = dev(x).view(torch.bfloat16)
    dp, ds, dz = dev(packed), dev(scales).view(torch.float16), dev(zeros)
    c32 = host(ops.w4a16_gemm(dx, dp, ds, gs, out_dtype=torch.float32, zeros=dz))
    w = O.bf16_bits_to_f32(O.dequantize_w4_bf16(packed, scales, N, K, gs, zeros=zeros)).astype(np.float64)
    ref = O.bf16_bits_to_f32(x).astype(np.float64) @ w.T
    assert normwise_err(c32, ref) <= 1e-5
    c16 = host(ops.w4a16_gemm(dx, dp, ds, gs, zeros=dz).float())
    assert normwise_err(c16, O.gemm_w4a16(x, packed, scales, M, N, K, gs, zeros=zeros)) <= 1e-2


def test_awq_checkpoint_through_the_kernels(cuda):
    """An asymmetric AWQ layer (qweight/qzeros packed with AWQ's column
    interleave) converted by checkpoint.from_awq runs through the GEMV and
    the GEMM against the checkpoint's own dequantization."""
    import kernel_craft_torch_ops as ops
    K, N, gs, M = 1024, 256, 128, 64
    rng = np.random.default_rng(71)
    u = rng.integers(0, 16, (K, N), dtype=np.uint8)
    z = rng.integers(0, 16, (K // gs, N), dtype=np.uint8)
    s = rng.uniform(0.002, 0.02, (K // gs, N)).astype(np.float16)

    def awq_pack(q):  # AWQ packing: columns interleaved 0 2 4 6 1 3 5 7 within a word
        q = q.astype(np.uint32).reshape(-1, 8)[:, [0, 2, 4, 6, 1, 3, 5, 7]].reshape(q.shape)
        out = np.zeros((q.shape[0], q.shape[1] // 8), np.uint32)
        for j in range(8):
            out |= q[:, j::8] << (4 * j)
        return out.astype(np.int32)

    w = C.from_awq(awq_pack(u), awq_pack(z), s, group_size=gs)
    assert w.zeros is not None
    wt = ((u.astype(np.float64) - z[np.arange(K) // gs]) * s[np.arange(K) // gs].astype(np.float64)).T
    x = O.make_activations_bf16(M, K, seed=72)
    xf = O.bf16_bits_to_f32(x).astype(np.float64)
    dp, ds, dz = dev(w.packed), dev(w.scales).view(torch.float16), dev(w.zeros)
    dx = dev(x).view(torch.bfloat16)
    y = host(ops.w4a16_gemv(dp, ds, dx[:1], gs, zeros=dz))
    assert normwise_err(y, xf[:1] @ wt.T) <= GEMV_TOL
    c = host(ops.w4a16_gemm(dx, dp, ds, gs, zeros=dz).float())
    assert normwise_err(c, xf @ wt.T) <= 1e-2

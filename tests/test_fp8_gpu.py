"""GPU parity: FP8 E4M3 quantization, dequantization and SmoothQuant.

Bar: bit-exact codes, scales and dequantized values against the oracle, and
against the reference's own kernels (oracle/_ref/libkcref.so) when present.
"""
import numpy as np
import pytest
import torch

import kc_lib
import kcref
import oracle as O
from kc_testutil import dev, host, last_error, misaligned, ptr, stream

pytestmark = pytest.mark.gpu


def _quant_per_token(x_dev, rows, cols):
    q = torch.full((rows, cols), 0x55, dtype=torch.int8, device=x_dev.device)
    s = torch.full((rows,), -1.0, dtype=torch.float32, device=x_dev.device)
    kc_lib.check(kc_lib.lib().kc_quantize_fp8_per_token(ptr(x_dev), ptr(q), ptr(s), rows, cols,
                                                        stream()))
    return host(q).view(np.uint8), host(s)


def _edge_matrix(rows, cols, seed):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((rows, cols)).astype(np.float32)
    x *= (10.0 ** rng.integers(-3, 4, (rows, 1))).astype(np.float32)
    specials = np.array([np.nan, np.inf, -np.inf, -0.0, 0.0, 1e-40, -1e-40, 3.4e38, 448.0, 464.0,
                         -464.0, 2.0**-10, 2.0**-9 * 1.5], np.float32)
    if rows > 2:
        x[1, :] = 0.0                     # amax 0 -> scale 1
        x[2, : min(cols, len(specials))] = specials[: min(cols, len(specials))]
    if rows > 3:
        x[3, :] = -0.0
    return x


@pytest.mark.parametrize("rows,cols", [(256, 8192), (64, 4096), (33, 1000), (17, 4), (9, 3),
                                       (5, 31), (4, 65536 + 12), (3, 16384), (2, 1), (130, 20000)])
def test_per_token_bitexact(cuda, rows, cols):
    x = _edge_matrix(rows, cols, rows * 31 + cols)
    q, s = _quant_per_token(dev(x), rows, cols)
    wq, ws = O.quantize_fp8_per_token(x)
    np.testing.assert_array_equal(s.view(np.uint32), ws.view(np.uint32))
    np.testing.assert_array_equal(q, wq)
    if kcref.available() and cols >= 32 and cols % 32 == 0:
        # the reference kernel's warp reduction needs whole warps (fp8_quant.cu:43-44,211)
        rq, rs = kcref.quantize_fp8(dev(x), True)
        np.testing.assert_array_equal(host(rs).view(np.uint32), ws.view(np.uint32))
        np.testing.assert_array_equal(host(rq).view(np.uint8), wq)


def test_config1_outliers_bitexact(cuda):
    """Config 1 statistics (N(0,1), 1% channels x20) on a 512-row slice."""
    x = O.make_outlier_activations(8192, 8192, seed=0)[:512].copy()
    q, s = _quant_per_token(dev(x), 512, 8192)
    wq, ws = O.quantize_fp8_per_token(x)
    np.testing.assert_array_equal(s.view(np.uint32), ws.view(np.uint32))
    np.testing.assert_array_equal(q, wq)
    w = O.make_weight_f32(256, 8192, seed=2)
    qw = torch.empty(256, 8192, dtype=torch.int8, device=cuda)
    sw = torch.empty(256, dtype=torch.float32, device=cuda)
    dw = dev(w)
    kc_lib.check(kc_lib.lib().kc_quantize_fp8_per_channel(ptr(dw), ptr(qw), ptr(sw), 256, 8192,
                                                          stream()))
    wq2, ws2 = O.quantize_fp8_per_token(w)
    np.testing.assert_array_equal(host(sw), ws2)
    np.testing.assert_array_equal(host(qw).view(np.uint8), wq2)


def test_unaligned_input_generic_path(cuda):
    x = _edge_matrix(7, 1024, 3)
    q, s = _quant_per_token(misaligned(dev(x), 4), 7, 1024)
    wq, ws = O.quantize_fp8_per_token(x)
    np.testing.assert_array_equal(q, wq)
    np.testing.assert_array_equal(s, ws)


@pytest.mark.parametrize("count", [4096 * 33, 1001, 4])
def test_per_tensor_device_scale(cuda, count):
    rng = np.random.default_rng(count)
    x = (rng.standard_normal(count) * 3).astype(np.float32)
    scale = O.per_tensor_scale(x)
    dx = dev(x)
    ds = dev(np.array([scale], np.float32))
    q = torch.empty(count, dtype=torch.int8, device=cuda)
    kc_lib.check(kc_lib.lib().kc_quantize_fp8_per_tensor(ptr(dx), ptr(q), ptr(ds), count, stream()))
    want = O.quantize_fp8_per_tensor(x, scale)
    np.testing.assert_array_equal(host(q).view(np.uint8), want)
    # reference ABI: per_token = false reads the caller's scale (fp8_quant.cu:215-223)
    q2 = torch.empty(count, dtype=torch.int8, device=cuda)
    kc_lib.lib().launch_quantize_fp8(ptr(dx), ptr(q2), ptr(ds), 1, count, False, stream())
    kc_lib.check_last()
    np.testing.assert_array_equal(host(q2).view(np.uint8), want)
    # dynamic: the scale computed on the device
    q3 = torch.empty(count, dtype=torch.int8, device=cuda)
    s3 = torch.empty(1, dtype=torch.float32, device=cuda)
    ws = torch.empty(1, dtype=torch.int32, device=cuda)
    kc_lib.check(kc_lib.lib().kc_quantize_fp8_per_tensor_dynamic(ptr(dx), ptr(q3), ptr(s3), count,
                                                                 ptr(ws), 4, stream()))
    assert host(s3)[0] == scale
    np.testing.assert_array_equal(host(q3).view(np.uint8), want)
    if kcref.available():
        rq, _ = kcref.quantize_fp8(dx.view(1, count), False, scale=float(scale))
        np.testing.assert_array_equal(host(rq).view(np.uint8).reshape(-1), want)


@pytest.mark.parametrize("rows,cols,per_token", [(64, 4096, True), (33, 1000, True),
                                                 (8, 64, False), (5, 7, True)])
def test_dequant_bitexact(cuda, rows, cols, per_token):
    rng = np.random.default_rng(rows + cols)
    codes = rng.integers(0, 256, (rows, cols), dtype=np.uint8)
    scales = rng.uniform(0.001, 2.0, rows if per_token else 1).astype(np.float32)
    out = torch.empty(rows, cols, dtype=torch.float32, device=cuda)
    dc, ds = dev(codes), dev(scales)   # keep the device copies alive across the call
    kc_lib.lib().launch_dequantize_fp8(ptr(dc), ptr(ds), ptr(out), rows, cols, per_token, stream())
    kc_lib.check_last()
    got = host(out)
    want = O.dequantize_fp8(codes, scales, rows, cols, per_token)
    nan = np.isnan(want)
    np.testing.assert_array_equal(np.isnan(got), nan)
    np.testing.assert_array_equal(got[~nan].view(np.uint32), want[~nan].view(np.uint32))
    if kcref.available():
        r = host(kcref.dequantize_fp8(dev(codes.view(np.int8)), dev(scales), rows, cols, per_token))
        np.testing.assert_array_equal(np.isnan(r), nan)
        np.testing.assert_array_equal(r[~nan].view(np.uint32), got[~nan].view(np.uint32))


@pytest.mark.parametrize("rows,cols", [(64, 4096), (4, 16), (7, 33)])
def test_smoothquant_and_fused(cuda, rows, cols):
    rng = np.random.default_rng(cols)
    x = O.make_outlier_activations(rows, cols, seed=cols)
    s = rng.uniform(0.5, 20.0, cols).astype(np.float32)
    out = torch.empty(rows, cols, dtype=torch.float32, device=cuda)
    dx, dsm = dev(x), dev(s)
    kc_lib.lib().launch_smoothquant_scale(ptr(dx), ptr(dsm), ptr(out), rows, cols, stream())
    kc_lib.check_last()
    sm = O.smoothquant_scale(x, s)
    np.testing.assert_array_equal(host(out).view(np.uint32), sm.view(np.uint32))
    # fused divide + per-token quant == the two reference steps
    q = torch.empty(rows, cols, dtype=torch.int8, device=cuda)
    sc = torch.empty(rows, dtype=torch.float32, device=cuda)
    kc_lib.check(kc_lib.lib().kc_smoothquant_quantize_fp8(ptr(dx), ptr(dsm), ptr(q), ptr(sc),
                                                          rows, cols, stream()))
    wq, ws = O.quantize_fp8_per_token(sm)
    np.testing.assert_array_equal(host(sc), ws)
    np.testing.assert_array_equal(host(q).view(np.uint8), wq)
    if kcref.available():
        np.testing.assert_array_equal(host(kcref.smoothquant_scale(dev(x), dev(s))).view(np.uint32),
                                      sm.view(np.uint32))


def test_reference_fp8_kats(cuda, golden):
    d = golden("kat_fp8.npz")
    import kernel_craft_torch_ops as ops
    x = d["pt_in"]
    q, s = ops.fp8_quantize(dev(x), per_token=True)
    xh = host(ops.fp8_dequantize(q, s, 8, 64, per_token=True))
    nz = np.abs(x) > 1e-6
    assert np.max(np.abs(xh[nz] - x[nz]) / np.abs(x[nz])) < 0.15        # test_fp8_quant.cpp:67
    q0, s0 = ops.fp8_quantize(torch.zeros(4, 32, device=cuda), per_token=True)
    assert torch.all(ops.fp8_dequantize(q0, s0, 4, 32, True) == 0)      # :94
    out = ops.smoothquant_scale(dev(d["sq_in"]), dev(d["sq_smooth"]))
    np.testing.assert_array_equal(host(out), d["sq_expected"])         # :125-132
    qt, st = ops.fp8_quantize(dev(d["tensor_in"]), per_token=False)
    assert host(st)[0] == d["tensor_scale"][0]                          # scale = max_abs / 448
    xt = host(ops.fp8_dequantize(qt, st, 4, 32, per_token=False))
    nz = np.abs(d["tensor_in"]) > 1e-6
    assert np.max(np.abs(xt[nz] - d["tensor_in"][nz]) / np.abs(d["tensor_in"][nz])) < 0.15
    assert q.shape == (8, 64) and s.shape == (8,) and st.shape == (1,)


def test_rejects_bad_args(cuda):
    l = kc_lib.lib()
    b = torch.zeros(16, dtype=torch.float32, device=cuda)
    last_error()
    l.launch_quantize_fp8(ptr(b), None, ptr(b), 4, 4, True, stream())
    assert last_error()[0] == kc_lib.KC_ERR_INVALID_ARG
    with pytest.raises(kc_lib.KcError):
        kc_lib.check(l.kc_quantize_fp8_per_tensor_dynamic(ptr(b), ptr(b), ptr(b), 16, ptr(b), 2,
                                                          stream()))

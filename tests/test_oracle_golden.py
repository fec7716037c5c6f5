"""Pins the CPU oracle to the reference's own known answers (CPU only).

Fixtures come from tests/golden/make_golden.py (the reference's KATs) and,
when present, tests/golden/ref_*.npz (outputs of the reference's own CUDA
kernels run on a B200 by tests/golden/make_golden_ref.py).
"""
import numpy as np
import pytest
import torch

import oracle as O

GOLDEN = O.HERE.parent / "tests" / "golden"


# ---------------------------------------------------------------- INT4 KATs --
def test_dequant_kat_4x8(golden):
    # tests/test_quant_int4.cpp:35-88 (max abs err < 1e-5); here bit-exact.
    d = golden("kat_quant_int4.npz")
    out = O.dequantize_int4(d["deq4x8_packed"], d["deq4x8_scales"], d["deq4x8_zeros"], 4, 8, 8)
    np.testing.assert_array_equal(out, d["deq4x8_expected"])


def test_dequant_kat_multigroup(golden):
    # tests/test_quant_int4.cpp:148-199 (srand(13), per-group scales); bit-exact.
    d = golden("kat_quant_int4.npz")
    out = O.dequantize_int4(d["mg_packed"], d["mg_scales"], d["mg_zeros"], 4, 128, 64)
    np.testing.assert_array_equal(out, d["mg_expected"])


def test_gemv_kat_16x16(golden):
    # tests/test_quant_int4.cpp:90-146: |err| < 1e-4 against the test's fp32 loop.
    d = golden("kat_quant_int4.npz")
    y = O.gemv_int4(d["gemv16_packed"], d["gemv16_scales"], d["gemv16_zeros"], d["gemv16_x"],
                    16, 16, 8)
    assert np.max(np.abs(y - d["gemv16_expected"])) < 1e-4


def test_bindings_dequant_kat(golden):
    # src/python/tests/test_transformer_bindings.py:185-196 (atol 1e-5); bit-exact.
    d = golden("kat_bindings.npz")
    out = O.dequantize_int4(d["bind_packed"], d["bind_scales"], d["bind_zeros"], 4, 16, 8)
    np.testing.assert_array_equal(out, d["bind_expected"])


@pytest.mark.parametrize("tag", ["small", "medium", "gs64"])
def test_triton_gemv_reference(golden, tag):
    # src/python/tests/test_triton_kernels.py:230-257 (its numpy reference);
    # the reference test's tolerance is rtol 1e-2, atol 5e-3; the oracle is far tighter.
    d = golden("kat_triton_int4.npz")
    rows, cols, gs = (int(v) for v in d[f"tri_{tag}_shape"])
    y = O.gemv_int4(d[f"tri_{tag}_packed"], d[f"tri_{tag}_scales"], d[f"tri_{tag}_zeros"],
                    d[f"tri_{tag}_x"], rows, cols, gs)
    ref = d[f"tri_{tag}_expected"]
    assert np.max(np.abs(y - ref)) <= 1e-5 * max(1.0, np.max(np.abs(ref)))


def test_gptq_identity_matches_reference_formula():
    # (u - 8) * s == reference dequant of (packed ^ 0x88) with zero points 0.
    packed, scales16 = O.make_w4_gptq(8, 256, 128, seed=3)
    gptq = O.bf16_bits_to_f32(O.dequantize_w4_bf16(packed, scales16, 8, 256, 128))
    ref = O.dequantize_int4(packed ^ 0x88, scales16.astype(np.float32), np.zeros((8, 1), np.uint8),
                            8, 256, 128)
    np.testing.assert_array_equal(gptq, O.bf16_bits_to_f32(O.f32_to_bf16_bits(ref)))


def test_zero_point_semantics_unsigned_and_floor_stride():
    # quant_int4.cu:93-96: zero points unsigned, byte stride floor(G/2) per row.
    rows, cols, gs = 3, 24, 8            # G = 3 groups (odd): stride floor(3/2) = 1
    rng = np.random.default_rng(5)
    packed = rng.integers(0, 256, (rows, cols // 2), dtype=np.uint8)
    scales = rng.uniform(0.1, 1.0, (rows, 3)).astype(np.float32)
    zeros = rng.integers(0, 256, (rows * 2,), dtype=np.uint8)
    out = O.dequantize_int4(packed, scales, zeros, rows, cols, gs)
    for r in range(rows):
        for c in range(cols):
            g = c // gs
            zb = int(zeros[r * 1 + g // 2])
            zp = (zb & 15) if g % 2 == 0 else (zb >> 4)
            p = int(packed[r, c // 2])
            v = (p >> 4) if c & 1 else (p & 15)
            v = v - 16 if v >= 8 else v
            assert out[r, c] == np.float32(np.float32(v - zp) * scales[r, g])


# ----------------------------------------------------------------- FP8 -------
def test_e4m3_encoder_matches_torch_cast_sampled():
    # Independent implementation check: torch's CPU float8_e4m3fn cast (RNE).
    # Within +-448 the saturating and non-saturating encoders agree.
    rng = np.random.default_rng(0)
    bits = rng.integers(0, 2**32, size=2_000_000, dtype=np.uint64).astype(np.uint32)
    x = bits.view(np.float32)
    x = x[np.isfinite(x) & (np.abs(x) <= 448.0)]
    # add edge values: subnormal midpoints, exponent boundaries, ties
    extra = []
    for e in range(-10, 9):
        for m in range(16):
            v = np.ldexp(1 + m / 16.0, e)
            extra += [v, -v, np.nextafter(np.float32(v), np.float32(0)),
                      np.nextafter(np.float32(v), np.float32(1e9))]
    extra += [0.0, -0.0, 448.0, -448.0, 2.0**-9, 2.0**-10, 3 * 2.0**-10, 2.0**-6]
    x = np.concatenate([x, np.array(extra, np.float32)])
    x = x[np.abs(x) <= 448.0]
    mine = O.e4m3_encode(x, clamp=False)
    theirs = torch.from_numpy(x).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    np.testing.assert_array_equal(mine, theirs)


def test_e4m3_saturation_and_nan():
    # clamp fmaxf(-448, fminf(448, v)) then SATFINITE: big -> 0x7E, NaN -> +448.
    x = np.array([1e9, -1e9, np.inf, -np.inf, np.nan, 460.0, 464.0, 447.9, -0.0, 1e-30],
                 np.float32)
    codes = O.e4m3_encode(x, clamp=True)
    assert list(codes) == [0x7E, 0xFE, 0x7E, 0xFE, 0x7E, 0x7E, 0x7E, 0x7E, 0x80, 0x00]


def test_e4m3_decode_table_roundtrip():
    t = O.e4m3_decode_table()
    finite = np.isfinite(t)
    assert (~finite).sum() == 2 and np.isnan(t[0x7F]) and np.isnan(t[0xFF])
    np.testing.assert_array_equal(O.e4m3_encode(t[finite], clamp=False),
                                  np.arange(256, dtype=np.uint8)[finite])


def test_fp8_per_token_reference_tests(golden):
    # tests/test_fp8_quant.cpp:34-71 (rel err < 15%) and :73-97 (zeros -> zeros)
    d = golden("kat_fp8.npz")
    x = d["pt_in"]
    q, s = O.quantize_fp8_per_token(x)
    xh = O.dequantize_fp8(q, s, 8, 64, True)
    nz = np.abs(x) > 1e-6
    assert np.max(np.abs(xh[nz] - x[nz]) / np.abs(x[nz])) < 0.15
    z = np.zeros((4, 32), np.float32)
    qz, sz = O.quantize_fp8_per_token(z)
    assert np.all(sz == 1.0) and np.all(O.dequantize_fp8(qz, sz, 4, 32, True) == 0)
    # binding test src/python/tests/test_transformer_bindings.py:213-221
    xb = golden("kat_bindings.npz")["bind_fp8_in"]
    qb, sb = O.quantize_fp8_per_token(xb)
    xbh = O.dequantize_fp8(qb, sb, *xb.shape, True)
    nzb = np.abs(xb) > 1e-6
    assert np.max(np.abs(xbh[nzb] - xb[nzb]) / np.abs(xb[nzb])) < 0.15


def test_fp8_smoothquant_and_per_tensor_reference_tests(golden):
    d = golden("kat_fp8.npz")
    # tests/test_fp8_quant.cpp:99-135: exact ones
    np.testing.assert_array_equal(O.smoothquant_scale(d["sq_in"], d["sq_smooth"]), d["sq_expected"])
    # :137-174: per-tensor round trip with scale = max_abs / 448
    x, s = d["tensor_in"], float(d["tensor_scale"][0])
    q = O.quantize_fp8_per_tensor(x, s)
    xh = O.dequantize_fp8(q, np.array([s], np.float32), 4, 32, False)
    nz = np.abs(x) > 1e-6
    assert np.max(np.abs(xh[nz] - x[nz]) / np.abs(x[nz])) < 0.15
    assert O.per_tensor_scale(x) == np.float32(s)


def test_fp8_scale_rules():
    x = np.zeros((3, 8), np.float32)
    x[1, 3] = np.nan               # NaN ignored by the fmaxf amax
    x[1, 4] = -2.5
    x[2, :] = -0.0
    q, s = O.quantize_fp8_per_token(x)
    assert s[0] == 1.0 and s[2] == 1.0
    assert s[1] == np.float32(np.float32(2.5) / np.float32(448))
    assert q[1, 3] == 0x7E          # NaN / scale -> NaN -> clamp -> +448
    assert q[1, 4] == 0xFE          # -amax -> -448
    assert np.all(q[2] == 0x80)     # -0.0 keeps its sign


# ------------------------------------------------------- tensor parallel ----
def test_tensor_parallel_kats(golden):
    d = golden("kat_tensor_parallel.npz")
    # col-parallel 2 ranks + host re-interleave (test_tensor_parallel.cpp:209-259)
    x, W = d["col_x"], d["col_W"]
    y0, y1 = O.gemm_nt_f32(x, W[:3]), O.gemm_nt_f32(x, W[3:])
    assert np.max(np.abs(np.concatenate([y0, y1], axis=1) - d["col_ref"])) < 1e-3
    # row-parallel 2 ranks, summed partials (:272-330)
    x, W = d["row_x"], d["row_W"]
    p = O.gemm_nt_f32(x[:, :4], W[:, :4]) + O.gemm_nt_f32(x[:, 4:], W[:, 4:])
    assert np.max(np.abs(p - d["row_ref"])) < 1e-3
    # chain (:339-376)
    mid = O.gemm_nt_f32(d["chain_x"], d["chain_W1"])
    assert np.max(np.abs(O.gemm_nt_f32(mid, d["chain_W2"]) - d["chain_ref"])) < 1e-3
    # simulated collectives (:84-196)
    np.testing.assert_array_equal(O.ring_allreduce(d["ar2_in"]), np.tile(d["ar2_expected"], (2, 1)))
    np.testing.assert_array_equal(O.ring_allreduce(d["ar4_in"]), np.tile(d["ar4_expected"], (4, 1)))
    np.testing.assert_array_equal(O.allgather(d["ag_chunks"]), d["ag_expected"])


def test_ring_allreduce_order_is_reference_order():
    # chunk c accumulates rank c's value first, then ranks 0..R-1 (r != c):
    # fp32 rounding exposes the order.
    R, count = 3, 7
    rng = np.random.default_rng(9)
    b = (rng.standard_normal((R, count)) * 10.0 ** rng.integers(-4, 5, (R, count))).astype(np.float32)
    got = O.ring_allreduce(b)
    chunk = -(-count // R)
    for i in range(count):
        c = i // chunk
        acc = np.float32(b[c, i])
        for r in range(R):
            if r != c:
                acc = np.float32(acc + b[r, i])
        assert np.all(got[:, i] == acc)


# ------------------------------------------- reference-kernel pins (B200) ---
def _ref_fixture(name):
    p = GOLDEN / name
    if not p.exists():
        pytest.skip(f"{name} not generated yet (tests/golden/make_golden_ref.py on a B200)")
    return np.load(p)


def test_oracle_matches_reference_kernels_fp8():
    d = _ref_fixture("ref_fp8.npz")
    for tag in [k[:-3] for k in d.files if k.endswith("_in")]:
        x = d[f"{tag}_in"]
        q, s = O.quantize_fp8_per_token(x)
        np.testing.assert_array_equal(s, d[f"{tag}_scales"])
        np.testing.assert_array_equal(q, d[f"{tag}_codes"].view(np.uint8))
        xh = O.dequantize_fp8(q, s, *x.shape, True)
        ref = d[f"{tag}_dequant"]
        # NaN payloads differ between x86 (0xFFC00000) and the GPU (0x7FFFFFFF):
        # compare the NaN positions, and the bits of everything else.
        nan = np.isnan(ref)
        np.testing.assert_array_equal(np.isnan(xh), nan)
        np.testing.assert_array_equal(xh[~nan].view(np.uint32), ref[~nan].view(np.uint32))


def test_oracle_matches_reference_kernels_int4():
    d = _ref_fixture("ref_int4.npz")
    for tag in [k[:-7] for k in d.files if k.endswith("_packed")]:
        rows, cols, gs = (int(v) for v in d[f"{tag}_shape"])
        out = O.dequantize_int4(d[f"{tag}_packed"], d[f"{tag}_scales"], d[f"{tag}_zeros"],
                                rows, cols, gs)
        np.testing.assert_array_equal(out.view(np.uint32), d[f"{tag}_dequant"].view(np.uint32))
        y = O.gemv_int4(d[f"{tag}_packed"], d[f"{tag}_scales"], d[f"{tag}_zeros"], d[f"{tag}_x"],
                        rows, cols, gs)
        ref = d[f"{tag}_gemv"]
        assert np.max(np.abs(y - ref)) <= 1e-3 * max(1e-6, np.max(np.abs(ref)))

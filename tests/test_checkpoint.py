"""Checkpoint conversion (kernel-craft_b200/checkpoint.py) on CPU.

GPTQ and AWQ tensors are packed by vLLM 0.22.0's own packers
(quant_utils.pack_rows / pack_cols / awq_pack) when vLLM is importable, and by
a restatement of the same packing otherwise; the converted weights must
dequantize (oracle) to exactly the integers and scales that were packed, act
order must come back as the input-channel permutation that makes the groups
contiguous, and the reference-ABI form must dequantize through the
reference's own arithmetic (ora_dequantize_int4, quant_int4.cu:68-105) to the
same fp32 weights.
"""
import numpy as np
import pytest
import torch

import checkpoint as C
import oracle as O


def _inputs(K, N, gs, seed, zero=8):
    rng = np.random.default_rng(seed)
    u = rng.integers(0, 16, (K, N), dtype=np.uint8)
    s = rng.uniform(0.002, 0.02, (K // gs, N)).astype(np.float16)
    z = np.full((K // gs, N), zero, np.uint8) if zero is not None else \
        rng.integers(0, 16, (K // gs, N), dtype=np.uint8)
    return u, s, z


def _dequant_checkpoint(u, s, z, g_of_k):
    """w[n, k] = (u[k, n] - z[g(k), n]) * s[g(k), n], fp32 [N, K]."""
    g = np.asarray(g_of_k)
    return ((u.astype(np.float32) - z[g].astype(np.float32)) * s[g].astype(np.float32)).T


def _dequant_w4a16(w: C.W4A16Weights, gs):
    """The converted weights as the library's kernels read them: (u - z) * s,
    z = 8 when the conversion found no zero points (checked against the
    oracle's dequantization of the same layout)."""
    N, half = w.packed.shape
    u = np.empty((N, 2 * half), np.float32)
    u[:, 0::2] = w.packed & 15
    u[:, 1::2] = w.packed >> 4
    z = 8.0 if w.zeros is None else np.repeat(w.zeros.astype(np.float32), gs, axis=1)
    out = (u - z) * np.repeat(w.scales.astype(np.float32), gs, axis=1)
    bf = O.bf16_bits_to_f32(O.dequantize_w4_bf16(w.packed, w.scales, N, 2 * half, gs, zeros=w.zeros))
    np.testing.assert_array_equal(bf, O.bf16_bits_to_f32(O.f32_to_bf16_bits(out)))
    return out


def _pack_rows(q):            # restated pack_rows: k = 8i + j in bits 4j of word [i, n]
    q = q.astype(np.uint32)
    out = np.zeros((q.shape[0] // 8, q.shape[1]), np.uint32)
    for j in range(8):
        out |= q[j::8] << (4 * j)
    return out.astype(np.int32)


def _pack_cols(q, interleave=None):   # restated pack_cols / awq_pack
    q = q.astype(np.uint32)
    if interleave is not None:
        q = q.reshape(-1, 8)[:, interleave].reshape(q.shape)
    out = np.zeros((q.shape[0], q.shape[1] // 8), np.uint32)
    for j in range(8):
        out |= q[:, j::8] << (4 * j)
    return out.astype(np.int32)


@pytest.fixture(scope="module")
def packers():
    """(pack_rows, pack_cols, awq_pack) of vLLM when importable, else restated."""
    try:
        from vllm.model_executor.layers.quantization.utils import quant_utils as q
    except Exception:                                   # vLLM absent or unusable here
        return (lambda a: _pack_rows(a), lambda a: _pack_cols(a),
                lambda a: _pack_cols(a, [0, 2, 4, 6, 1, 3, 5, 7]), "restated")
    t = lambda a: torch.from_numpy(a.astype(np.int32))
    return (lambda a: q.pack_rows(t(a), 4, *a.shape).numpy(),
            lambda a: q.pack_cols(t(a), 4, *a.shape).numpy(),
            lambda a: q.awq_pack(t(a), 4, *a.shape).numpy(), "vllm")


def test_restated_packers_match_vllm(packers):
    if packers[3] != "vllm":
        pytest.skip("vLLM not importable")
    u, _, z = _inputs(256, 64, 128, seed=1, zero=None)
    np.testing.assert_array_equal(packers[0](u), _pack_rows(u))
    np.testing.assert_array_equal(packers[1](z), _pack_cols(z))
    np.testing.assert_array_equal(packers[2](u), _pack_cols(u, [0, 2, 4, 6, 1, 3, 5, 7]))


@pytest.mark.parametrize("fmt", ["gptq", "gptq_v2"])
@pytest.mark.parametrize("K,N,gs", [(256, 64, 128), (512, 40, 64), (384, 16, 128)])
def test_gptq(packers, fmt, K, N, gs):
    pack_rows, pack_cols = packers[0], packers[1]
    u, s, z = _inputs(K, N, gs, seed=K + N)
    stored_z = (z.astype(np.int32) - (1 if fmt == "gptq" else 0)) & 0xF
    w = C.from_gptq(pack_rows(u), pack_cols(stored_z), s, group_size=gs, checkpoint_format=fmt)
    assert w.perm is None and w.packed.shape == (N, K // 2) and w.scales.shape == (N, K // gs)
    np.testing.assert_array_equal(_dequant_w4a16(w, gs), _dequant_checkpoint(u, s, z, np.arange(K) // gs))
    # the oracle's bf16 dequantization of the converted weights (the kernels' weights)
    want = O.f32_to_bf16_bits(_dequant_checkpoint(u, s, z, np.arange(K) // gs))
    np.testing.assert_array_equal(O.dequantize_w4_bf16(w.packed, w.scales, N, K, gs), want)


def test_gptq_act_order(packers):
    K, N, gs = 512, 32, 128
    u, s, z = _inputs(K, N, gs, seed=3)
    g_idx = np.random.default_rng(4).permutation(np.arange(K) // gs).astype(np.int32)
    w = C.from_gptq(packers[0](u), packers[1]((z - 1) & 0xF), s, g_idx=torch.from_numpy(g_idx),
                    group_size=gs)
    assert w.perm is not None and sorted(w.perm.tolist()) == list(range(K))
    assert np.all(np.diff(g_idx[w.perm]) >= 0)          # groups contiguous after the permutation
    ref = _dequant_checkpoint(u, s, z, g_idx)            # [N, K] in checkpoint order
    np.testing.assert_array_equal(_dequant_w4a16(w, gs), ref[:, w.perm])
    # y = W x with the kernels' layout and x[:, perm]
    x = O.make_activations_bf16(3, K, seed=5)
    y = O.gemv_w4a16(w.packed, w.scales, np.ascontiguousarray(x[:, w.perm]), 3, N, K, gs)
    y_ref = O.bf16_bits_to_f32(x).astype(np.float64) @ ref.T.astype(np.float64)
    assert np.max(np.abs(y - y_ref)) / np.max(np.abs(y_ref)) <= 1e-5


def test_gptq_bad_g_idx(packers):
    K, N, gs = 256, 16, 128
    u, s, z = _inputs(K, N, gs, seed=6)
    g_idx = np.zeros(K, np.int32)                        # every channel in group 0
    with pytest.raises(ValueError):
        C.from_gptq(packers[0](u), packers[1]((z - 1) & 0xF), s, g_idx=g_idx, group_size=gs)


@pytest.mark.parametrize("K,N,gs", [(256, 64, 128), (512, 24, 64)])
def test_awq(packers, K, N, gs):
    u, s, z = _inputs(K, N, gs, seed=K - N)
    w = C.from_awq(packers[2](u), packers[2](z), s, group_size=gs)
    np.testing.assert_array_equal(_dequant_w4a16(w, gs), _dequant_checkpoint(u, s, z, np.arange(K) // gs))


@pytest.mark.parametrize("K,N,gs", [(256, 32, 128), (384, 24, 128), (512, 16, 64)])
def test_asymmetric_zero_points_convert(packers, K, N, gs):
    """AWQ and asymmetric GPTQ: the zero points come along, u8 [N, K/gs], and
    the converted weights dequantize to exactly (q - z) * s."""
    u, s, z = _inputs(K, N, gs, seed=7 + K, zero=None)
    g = np.arange(K) // gs
    w = C.from_gptq(packers[0](u), packers[1](z), s, group_size=gs, checkpoint_format="gptq_v2")
    assert w.zeros is not None and w.zeros.shape == (N, K // gs) and w.zeros.dtype == np.uint8
    np.testing.assert_array_equal(_dequant_w4a16(w, gs), _dequant_checkpoint(u, s, z, g))
    w1 = C.from_gptq(packers[0](u), packers[1]((z - 1) & 0xF), s, group_size=gs)   # stored z - 1
    np.testing.assert_array_equal(w1.zeros, w.zeros)
    a = C.from_awq(packers[2](u), packers[2](z), s, group_size=gs)
    np.testing.assert_array_equal(_dequant_w4a16(a, gs), _dequant_checkpoint(u, s, z, g))


def test_asymmetric_act_order(packers):
    K, N, gs = 512, 16, 128
    u, s, z = _inputs(K, N, gs, seed=11, zero=None)
    g_idx = np.random.default_rng(12).permutation(np.arange(K) // gs)
    w = C.from_gptq(packers[0](u), packers[1](z), s, g_idx=g_idx, group_size=gs,
                    checkpoint_format="gptq_v2")
    got = _dequant_w4a16(w, gs)
    want = _dequant_checkpoint(u, s, z, g_idx)          # [N, K] in the checkpoint's k order
    np.testing.assert_array_equal(got, want[:, w.perm])


def test_reference_abi_zero_points():
    """Zero points >= 8 map onto the reference's zp = z - 8; below 8 refused."""
    K, N, gs = 512, 8, 128
    rng = np.random.default_rng(5)
    u = rng.integers(0, 16, (K, N), dtype=np.uint8)
    s = rng.uniform(0.002, 0.02, (K // gs, N)).astype(np.float16)
    z = rng.integers(8, 16, (K // gs, N), dtype=np.uint8)
    w = C.W4A16Weights(C._pack_w4(u), np.ascontiguousarray(s.T), None, np.ascontiguousarray(z.T))
    packed, scales32, zeros = C.to_reference_abi(w, gs)
    got = O.dequantize_int4(packed, scales32, zeros, N, K, gs)
    np.testing.assert_array_equal(got, _dequant_checkpoint(u, s, z, np.arange(K) // gs))
    low = w._replace(zeros=np.full((N, K // gs), 3, np.uint8))
    with pytest.raises(ValueError, match="below 8"):
        C.to_reference_abi(low, gs)


@pytest.mark.parametrize("K,gs", [(512, 128), (384, 128), (128, 128)])   # 4, 3 (odd) and 1 group
def test_reference_abi_form(packers, K, gs):
    N = 24
    u, s, z = _inputs(K, N, gs, seed=K)
    w = C.from_gptq(packers[0](u), packers[1](z), s, group_size=gs, checkpoint_format="gptq_v2")
    packed, scales32, zeros = C.to_reference_abi(w, gs)
    got = O.dequantize_int4(packed, scales32, zeros, N, K, gs)
    np.testing.assert_array_equal(got, _dequant_checkpoint(u, s, z, np.arange(K) // gs))


def test_archive_round_trip(packers, tmp_path):
    """checkpoint.save / load: converted layers (symmetric, asymmetric, act
    order) come back bit for bit, with the group size."""
    K, N, gs = 512, 24, 128
    u, s, z = _inputs(K, N, gs, seed=41, zero=None)
    g_idx = np.random.default_rng(42).permutation(np.arange(K) // gs)
    layers = {
        "qkv": C.from_gptq(packers[0](u), packers[1](np.full_like(z, 8)), s, group_size=gs,
                           checkpoint_format="gptq_v2"),
        "o": C.from_awq(packers[2](u), packers[2](z), s, group_size=gs),
        "down": C.from_gptq(packers[0](u), packers[1](z), s, g_idx=g_idx, group_size=gs,
                            checkpoint_format="gptq_v2"),
    }
    path = tmp_path / "model.npz"
    C.save(path, layers, gs)
    back, g = C.load(path)
    assert g == gs and sorted(back) == sorted(layers)
    for name, w in layers.items():
        b = back[name]
        np.testing.assert_array_equal(b.packed, w.packed)
        np.testing.assert_array_equal(b.scales.view(np.uint16), w.scales.view(np.uint16))
        for part in ("perm", "zeros"):
            x, y = getattr(w, part), getattr(b, part)
            assert (x is None) == (y is None)
            if x is not None:
                np.testing.assert_array_equal(x, y)


def test_archive_rejects_bad_layers(tmp_path):
    K, N, gs = 256, 8, 128
    good = C.W4A16Weights(np.zeros((N, K // 2), np.uint8), np.ones((N, K // gs), np.float16), None)
    with pytest.raises(ValueError, match="scales"):
        C.save(tmp_path / "a.npz", {"l": good._replace(scales=np.ones((N, 3), np.float16))}, gs)
    with pytest.raises(ValueError, match="zeros"):
        C.save(tmp_path / "b.npz", {"l": good._replace(zeros=np.full((N, K // gs), 16, np.uint8))}, gs)
    with pytest.raises(ValueError, match="'.'"):
        C.save(tmp_path / "c.npz", {"a.b": good}, gs)
    np.savez(tmp_path / "d.npz", x=np.zeros(3))
    with pytest.raises(ValueError, match="not a W4A16 weight archive"):
        C.load(tmp_path / "d.npz")


def test_tile_w4_layout():
    """checkpoint.tile_w4: chunk (tile t, k-chunk c) is the 1 KB at
    (t * K/128 + c) * 1024, its row r the 64 bytes packed[16 t + r, 64 c:64 c + 64],
    rows past N zero."""
    rng = np.random.default_rng(3)
    N, K = 40, 512
    p = rng.integers(0, 256, (N, K // 2), dtype=np.uint8)
    t = C.tile_w4(p)
    C_ = K // 128
    assert t.shape == (48 * K // 2,)
    for tile in range(3):
        for c in range(C_):
            blk = t[(tile * C_ + c) * 1024:(tile * C_ + c + 1) * 1024].reshape(16, 64)
            for r in range(16):
                row = tile * 16 + r
                want = p[row, 64 * c:64 * c + 64] if row < N else np.zeros(64, np.uint8)
                np.testing.assert_array_equal(blk[r], want)
    with pytest.raises(ValueError):
        C.tile_w4(p[:, :100])

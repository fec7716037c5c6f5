"""checkpoint -- GPTQ / AWQ checkpoint tensors -> this library's INT4 weight layouts.

Host-side (numpy), run once when weights are loaded.  The reference has no
loader: its kernels take a W4 matrix W [N, K] (N output channels) as packed
bytes [N, K/2] with the low nibble holding the even k (quant_int4.cu:34-48),
and this library's W4A16 GEMV / GEMM read that layout with fp16 scales
[N, K/gs] and the implicit zero point 8 (w = (u - 8) * s).  Checkpoints store
the same integers in other layouts:

* GPTQ (AutoGPTQ "gptq" and "gptq_v2" formats): qweight int32 [K/8, N], input
  channel k = 8*i + j in bits 4j..4j+3 of qweight[i, n]; qzeros int32
  [K/gs, N/8], output channel n = 8*c + j in bits 4j.. of qzeros[g, c], stored
  as z - 1 in the "gptq" format and as z in "gptq_v2"; scales fp16 [K/gs, N];
  g_idx int32 [K] the group of input channel k (act order, "desc_act",
  assigns groups out of k order).
* AWQ: qweight int32 [K, N/8] and qzeros int32 [K/gs, N/8], output channel
  n = 8*c + j in bits 4*p.. with p = (0, 4, 1, 5, 2, 6, 3, 7)[j] (the packing
  interleave (0, 2, 4, 6, 1, 3, 5, 7)); scales fp16 [K/gs, N];
  w = (q - z) * s.

These are the layouts vLLM 0.22.0 packs and unpacks
(vllm/model_executor/layers/quantization/utils/quant_utils.py: pack_rows,
pack_cols, awq_pack; awq_triton.py's reverse order), which the tests use as
the independent packer.

Symmetric checkpoints (every zero point 8) convert to packed weights and
scales alone, for the kernels' (u - 8) * s.  Others (AWQ usually,
asymmetric GPTQ) convert with their zero points as well, u8 [N, K/gs] one
per byte, for the kc_*_zp entry points ((u - z) * s).  Act-order checkpoints convert
with a permutation of the input channels that makes every group contiguous:
the kernels then take x[:, perm] instead of x (a gather, or folded into the
producer of x).
"""
from __future__ import annotations

from typing import Dict, NamedTuple, Optional, Tuple

import numpy as np

_AWQ_SHIFT_OF_COL = np.array([0, 4, 1, 5, 2, 6, 3, 7])   # nibble position of column j of a word


class W4A16Weights(NamedTuple):
    packed: np.ndarray             # u8 [N, K/2], low nibble = even k
    scales: np.ndarray             # fp16 [N, K/gs]
    perm: Optional[np.ndarray]     # int64 [K]: the kernels take x[:, perm]; None = identity
    zeros: Optional[np.ndarray] = None   # u8 [N, K/gs] zero points 0..15; None = all 8


def _np(a) -> np.ndarray:
    """numpy view of an array or a (CPU or CUDA) torch tensor."""
    if hasattr(a, "detach"):
        a = a.detach().cpu().numpy()
    return np.asarray(a)


def _nibbles_rows(q: np.ndarray) -> np.ndarray:
    """int32 [R, C] holding 8 nibbles per word along the rows -> u8 [8R, C]."""
    w = q.astype(np.uint32)
    out = np.empty((w.shape[0] * 8, w.shape[1]), np.uint8)
    for j in range(8):
        out[j::8] = (w >> (4 * j)) & 0xF
    return out


def _nibbles_cols(q: np.ndarray, shift_of_col=None) -> np.ndarray:
    """int32 [R, C] holding 8 nibbles per word along the columns -> u8 [R, 8C];
    column 8c + j sits at nibble position shift_of_col[j] (default j)."""
    w = q.astype(np.uint32)
    out = np.empty((w.shape[0], w.shape[1] * 8), np.uint8)
    for j in range(8):
        p = j if shift_of_col is None else int(shift_of_col[j])
        out[:, j::8] = (w >> (4 * p)) & 0xF
    return out


def _pack_w4(u_kn: np.ndarray) -> np.ndarray:
    """u8 [K, N] integers 0..15 -> the library's packed u8 [N, K/2]."""
    u = u_kn.T
    return np.ascontiguousarray(u[:, 0::2] | (u[:, 1::2] << 4)).astype(np.uint8)


def _zero_points(z_gn: np.ndarray) -> Optional[np.ndarray]:
    """Zero points [K/gs, N] -> None when every one is 8 (the symmetric kernels
    need none), else u8 [N, K/gs] for the zero-point entry points."""
    if np.all(z_gn == 8):
        return None
    return np.ascontiguousarray(z_gn.T).astype(np.uint8)


def _group_order(g_idx: np.ndarray, K: int, group_size: int) -> Optional[np.ndarray]:
    """None when g_idx is the plain k // group_size, else the stable order of
    the input channels by group (each group then holds group_size consecutive
    channels)."""
    g = _np(g_idx).astype(np.int64).reshape(-1)
    if g.shape[0] != K:
        raise ValueError(f"g_idx has {g.shape[0]} entries for K = {K}")
    if np.array_equal(g, np.arange(K) // group_size):
        return None
    counts = np.bincount(g, minlength=K // group_size)
    if counts.shape[0] != K // group_size or np.any(counts != group_size):
        raise ValueError("g_idx must assign exactly group_size input channels to every group")
    return np.argsort(g, kind="stable")


def from_gptq(qweight, qzeros, scales, g_idx=None, group_size: int = 128,
              checkpoint_format: str = "gptq") -> W4A16Weights:
    """GPTQ tensors (qweight int32 [K/8, N], qzeros int32 [K/gs, N/8], scales
    fp16 [K/gs, N], optional g_idx [K]) -> the W4A16 layout.
    checkpoint_format "gptq" stores zero points minus one, "gptq_v2" as is."""
    if checkpoint_format not in ("gptq", "gptq_v2"):
        raise ValueError("checkpoint_format must be 'gptq' or 'gptq_v2'")
    qw, qz, s = _np(qweight), _np(qzeros), _np(scales)
    u = _nibbles_rows(qw)                                  # [K, N]
    K, N = u.shape
    if K % group_size or s.shape != (K // group_size, N):
        raise ValueError(f"scales {s.shape} do not match K={K}, N={N}, group_size={group_size}")
    z = _nibbles_cols(qz)[:, :N].astype(np.int32)          # [K/gs, N]
    if checkpoint_format == "gptq":
        z = (z + 1) & 0xF
    perm = None if g_idx is None else _group_order(g_idx, K, group_size)
    if perm is not None:
        u = u[perm]
    # after the permutation, block g of the channels is group g: zero points
    # and scales stay indexed by group
    return W4A16Weights(_pack_w4(u), np.ascontiguousarray(s.T).astype(np.float16), perm,
                        _zero_points(z))


def from_awq(qweight, qzeros, scales, group_size: int = 128) -> W4A16Weights:
    """AWQ tensors (qweight int32 [K, N/8], qzeros int32 [K/gs, N/8], scales
    fp16 [K/gs, N]) -> the W4A16 layout."""
    qw, qz, s = _np(qweight), _np(qzeros), _np(scales)
    u = _nibbles_cols(qw, _AWQ_SHIFT_OF_COL)               # [K, N]
    K, N = u.shape
    if K % group_size or s.shape != (K // group_size, N):
        raise ValueError(f"scales {s.shape} do not match K={K}, N={N}, group_size={group_size}")
    z = _nibbles_cols(qz, _AWQ_SHIFT_OF_COL)[:, :N]
    return W4A16Weights(_pack_w4(u), np.ascontiguousarray(s.T).astype(np.float16), None,
                        _zero_points(z))


def to_reference_abi(w: W4A16Weights, group_size: int = 128) -> Tuple[np.ndarray, np.ndarray, np.ndarray]:
    """The same weights for the reference ABI (launch_dequantize_int4 /
    launch_gemv_int4, quant_int4.cu:68-105): weight nibbles as sign-extended
    two's complement (sx4(u ^ 8) = u - 8, so packed ^ 0x88), fp32 scales
    [N, K/gs], and zero points 0 in the row stride the reference kernel reads,
    floor(K/gs/2) bytes (quant_int4.cu:93; its tests allocate the ceiling,
    test_quant_int4.cpp:56, which only differs for an odd group count, where
    all-zero points read the same either way).  One trailing byte keeps the
    last row's odd group inside the buffer.

    Zero points z other than 8 become the reference's zp = z - 8 (its weight
    (sx4(u ^ 8) - zp) * s = (u - z) * s); the reference reads zero points
    unsigned, so z < 8 cannot be represented and raises ValueError."""
    packed = np.ascontiguousarray(w.packed ^ np.uint8(0x88))
    N, G = w.scales.shape
    zeros = np.zeros(N * (G // 2) + 1, np.uint8)
    if w.zeros is not None:
        z = w.zeros.astype(np.int32)
        if np.any(z < 8):
            raise ValueError(f"{int(np.count_nonzero(z < 8))} zero points are below 8: the reference "
                             "ABI reads zero points unsigned after sign-extending the weights "
                             "(quant_int4.cu:34-38, 93-96) and cannot represent them")
        zp = (z - 8).astype(np.uint8)                       # [N, G]
        stride = G // 2
        body = zp[:, 0:2 * stride:2] | (zp[:, 1:2 * stride:2] << 4)   # [N, stride]
        zeros[:N * stride] = body.reshape(-1)
        if G % 2:
            # the reference reads row r's last (even-indexed) group from the low
            # nibble of byte r*stride + stride, which is row r+1's first byte:
            # representable only when the two zero points agree
            last, first_next = zp[:-1, G - 1], zp[1:, 0]
            if np.any(last != first_next):
                raise ValueError("odd group count: the reference's floor zero-point stride "
                                 "(quant_int4.cu:93) makes row r's last group share a nibble with "
                                 "row r+1's first; these zero points differ there")
            zeros[N * stride] = zp[N - 1, G - 1]
    return packed, w.scales.astype(np.float32), zeros


def tile_w4(packed: np.ndarray) -> np.ndarray:
    """packed u8 [N, K/2] -> the tile-ordered layout the W4A16 GEMV streams
    fastest (kc_w4a16_tile_weights does the same on the GPU): every 16-row x
    128-k chunk contiguous, [ceil(N/16)][K/128][16 rows][64 bytes], rows past
    N zero.  K must be a multiple of 128."""
    p = np.asarray(packed)
    N, half = p.shape
    if p.dtype != np.uint8 or half % 64:
        raise ValueError("packed must be u8 [N, K/2] with K a multiple of 128")
    Np = (N + 15) // 16 * 16
    pad = np.zeros((Np, half), np.uint8)
    pad[:N] = p
    return pad.reshape(Np // 16, 16, half // 64, 64).transpose(0, 2, 1, 3).reshape(-1).copy()


# ---------------------------------------------------------------------------
# On-disk form of converted weights
# ---------------------------------------------------------------------------
# One .npz archive per model: for every layer name the arrays "<name>.packed"
# (u8 [N, K/2]), "<name>.scales" (fp16 [N, K/gs]) and, where present,
# "<name>.perm" (int64 [K]) and "<name>.zeros" (u8 [N, K/gs]); plus
# "__kc_w4a16__" = [format version, group size].  The arrays are stored
# exactly as the kernels read them, so loading is a file read and a copy to
# the device -- no conversion at start-up.

FORMAT_VERSION = 1
_HEADER = "__kc_w4a16__"


def _check_layer(name: str, w: W4A16Weights, group_size: int) -> None:
    p, s = np.asarray(w.packed), np.asarray(w.scales)
    if p.dtype != np.uint8 or p.ndim != 2:
        raise ValueError(f"{name}: packed must be u8 [N, K/2], got {p.dtype} {p.shape}")
    N, K = p.shape[0], 2 * p.shape[1]
    if K % group_size:
        raise ValueError(f"{name}: K={K} is not a multiple of the group size {group_size}")
    if s.dtype != np.float16 or s.shape != (N, K // group_size):
        raise ValueError(f"{name}: scales must be fp16 [{N}, {K // group_size}], got {s.dtype} {s.shape}")
    if w.perm is not None:
        perm = np.asarray(w.perm)
        if perm.shape != (K,) or not np.array_equal(np.sort(perm), np.arange(K)):
            raise ValueError(f"{name}: perm must be a permutation of {K} input channels")
    if w.zeros is not None:
        z = np.asarray(w.zeros)
        if z.dtype != np.uint8 or z.shape != (N, K // group_size) or np.any(z > 15):
            raise ValueError(f"{name}: zeros must be u8 [{N}, {K // group_size}] in 0..15")


def save(path, layers: Dict[str, W4A16Weights], group_size: int = 128) -> None:
    """Write converted layers (name -> W4A16Weights) to one .npz archive."""
    arrays = {_HEADER: np.array([FORMAT_VERSION, group_size], np.int64)}
    for name, w in layers.items():
        if "." in name or name == _HEADER:
            raise ValueError(f"layer name {name!r} must not contain '.'")
        _check_layer(name, w, group_size)
        arrays[f"{name}.packed"] = np.ascontiguousarray(w.packed)
        arrays[f"{name}.scales"] = np.ascontiguousarray(w.scales)
        if w.perm is not None:
            arrays[f"{name}.perm"] = np.asarray(w.perm, np.int64)
        if w.zeros is not None:
            arrays[f"{name}.zeros"] = np.ascontiguousarray(w.zeros)
    np.savez(path, **arrays)


def load(path) -> Tuple[Dict[str, W4A16Weights], int]:
    """Read an archive written by save(): (name -> W4A16Weights, group size).
    Every layer is checked against the layout the kernels expect."""
    with np.load(path, allow_pickle=False) as f:
        if _HEADER not in f.files:
            raise ValueError(f"{path}: not a W4A16 weight archive (no {_HEADER} entry)")
        version, group_size = (int(v) for v in f[_HEADER])
        if version != FORMAT_VERSION:
            raise ValueError(f"{path}: format version {version}, this library reads {FORMAT_VERSION}")
        names = sorted({k.split(".")[0] for k in f.files if k != _HEADER})
        layers = {}
        for name in names:
            get = lambda part: f[f"{name}.{part}"] if f"{name}.{part}" in f.files else None
            if get("packed") is None or get("scales") is None:
                raise ValueError(f"{path}: layer {name!r} lacks packed weights or scales")
            w = W4A16Weights(get("packed"), get("scales"), get("perm"), get("zeros"))
            _check_layer(name, w, group_size)
            layers[name] = w
    return layers, group_size

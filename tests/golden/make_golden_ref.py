"""Generates tests/golden/ref_*.npz by running the reference's own CUDA kernels
(oracle/_ref/libkcref.so, built from the reference sources by oracle/build_ref.sh)
on a GPU, on seeded inputs.  These fixtures pin the oracle bit-exactly where
the reference's own tests only check tolerances (E4M3 codes, scales,
dequantized weights for nonzero and odd-count zero points).

    python tests/golden/make_golden_ref.py [out_dir]     # needs a CUDA device

Inputs respect the reference kernels' preconditions: per-token rows whose
length is a multiple of 32 (its warp reduction uses full-warp shuffles,
fp8_quant.cu:43-44,211) and zero-point buffers of ceil(G/2) bytes per row, as
its tests allocate (test_quant_int4.cpp:56).
"""
import sys
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT / "oracle"))
import kcref  # noqa: E402
import oracle as O  # noqa: E402


def to_dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def fp8_cases():
    out = {}
    rng = np.random.default_rng(123)
    edge = rng.standard_normal((16, 1024)).astype(np.float32)
    edge *= (10.0 ** rng.integers(-4, 5, (16, 1))).astype(np.float32)
    edge[1] = 0.0
    edge[2, :13] = [np.nan, np.inf, -np.inf, -0.0, 0.0, 1e-40, -1e-40, 3.4e38, 448.0, 464.0,
                    -464.0, 2.0**-10, 1.5 * 2.0**-9]
    edge[3] = -0.0
    edge[4] = np.float32(2.0**-9) * rng.integers(-64, 64, 1024).astype(np.float32) * 0.37
    cases = {
        "edge": edge,
        "outlier": O.make_outlier_activations(8192, 8192, seed=0)[:16].copy(),
        "weight": O.make_weight_f32(16, 4096, seed=2),
        "uniform": rng.uniform(-1, 1, (8, 64)).astype(np.float32),
    }
    for tag, x in cases.items():
        q, s = kcref.quantize_fp8(to_dev(x), True)
        xh = kcref.dequantize_fp8(q, s, *x.shape, True)
        torch.cuda.synchronize()
        out[f"{tag}_in"] = x
        out[f"{tag}_codes"] = q.cpu().numpy()
        out[f"{tag}_scales"] = s.cpu().numpy()
        out[f"{tag}_dequant"] = xh.cpu().numpy()
    return out


def int4_cases():
    out = {}
    for tag, (rows, cols, gs, zmode) in {"z0": (32, 512, 128, "zero"), "z88": (16, 1024, 128, "eight"),
                                         "zrand": (24, 768, 64, "random"),
                                         "oddG": (8, 24, 8, "random"), "gs32": (8, 256, 32, "random")}.items():
        rng = np.random.default_rng(rows * cols + gs)
        G = cols // gs
        zc = -(-G // 2)
        packed = rng.integers(0, 256, (rows, cols // 2), dtype=np.uint8)
        scales = rng.uniform(0.002, 0.02, (rows, G)).astype(np.float32)
        zeros = {"zero": np.zeros((rows, zc), np.uint8), "eight": np.full((rows, zc), 0x88, np.uint8),
                 "random": rng.integers(0, 256, (rows, zc), dtype=np.uint8)}[zmode]
        x = rng.standard_normal(cols).astype(np.float32)
        dp, ds, dz, dx = to_dev(packed), to_dev(scales), to_dev(zeros), to_dev(x)
        deq = kcref.dequantize_int4(dp, ds, dz, rows, cols, gs)
        y = kcref.gemv_int4(dp, ds, dz, dx, rows, cols, gs)
        torch.cuda.synchronize()
        out.update({f"{tag}_packed": packed, f"{tag}_scales": scales, f"{tag}_zeros": zeros,
                    f"{tag}_x": x, f"{tag}_dequant": deq.cpu().numpy(), f"{tag}_gemv": y.cpu().numpy(),
                    f"{tag}_shape": np.array([rows, cols, gs], np.int32)})
    return out


def main():
    if not torch.cuda.is_available() or not kcref.available():
        print("needs a CUDA device and oracle/_ref/libkcref.so", file=sys.stderr)
        return 1
    out_dir = Path(sys.argv[1]) if len(sys.argv) > 1 else ROOT / "tests" / "golden"
    out_dir.mkdir(parents=True, exist_ok=True)
    np.savez_compressed(out_dir / "ref_fp8.npz", **fp8_cases())
    np.savez_compressed(out_dir / "ref_int4.npz", **int4_cases())
    print("wrote", out_dir / "ref_fp8.npz", out_dir / "ref_int4.npz")
    return 0


if __name__ == "__main__":
    sys.exit(main())

"""Host-side tensor-parallel logic on CPU: two gloo ranks shard the oracle's
W4A16 and FP8 GEMMs the way kernel-craft_b200/tp.py shards the CUDA ones, and
the gathered / reduced results must equal the unsharded oracle (column
parallel bit for bit: every output column is computed by exactly one rank with
the same arithmetic; row parallel within fp32 summation-order noise: the
reference's launch_row_parallel_linear + all-reduce, tensor_parallel.cu:235,
adds the rank partials in another order than one full-K sum)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle as O
from tp import shard_range

M, N, K, GS = 24, 256, 512, 128


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs():
    packed, scales = O.make_w4_gptq(N, K, GS, seed=7)
    x = O.make_activations_bf16(M, K, seed=8)
    xa = O.make_outlier_activations(M, K, seed=9)
    w = O.make_weight_f32(N, K, seed=10)
    qa, sa = O.quantize_fp8_per_token(xa)
    qw, sw = O.quantize_fp8_per_token(w)
    return packed, scales, x, qa, sa, qw, sw


def _rank_main(rank, world, port, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        packed, scales, x, qa, sa, qw, sw = _inputs()
        # column parallel: this rank's weight rows, then all-gather along N
        n0, n1 = shard_range(N, world, rank)
        y_shard = O.gemm_w4a16(x, packed[n0:n1], scales[n0:n1], M, n1 - n0, K, GS)
        parts = [torch.empty(M, n1 - n0) for _ in range(world)]
        dist.all_gather(parts, torch.from_numpy(np.ascontiguousarray(y_shard)))
        col = torch.cat(parts, dim=1).numpy()
        # row parallel: this rank's K columns of both code matrices, full-row scales
        k0, k1 = shard_range(K, world, rank)
        part = torch.from_numpy(O.gemm_fp8_rowcol(np.ascontiguousarray(qa[:, k0:k1]), sa,
                                                  np.ascontiguousarray(qw[:, k0:k1]), sw))
        dist.all_reduce(part)
        if rank == 0:
            np.save(os.path.join(out_dir, "col.npy"), col)
            np.save(os.path.join(out_dir, "row.npy"), part.numpy())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2])
def test_sharded_oracle_matches_unsharded(tmp_path, world):
    mp.spawn(_rank_main, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    packed, scales, x, qa, sa, qw, sw = _inputs()
    np.testing.assert_array_equal(np.load(tmp_path / "col.npy"),
                                  O.gemm_w4a16(x, packed, scales, M, N, K, GS))
    full = O.gemm_fp8_rowcol(qa, sa, qw, sw)
    row = np.load(tmp_path / "row.npy")
    assert np.max(np.abs(row - full)) / np.max(np.abs(full)) <= 1e-6


def test_shard_range():
    assert shard_range(28672, 8, 0) == (0, 3584)
    assert shard_range(28672, 8, 7) == (25088, 28672)
    with pytest.raises(ValueError):
        shard_range(100, 3, 0)
    with pytest.raises(ValueError):
        shard_range(100, 2, 2)

"""Host-side tensor-parallel logic on CPU: two gloo ranks shard the oracle's
W4A16 and FP8 GEMMs the way kernel-craft_b200/tp.py shards the CUDA ones, and
the gathered / reduced results must equal the unsharded oracle (column
parallel bit for bit: every output column is computed by exactly one rank with
the same arithmetic; row parallel within fp32 summation-order noise: the
reference's launch_row_parallel_linear + all-reduce, tensor_parallel.cu:235,
adds the rank partials in another order than one full-K sum).  The MLP block
(the reference's col-parallel -> GELU -> row-parallel chain,
examples/python/transformer/tensor_parallel.py:150-172) is sharded the way
tp.MLPBlockW4A16 shards it: W1 by rows, W2 by the same columns, one
all-reduce."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle as O
from tp import shard_range, shard_w4_cols, shard_w4_rows

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


MH, MI = 256, 512      # MLP block: hidden H, intermediate I


def _mlp_inputs():
    w1p, w1s = O.make_w4_gptq(MI, MH, GS, seed=21)     # W1 [I, H]
    w2p, w2s = O.make_w4_gptq(MH, MI, GS, seed=22)     # W2 [H, I]
    x = O.make_activations_bf16(M, MH, seed=23)
    return w1p, w1s, w2p, w2s, x


def _mlp_rank_main(rank, world, port, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        w1p, w1s, w2p, w2s, x = _mlp_inputs()
        p1, s1 = shard_w4_rows(torch.from_numpy(w1p), torch.from_numpy(w1s.view(np.uint16)), world, rank)
        p2, s2 = shard_w4_cols(torch.from_numpy(w2p), torch.from_numpy(w2s.view(np.uint16)), GS, world,
                               rank)
        ir = MI // world
        h = O.gelu_quick(O.gemm_w4a16(x, p1.numpy(), s1.numpy().view(np.float16), M, ir, MH, GS))
        part = torch.from_numpy(O.gemm_w4a16(O.f32_to_bf16_bits(h), p2.numpy(),
                                             s2.numpy().view(np.float16), M, MH, ir, GS))
        dist.all_reduce(part)
        if rank == 0:
            np.save(os.path.join(out_dir, "mlp.npy"), part.numpy())
    finally:
        dist.destroy_process_group()


def test_sharded_mlp_block_matches_unsharded(tmp_path):
    world = 2
    mp.spawn(_mlp_rank_main, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    w1p, w1s, w2p, w2s, x = _mlp_inputs()
    full = O.mlp_block_w4a16(x, w1p, w1s, w2p, w2s, M, MH, MI, GS)
    got = np.load(tmp_path / "mlp.npy")
    assert np.max(np.abs(got - full)) / np.max(np.abs(full)) <= 1e-6


def test_w4_shard_helpers():
    packed = torch.arange(8 * 128, dtype=torch.int32).reshape(8, 128).to(torch.uint8)
    scales = torch.arange(8 * 4, dtype=torch.int16).reshape(8, 4)     # K = 256, gs = 64
    p, s = shard_w4_rows(packed, scales, 2, 1)
    assert torch.equal(p, packed[4:]) and torch.equal(s, scales[4:])
    p, s = shard_w4_cols(packed, scales, 64, 2, 1)
    assert torch.equal(p, packed[:, 64:]) and torch.equal(s, scales[:, 2:])
    assert p.is_contiguous() and s.is_contiguous()
    assert shard_w4_cols(packed, scales, 64, 4, 3)[1].shape == (8, 1)   # K shard 64: one group
    with pytest.raises(ValueError):
        shard_w4_cols(packed, scales, 64, 8, 0)      # K shard 32 would split a scale group


def test_driver_operand_checks():
    """The tensor-parallel drivers refuse mismatched shards on the host (the
    kernels would read them out of bounds); shown with CPU tensors, cuda=False."""
    import tp
    M, H, I, gs = 8, 256, 512, 128
    x = torch.zeros(M, H, dtype=torch.bfloat16)
    ok = dict(w1_packed=torch.zeros(I, H // 2, dtype=torch.uint8),
              w1_scales=torch.zeros(I, H // gs, dtype=torch.float16),
              w2_packed=torch.zeros(H, I // 2, dtype=torch.uint8),
              w2_scales=torch.zeros(H, I // gs, dtype=torch.float16))
    tp.check_mlp_block_w4a16(M, H, I, gs, x, cuda=False, **ok)
    for key, bad in [("w1_packed", torch.zeros(I // 2, H // 2, dtype=torch.uint8)),    # half the rows
                     ("w2_packed", torch.zeros(H, I, dtype=torch.uint8)),              # unpacked
                     ("w1_scales", torch.zeros(I, H // gs, dtype=torch.float32)),      # fp32 scales
                     ("w2_scales", torch.zeros(I // gs, H, dtype=torch.float16).t())]: # transposed view
        with pytest.raises(ValueError, match=key):
            tp.check_mlp_block_w4a16(M, H, I, gs, x, cuda=False, **{**ok, key: bad})
    with pytest.raises(ValueError, match="CUDA"):
        tp.check_mlp_block_w4a16(M, H, I, gs, x, **ok)
    p = torch.zeros(64, H // 2, dtype=torch.uint8)
    s = torch.zeros(64, H // gs, dtype=torch.float16)
    tp.check_col_parallel_w4a16(M, H, 64, gs, x, p, s, cuda=False)
    with pytest.raises(ValueError, match="x"):
        tp.check_col_parallel_w4a16(M, H, 64, gs, x.float(), p, s, cuda=False)
    a = torch.zeros(M, 128, dtype=torch.int8)
    w = torch.zeros(32, 128, dtype=torch.int8)
    tp.check_row_parallel_fp8(M, 32, a, torch.zeros(M), w, torch.zeros(32), cuda=False)
    with pytest.raises(ValueError, match="w_codes_shard"):
        tp.check_row_parallel_fp8(M, 32, a, torch.zeros(M), w[:, :64], torch.zeros(32), cuda=False)


def _fused_schedule(R, tiles_m, tiles_n, rank, L):
    """The tile walk of kc_gemm_fp8_allreduce (gemm_fp8.cu, tile_coords<RS>):
    linear tile L -> (m_tile, n_tile, owner, index within the owner's block).
    Output rows are owned in R blocks; rank walks the owners rank+1, ..., rank."""
    tmo, per = tiles_m // R, (tiles_m // R) * tiles_n
    b, j = L // per, L % per
    owner = (rank + 1 + b) % R
    return owner * tmo + j % tmo, j // tmo, owner, j


@pytest.mark.parametrize("R", [2, 4, 8])
def test_fused_row_parallel_schedule(R):
    """The epilogue-fused row-parallel sum, restated on the host with numpy:
    every rank visits every tile once; every (owner, source) partial has its
    own receive slot (rank - owner - 1) mod R; a source reaches each tile of
    an owner's block before the owner does (the owner's block comes last in
    its own walk, so its flag waits follow the partials); and owner-side
    sums of bf16-rounded partials into the owner's fp32 tile give the
    unsharded FP8 GEMM within the bf16 bound."""
    tiles_m, tiles_n = 2 * R, 3
    tiles = tiles_m * tiles_n
    seen = {}
    for rank in range(R):
        coords = [_fused_schedule(R, tiles_m, tiles_n, rank, L) for L in range(tiles)]
        assert len({(m, n) for m, n, _, _ in coords}) == tiles          # every tile once
        for pos, (m, n, owner, j) in enumerate(coords):
            seen.setdefault((m, n), {})[rank] = (pos, owner, j)
    for (m, n), by_rank in seen.items():
        owners = {o for _, o, _ in by_rank.values()}
        assert len(owners) == 1
        owner = owners.pop()
        own_pos = by_rank[owner][0]
        slots = {(src - owner - 1) % R for src in by_rank if src != owner}
        assert slots == set(range(R - 1))                               # one slot per source
        # the owner handles its block last, so every source's block position is earlier
        tmo = tiles_m // R
        assert own_pos // (tmo * tiles_n) == R - 1
        for src, (pos, _, _) in by_rank.items():
            if src != owner:
                assert pos // (tmo * tiles_n) < R - 1
    # numerics: K split in R shards, bf16 partials summed by the owner in slot order
    rng = np.random.default_rng(R)
    Mt, Nt, Kt = 8 * R, 16, 64 * R
    a = rng.standard_normal((Mt, Kt)).astype(np.float32)
    w = rng.standard_normal((Nt, Kt)).astype(np.float32)
    full = a.astype(np.float64) @ w.T.astype(np.float64)
    parts = [a[:, r * Kt // R:(r + 1) * Kt // R] @ w[:, r * Kt // R:(r + 1) * Kt // R].T for r in range(R)]
    bf16 = lambda v: O.bf16_bits_to_f32(O.f32_to_bf16_bits(v.astype(np.float32)))   # noqa: E731
    rows = Mt // R
    out = np.empty((Mt, Nt), np.float32)
    for owner in range(R):
        blk = slice(owner * rows, (owner + 1) * rows)
        acc = parts[owner][blk].astype(np.float32)
        for sl in range(R - 1):
            src = (owner + 1 + sl) % R                                   # slot sl's source
            acc = acc + bf16(parts[src][blk])
        out[blk] = bf16(acc)
    assert np.max(np.abs(out - full)) / np.max(np.abs(full)) <= 1e-2

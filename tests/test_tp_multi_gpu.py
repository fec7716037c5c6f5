"""Multi-GPU: the tensor-parallel drivers on 2 GPUs (one process per GPU, NCCL).

Column parallel: the fused GEMM + all-gather (kc_gemm_w4a16_allgather, and
kc_gemm_w4a16_allgather_mc through the switch's multicast where available)
must give every rank the single-GPU kc_gemm_w4a16 result of the full problem
bit for bit (each output tile is computed by one rank with the same arithmetic and
stored, unchanged, into every rank's buffer).  Row parallel: the K-sharded FP8
GEMM + bf16 sum -- by NCCL all-reduce (also row block by row block, each
block's all-reduce overlapping the next block's GEMM) and by the peer-memory kernel
kc_allreduce_bf16_peer -- against the single-GPU FP8 GEMM, normwise <= 1e-2
(bf16 partials are rounded before the sum); the peer sum is identical on
every rank; so are the sum fused into the GEMM epilogue
(kc_gemm_fp8_allreduce: partial tiles to their row owner, the owner's bf16
sum to every rank) and the in-switch sums (RowParallelFP8 reduce="nvls" and "fused_nvls":
multimem.ld_reduce / multimem.st through NVLink SHARP, where the platform has
multicast).  MLP block (tp.MLPBlockW4A16, the reference's col-parallel ->
GELU -> row-parallel chain): the sharded block against the two unsharded
GEMMs on one GPU, normwise <= 1e-5 (the activations are the same bits; only
the fp32 order of the K sum differs).  Skipped with fewer than 2 GPUs.
"""
import datetime
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
WORLD = 2


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, out_dir):
    import ctypes
    import torch.distributed as dist
    import kc_lib
    import tp
    torch.cuda.set_device(rank)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    l = kc_lib.lib()
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    try:
        g = torch.Generator(device="cuda").manual_seed(5)   # same inputs on every rank
        M, N, K, gs = 300, 1024, 1024, 128
        x = torch.randn(M, K, device="cuda", generator=g).bfloat16()
        packed = torch.randint(0, 256, (N, K // 2), dtype=torch.uint8, device="cuda", generator=g)
        scales = (torch.rand(N, K // gs, device="cuda", generator=g) * 0.018 + 0.002).half()
        full = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
        kc_lib.check(l.kc_gemm_w4a16(x.data_ptr(), packed.data_ptr(), scales.data_ptr(),
                                     full.data_ptr(), 0, M, N, K, gs, N, st))
        n0, n1 = tp.shard_range(N, world, rank)
        col = tp.ColParallelW4A16(M, N, K, gs)
        y = col(x, packed[n0:n1].contiguous(), scales[n0:n1].contiguous())
        torch.cuda.synchronize()
        col_ok = bool(torch.equal(y.view(torch.int16), full.view(torch.int16)))
        # the same through the switch's multicast (one store per tile), where available
        try:
            colm = tp.ColParallelW4A16(M, N, K, gs, store="nvls")
        except RuntimeError:
            colm = None
        if colm is not None:
            for _ in range(2):
                ym = colm(x, packed[n0:n1].contiguous(), scales[n0:n1].contiguous())
            torch.cuda.synchronize()
            col_ok = col_ok and bool(torch.equal(ym.view(torch.int16), full.view(torch.int16)))
            colm.close()

        # row parallel FP8
        M2, N2, K2 = 256, 512, 2048
        xa = torch.randn(M2, K2, device="cuda", generator=g)
        w = torch.randn(N2, K2, device="cuda", generator=g) * 0.02
        qa = torch.empty(M2, K2, dtype=torch.int8, device="cuda"); sa = torch.empty(M2, device="cuda")
        qw = torch.empty(N2, K2, dtype=torch.int8, device="cuda"); sw = torch.empty(N2, device="cuda")
        kc_lib.check(l.kc_quantize_fp8_per_token(xa.data_ptr(), qa.data_ptr(), sa.data_ptr(), M2, K2, st))
        kc_lib.check(l.kc_quantize_fp8_per_channel(w.data_ptr(), qw.data_ptr(), sw.data_ptr(), N2, K2, st))
        ref = torch.empty(M2, N2, dtype=torch.float32, device="cuda")
        kc_lib.check(l.kc_gemm_fp8(qa.data_ptr(), sa.data_ptr(), qw.data_ptr(), sw.data_ptr(),
                                   ref.data_ptr(), 1, M2, N2, K2, N2, st))
        k0, k1 = tp.shard_range(K2, world, rank)
        qa_s, qw_s = qa[:, k0:k1].contiguous(), qw[:, k0:k1].contiguous()
        out = torch.empty(M2, N2, dtype=torch.bfloat16, device="cuda")
        tp.row_parallel_fp8(qa_s, sa, qw_s, sw, out)
        torch.cuda.synchronize()
        row_err = float((out.float() - ref).abs().max() / ref.abs().max())
        # the overlapped form: row blocks whose all-reduce runs under the next block's GEMM
        out_ov = torch.empty(M2, N2, dtype=torch.bfloat16, device="cuda")
        tp.row_parallel_fp8_overlap(qa_s, sa, qw_s, sw, out_ov, chunks=2)
        torch.cuda.synchronize()
        row_err = max(row_err, float((out_ov.float() - ref).abs().max() / ref.abs().max()))
        rp = tp.RowParallelFP8(M2, N2)
        y2 = rp(qa_s, sa, qw_s, sw)
        torch.cuda.synchronize()
        row_err = max(row_err, float((y2.float() - ref).abs().max() / ref.abs().max()))
        # the peer reduction sums in fp32 once: every rank holds identical bits
        gathered = [torch.empty_like(y2) for _ in range(world)]
        dist.all_gather(gathered, y2.clone())
        row_same = all(torch.equal(gathered[0].view(torch.int16), g.view(torch.int16)) for g in gathered)
        rp.close()
        # the sum fused into the GEMM epilogue (partials to their row owner, the
        # owner's sum to every rank), twice: the second call reuses the buffers
        # and flags with the next epoch
        rf = tp.RowParallelFP8(M2, N2, reduce="fused")
        rf(qa_s, sa, qw_s, sw)
        y5 = rf(qa_s, sa, qw_s, sw).clone()
        torch.cuda.synchronize()
        fused_err = float((y5.float() - ref).abs().max() / ref.abs().max())
        gathered = [torch.empty_like(y5) for _ in range(world)]
        dist.all_gather(gathered, y5)
        fused_same = float(all(torch.equal(gathered[0].view(torch.int16), g.view(torch.int16))
                               for g in gathered))
        rf.close()
        # the in-switch sum (NVLink SHARP multicast): after the GEMM in two row
        # blocks, and inside the GEMM's epilogue; each twice in a row (the
        # second call reuses the symmetric buffer behind the barriers)
        nvls_err, nvls_same = -1.0, -1.0               # stay -1 without multicast
        for mode in ("nvls", "fused_nvls"):
            try:
                rn = tp.RowParallelFP8(M2, N2, reduce=mode, chunks=2)
            except RuntimeError:
                continue
            rn(qa_s, sa, qw_s, sw)
            y4 = rn(qa_s, sa, qw_s, sw, entry_barrier=True).clone()
            torch.cuda.synchronize()
            nvls_err = max(nvls_err, float((y4.float() - ref).abs().max() / ref.abs().max()))
            gathered = [torch.empty_like(y4) for _ in range(world)]
            dist.all_gather(gathered, y4)
            same = float(all(torch.equal(gathered[0].view(torch.int16), g.view(torch.int16))
                             for g in gathered))
            nvls_same = same if nvls_same < 0 else min(nvls_same, same)
            rn.close()

        # MLP block: W1 [I, H] by rows, W2 [H, I] by the same columns, one all-reduce
        M3, H3, I3 = 200, 512, 2048
        x3 = torch.randn(M3, H3, device="cuda", generator=g).bfloat16()
        w1p = torch.randint(0, 256, (I3, H3 // 2), dtype=torch.uint8, device="cuda", generator=g)
        w1s = (torch.rand(I3, H3 // gs, device="cuda", generator=g) * 0.018 + 0.002).half()
        w2p = torch.randint(0, 256, (H3, I3 // 2), dtype=torch.uint8, device="cuda", generator=g)
        w2s = (torch.rand(H3, I3 // gs, device="cuda", generator=g) * 0.018 + 0.002).half()
        h_full = torch.empty(M3, I3, dtype=torch.bfloat16, device="cuda")
        y_full = torch.empty(M3, H3, dtype=torch.float32, device="cuda")
        kc_lib.check(l.kc_gemm_w4a16_act(x3.data_ptr(), w1p.data_ptr(), w1s.data_ptr(), h_full.data_ptr(),
                                         0, M3, I3, H3, gs, I3, kc_lib.KC_ACT_GELU_QUICK, st))
        kc_lib.check(l.kc_gemm_w4a16(h_full.data_ptr(), w2p.data_ptr(), w2s.data_ptr(), y_full.data_ptr(),
                                     1, M3, H3, I3, gs, H3, st))
        p1, s1 = tp.shard_w4_rows(w1p, w1s, world, rank)
        p2, s2 = tp.shard_w4_cols(w2p, w2s, gs, world, rank)
        mlp = tp.MLPBlockW4A16(M3, H3, I3, gs)
        y3 = mlp(x3, p1, s1, p2, s2)
        torch.cuda.synchronize()
        mlp_err = float((y3 - y_full).abs().max() / y_full.abs().max())
        status = l.kc_get_device_status()
        np.save(os.path.join(out_dir, f"rank{rank}.npy"),
                np.array([col_ok, row_err, status, row_same, mlp_err, nvls_err, nvls_same,
                          fused_err, fused_same], dtype=np.float64))
        col.close()
    finally:
        dist.destroy_process_group()


def test_tensor_parallel_two_gpus(tmp_path):
    if not torch.cuda.is_available() or torch.cuda.device_count() < WORLD:
        pytest.skip(f"needs {WORLD} GPUs")
    import torch.multiprocessing as mp
    mp.spawn(_rank_main, args=(WORLD, _free_port(), str(tmp_path)), nprocs=WORLD, join=True)
    for r in range(WORLD):
        (col_ok, row_err, status, row_same, mlp_err, nvls_err, nvls_same, fused_err,
         fused_same) = np.load(tmp_path / f"rank{r}.npy")
        assert row_same == 1.0, "peer all-reduce outputs differ between ranks"
        assert col_ok == 1.0, f"rank {r}: gathered W4A16 output differs from the single-GPU GEMM"
        assert row_err <= 1e-2, f"rank {r}: row-parallel FP8 error {row_err}"
        assert mlp_err <= 1e-5, f"rank {r}: MLP block error {mlp_err}"
        assert fused_err <= 1e-2, f"rank {r}: row-parallel FP8 (sum in the epilogue) error {fused_err}"
        assert fused_same == 1.0, "epilogue-sum outputs differ between ranks"
        if nvls_err >= 0:
            assert nvls_err <= 1e-2, f"rank {r}: row-parallel FP8 (in-switch sum) error {nvls_err}"
            assert nvls_same == 1.0, "in-switch sum outputs differ between ranks"
        assert status == 0

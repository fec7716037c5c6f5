"""GPU parity: fp32 shard GEMM, simulated collectives, NCCL reference API."""
import ctypes

import numpy as np
import pytest
import torch

import kc_lib
import kcref
import oracle as O
from kc_testutil import dev, host, last_error, normwise_err, ptr, stream

pytestmark = pytest.mark.gpu


def _sgemm(A, B):
    M, K = A.shape
    N = B.shape[0]
    C = torch.full((M, N), float("nan"), dtype=torch.float32, device=A.device)
    kc_lib.lib().launch_col_parallel_linear(ptr(A), ptr(B), ptr(C), M, N, K, stream())
    kc_lib.check_last()
    return host(C)


@pytest.mark.parametrize("M,N,K", [(1, 4096, 4096), (128, 1024, 512), (65, 33, 17), (3, 4, 8),
                                   (256, 256, 1)])
def test_sgemm_vs_oracle(cuda, M, N, K):
    rng = np.random.default_rng(M + N + K)
    A = rng.standard_normal((M, K)).astype(np.float32)
    B = rng.standard_normal((N, K)).astype(np.float32)
    C = _sgemm(dev(A), dev(B))
    assert normwise_err(C, O.gemm_nt_f32(A, B)) <= 1e-5
    if kcref.available() and M * N * K <= 2**27:
        assert normwise_err(C, host(kcref.sgemm_nt(dev(A), dev(B)))) <= 1e-5


def test_reference_tp_kats(cuda, golden):
    d = golden("kat_tensor_parallel.npz")
    l = kc_lib.lib()
    # column-parallel, 2 ranks, host re-interleave (test_tensor_parallel.cpp:209-259)
    y0, y1 = _sgemm(dev(d["col_x"]), dev(d["col_W"][:3].copy())), _sgemm(dev(d["col_x"]),
                                                                         dev(d["col_W"][3:].copy()))
    assert np.max(np.abs(np.concatenate([y0, y1], 1) - d["col_ref"])) < 1e-3
    # row-parallel, 2 ranks (:272-330)
    x, W = d["row_x"], d["row_W"]
    parts = []
    for sl in (slice(0, 4), slice(4, 8)):
        xs, Ws = dev(x[:, sl].copy()), dev(W[:, sl].copy())
        out = torch.empty(4, 6, dtype=torch.float32, device=cuda)
        l.launch_row_parallel_linear(ptr(xs), ptr(Ws), ptr(out), 4, 6, 4, stream())
        parts.append(host(out))
    assert np.max(np.abs(parts[0] + parts[1] - d["row_ref"])) < 1e-3
    # chain (:339-376)
    mid = _sgemm(dev(d["chain_x"]), dev(d["chain_W1"]))
    assert np.max(np.abs(_sgemm(dev(mid), dev(d["chain_W2"])) - d["chain_ref"])) < 1e-3


@pytest.mark.parametrize("R,count", [(2, 4), (4, 8), (3, 1000), (8, 1 << 20), (5, 7)])
def test_sim_allreduce_bitexact(cuda, R, count):
    rng = np.random.default_rng(R * count)
    b = (rng.standard_normal((R, count)) * 10.0 ** rng.integers(-3, 4, (R, count))).astype(np.float32)
    bufs = [dev(b[r].copy()) for r in range(R)]
    arr = (ctypes.c_void_p * R)(*[t.data_ptr() for t in bufs])
    kc_lib.lib().launch_ring_allreduce(arr, count, R, stream())
    kc_lib.check_last()
    want = O.ring_allreduce(b)
    for r in range(R):
        np.testing.assert_array_equal(host(bufs[r]).view(np.uint32), want[r].view(np.uint32))
    if kcref.available():
        rb = [dev(b[r].copy()) for r in range(R)]
        kcref.ring_allreduce(rb)
        for r in range(R):
            np.testing.assert_array_equal(host(rb[r]).view(np.uint32), want[r].view(np.uint32))


def test_sim_allreduce_single_rank_noop(cuda):
    b = dev(np.arange(16, dtype=np.float32))
    arr = (ctypes.c_void_p * 1)(b.data_ptr())
    kc_lib.lib().launch_ring_allreduce(arr, 16, 1, stream())
    np.testing.assert_array_equal(host(b), np.arange(16, dtype=np.float32))


def test_sim_allgather(cuda, golden):
    d = golden("kat_tensor_parallel.npz")
    chunks = [dev(c.copy()) for c in d["ag_chunks"]]
    out = torch.empty(12, dtype=torch.float32, device=cuda)
    arr = (ctypes.c_void_p * 4)(*[c.data_ptr() for c in chunks])
    kc_lib.lib().launch_allgather(arr, ptr(out), 3, 4, stream())
    kc_lib.check_last()
    np.testing.assert_array_equal(host(out), d["ag_expected"])


def test_nccl_reference_api_single_rank(cuda):
    """ncclCommInitAll with one device; fp32 in-place all-reduce and all-gather
    (tensor_parallel_nccl.cu:58-135) are identities at one rank."""
    l = kc_lib.lib()
    comms = (ctypes.c_void_p * 1)()
    devs = (ctypes.c_int * 1)(torch.cuda.current_device())
    l.nccl_comm_init_all(comms, 1, devs)
    st, msg = last_error()
    assert st == 0 and comms[0], msg
    try:
        assert l.nccl_comm_count(comms[0]) == 1 and l.nccl_comm_user_rank(comms[0]) == 0
        buf = dev(np.arange(1024, dtype=np.float32))
        l.launch_ring_allreduce_nccl(comms[0], ptr(buf), 1024, stream())
        recv = torch.empty(1024, dtype=torch.float32, device=cuda)
        l.launch_allgather_nccl(comms[0], ptr(buf), ptr(recv), 1024, stream())
        assert last_error()[0] == 0
        np.testing.assert_array_equal(host(buf), np.arange(1024, dtype=np.float32))
        np.testing.assert_array_equal(host(recv), np.arange(1024, dtype=np.float32))
        hb = torch.ones(64, dtype=torch.bfloat16, device=cuda)
        kc_lib.check(l.kc_allreduce_bf16(comms[0], ptr(hb), ptr(hb), 64, stream()))
        assert torch.all(hb == 1)
        kc_lib.check(l.kc_nccl_comm_check(comms[0]))
    finally:
        l.nccl_comm_destroy(comms[0])


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_nccl_reference_api_two_gpus(cuda):
    """The reference test's two-communicator group pattern (test_tensor_parallel.cpp:384-495)
    on two distinct GPUs."""
    l = kc_lib.lib()
    comms = (ctypes.c_void_p * 2)()
    devs = (ctypes.c_int * 2)(0, 1)
    l.nccl_comm_init_all(comms, 2, devs)
    assert last_error()[0] == 0 and comms[0] and comms[1]
    try:
        bufs, streams = [], []
        for r in range(2):
            with torch.cuda.device(r):
                bufs.append(torch.ones(1024, dtype=torch.float32, device=f"cuda:{r}"))
                streams.append(torch.cuda.Stream(device=r))
        l.nccl_group_start()
        for r in range(2):
            l.launch_ring_allreduce_nccl(comms[r], ptr(bufs[r]), 1024,
                                         ctypes.c_void_p(streams[r].cuda_stream))
        l.nccl_group_end()
        for r in range(2):
            streams[r].synchronize()
            assert torch.all(bufs[r] == 2.0)
    finally:
        l.nccl_comm_destroy(comms[0])
        l.nccl_comm_destroy(comms[1])

"""Failure detection without a GPU fault: a device-side wait that nothing
completes gives up after a short limit, the kernel returns, the host reads
KC_ERR_TIMEOUT, and the context keeps working."""
import ctypes

import numpy as np
import pytest
import torch

import kc_lib
import oracle as O
from kc_testutil import host, ptr, stream

pytestmark = pytest.mark.gpu


def test_bounded_wait_times_out_and_context_survives(cuda):
    l = kc_lib.lib()
    assert l.kc_get_device_status() == kc_lib.KC_OK
    waited = torch.full((1,), -7, dtype=torch.int32, device=cuda)
    kc_lib.check(l.kc_selftest_bounded_wait(200_000_000, ptr(waited), stream()))   # 0.2 s
    assert l.kc_get_device_status() == kc_lib.KC_ERR_TIMEOUT
    assert l.kc_get_last_error() == kc_lib.KC_ERR_TIMEOUT      # also recorded on the thread
    assert 200 <= int(host(waited)[0]) < 5000
    assert l.kc_get_device_status() == kc_lib.KC_OK          # reading cleared it
    # the context is still usable: a real kernel runs and is correct
    import kernel_craft_torch_ops as ops
    packed, scales = O.make_w4_gptq(64, 256, 128, seed=1)
    x = O.make_activations_bf16(1, 256, seed=2)
    y = ops.w4a16_gemv(torch.from_numpy(packed).to(cuda), torch.from_numpy(scales).to(cuda),
                       torch.from_numpy(x).to(cuda).view(torch.bfloat16), 128)
    ref = O.gemv_w4a16(packed, scales, x, 1, 64, 256, 128)
    assert np.max(np.abs(host(y) - ref)) / np.max(np.abs(ref)) <= 1e-3


def test_pipelined_gemv_reports_no_timeout(cuda):
    import kernel_craft_torch_ops as ops
    packed, scales = O.make_w4_gptq(4096, 4096, 128, seed=3)
    x = O.make_activations_bf16(1, 4096, seed=4)
    for _ in range(3):
        ops.w4a16_gemv(torch.from_numpy(packed).to(cuda), torch.from_numpy(scales).to(cuda),
                       torch.from_numpy(x).to(cuda).view(torch.bfloat16), 128)
    assert kc_lib.lib().kc_get_device_status() == kc_lib.KC_OK


def test_peer_barrier_timeout_is_surfaced_and_poisons_the_peer_sum(cuda):
    # one GPU, two "ranks": rank 1's flag array is a second local array that
    # nothing ever writes into rank 0's slot 1, so rank 0's wait gives up --
    # the failure is a flag nobody sets, never a fault
    l = kc_lib.lib()
    assert l.kc_get_device_status() == kc_lib.KC_OK
    f0 = torch.zeros(kc_lib.KC_MAX_RANKS, dtype=torch.int32, device=cuda)
    f1 = torch.zeros(kc_lib.KC_MAX_RANKS, dtype=torch.int32, device=cuda)
    flags = (ctypes.c_void_p * 2)(f0.data_ptr(), f1.data_ptr())
    status = torch.zeros(1, dtype=torch.int32).pin_memory()
    kc_lib.check(l.kc_peer_barrier(flags, 2, 0, 1, 200_000_000, ptr(status), stream()))  # 0.2 s
    torch.cuda.synchronize()
    assert int(status[0]) == kc_lib.KC_ERR_TIMEOUT            # seen on the host, no device read
    assert int(host(f1)[0]) == 1                              # the epoch was published to the peer
    # while the status is set, the peer all-reduce writes NaN instead of a sum
    part = torch.ones(64, dtype=torch.bfloat16, device=cuda)
    out = torch.zeros(64, dtype=torch.bfloat16, device=cuda)
    one = (ctypes.c_void_p * 1)(part.data_ptr())
    dst = (ctypes.c_void_p * 1)(out.data_ptr())
    kc_lib.check(l.kc_allreduce_bf16_peer(one, dst, 1, 0, 64, stream()))
    assert torch.isnan(out.float()).all()
    assert l.kc_get_device_status() == kc_lib.KC_ERR_TIMEOUT  # reading clears it
    kc_lib.check(l.kc_allreduce_bf16_peer(one, dst, 1, 0, 64, stream()))
    assert torch.equal(out.float().cpu(), torch.ones(64))
    # bad timeouts and unpinned status slots are refused on the host
    assert l.kc_peer_barrier(flags, 2, 0, 2, 10**15, None, stream()) == kc_lib.KC_ERR_INVALID_ARG
    plain = torch.zeros(1, dtype=torch.int32)
    assert l.kc_peer_barrier(flags, 2, 0, 2, 0, ptr(plain), stream()) == kc_lib.KC_ERR_INVALID_ARG
    assert l.kc_get_last_error() == kc_lib.KC_ERR_INVALID_ARG   # read (and cleared) here
    assert l.kc_get_device_status() == kc_lib.KC_OK

"""GPU: the allocation-free dynamic per-tensor FP8 quantization.

kc_quantize_fp8_per_tensor_dynamic_noalloc keeps its scratch in a static array
of the library's device image.  It must give the same codes and scale as
kc_quantize_fp8_per_tensor_dynamic (caller workspace) -- bit-exact, the
tolerance here is zero -- on consecutive calls, so that state left by one call
cannot leak into the next.  Collected last so it also runs after every other
test has used the library in the same process.
"""
import numpy as np
import pytest
import torch

import kc_lib
import oracle as O
from kc_testutil import dev, host, misaligned, ptr, stream

pytestmark = pytest.mark.gpu


def _with_workspace(dx, count):
    q = torch.full((max(count, 1),), 0x55, dtype=torch.int8, device=dx.device)
    s = torch.full((1,), -1.0, dtype=torch.float32, device=dx.device)
    ws = torch.empty(1, dtype=torch.int32, device=dx.device)
    kc_lib.check(kc_lib.lib().kc_quantize_fp8_per_tensor_dynamic(ptr(dx), ptr(q), ptr(s), count,
                                                                 ptr(ws), 4, stream()))
    return host(q)[:count].view(np.uint8), host(s)[0]


def _no_alloc(dx, count):
    q = torch.full((max(count, 1),), 0x55, dtype=torch.int8, device=dx.device)
    s = torch.full((1,), -1.0, dtype=torch.float32, device=dx.device)
    kc_lib.check(kc_lib.lib().kc_quantize_fp8_per_tensor_dynamic_noalloc(ptr(dx), ptr(q), ptr(s),
                                                                         count, stream()))
    return host(q)[:count].view(np.uint8), host(s)[0]


def _input(count, seed, magnitude):
    rng = np.random.default_rng(seed)
    return (rng.standard_normal(count) * magnitude).astype(np.float32)


def test_no_alloc_matches_workspace_variant_twice_in_a_row(cuda):
    # first call: many chunks, a ragged tail, large amax; second call: fewer
    # chunks and an amax 1e5 times smaller, so a stale amax or partial from the
    # first call would change the second call's scale
    cases = [(5_000_003, 11, 100.0), (70_001, 12, 1e-3)]
    for count, seed, mag in cases:
        x = _input(count, seed, mag)
        dx = dev(x)
        q_ref, s_ref = _with_workspace(dx, count)
        q, s = _no_alloc(dx, count)
        assert s == s_ref == O.per_tensor_scale(x)
        np.testing.assert_array_equal(q, q_ref)
    assert kc_lib.lib().kc_get_device_status() == kc_lib.KC_OK


def test_no_alloc_misaligned_and_empty(cuda):
    x = _input(4099, 13, 3.0)
    dx = misaligned(dev(x))
    q_ref, s_ref = _with_workspace(dx, x.size)
    q, s = _no_alloc(dx, x.size)
    assert s == s_ref
    np.testing.assert_array_equal(q, q_ref)
    # empty tensor: amax 0 -> scale 1, as in the workspace variant
    empty = torch.zeros(4, dtype=torch.float32, device=cuda)
    assert _no_alloc(empty, 0)[1] == _with_workspace(empty, 0)[1] == 1.0


def test_no_alloc_rejects_counts_beyond_its_scratch(cuda):
    # refused on the host before anything is launched
    b = torch.zeros(16, dtype=torch.float32, device=cuda)
    with pytest.raises(kc_lib.KcError) as err:
        kc_lib.check(kc_lib.lib().kc_quantize_fp8_per_tensor_dynamic_noalloc(
            ptr(b), ptr(b), ptr(b), (1 << 30) + 1, stream()))
    assert err.value.status == kc_lib.KC_ERR_INVALID_ARG
    assert "no-alloc maximum" in str(err.value)
    # a valid call right after the refusal still works
    x = _input(100, 14, 1.0)
    dx = dev(x)
    assert _no_alloc(dx, 100)[1] == _with_workspace(dx, 100)[1]

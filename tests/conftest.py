"""pytest configuration: the `gpu` marker, import paths, shared fixtures.

CPU tests (``-m "not gpu"``) cover the oracle against the golden fixtures, the
host-side logic, multi-process paths on gloo, and that libkernels.so loads and
exports every symbol include/kernel_craft.h declares.  GPU tests (``-m gpu``)
are the parity tests: they call the CUDA library through its C ABI and compare
with the oracle (and, when oracle/_ref/libkcref.so is present, with the
reference's own kernels run on the same inputs).
"""
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
for p in (ROOT / "kernel-craft_b200", ROOT / "oracle", ROOT):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def golden():
    def load(name):
        return np.load(GOLDEN / name)
    return load


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import kc_lib
    kc_lib.lib()  # the native library must load: no fallback
    return torch.device("cuda:0")

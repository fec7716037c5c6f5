"""bench.py's reference arm on CPU: one JSON line with the contract's keys
(the kc arm needs a GPU and is exercised by the GPU runs)."""
import json
import os
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent


@pytest.mark.parametrize("workload", ["gemv", "gemv_int4"])
def test_reference_arm_line(workload):
    # the contract, not the speed: one decode layer instead of the full 32
    out = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--workload",
                          workload, "--steps", "1", "--warmup", "3", "--layers", "1"],
                         capture_output=True, text=True, timeout=600, cwd=ROOT,
                         env={**os.environ, "RANK": "0"})
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [l for l in out.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
                "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config",
                "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference" and d["value"] > 0
    assert d["cpu_baseline"]["kind"] == "port" and d["cpu_baseline"]["cores"] >= 1
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["value"] == d["value"]


def test_reference_arm_other_ranks_print_nothing():
    out = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "1"],
                         capture_output=True, text=True, timeout=300, cwd=ROOT,
                         env={**os.environ, "RANK": "1"})
    assert out.returncode == 0 and not out.stdout.strip()

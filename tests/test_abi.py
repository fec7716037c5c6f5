"""C-ABI checks that need no GPU: the library loads, exports every symbol
include/kernel_craft.h declares, rejects invalid arguments on the host before
touching the device, and the reference's own ctypes bridge can bind it."""
import os
import re
import subprocess
import sys
from pathlib import Path

import pytest

import kc_lib

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "kernel_craft.h"
# the kernel-craft checkout: $KC_REF_DIR, else one named "reference" beside this repository
REF_DIR = Path(os.environ.get("KC_REF_DIR", ROOT.parent / "reference"))
REF_BRIDGE = REF_DIR / "src/python/kernel_craft_torch_ops.py"


def declared_symbols():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^KC_API\s+[\w\s\*]+?\b(\w+)\s*\(", text, re.M)))


def exported_symbols():
    out = subprocess.run(["nm", "-D", "--defined-only", str(kc_lib.lib_path())],
                         capture_output=True, text=True, check=True).stdout
    return {l.split()[-1] for l in out.splitlines() if " T " in l}


def test_header_declares_reference_launchers():
    syms = declared_symbols()
    for name in ["launch_dequantize_int4", "launch_gemv_int4", "launch_quantize_fp8",
                 "launch_dequantize_fp8", "launch_smoothquant_scale", "launch_col_parallel_linear",
                 "launch_row_parallel_linear", "launch_ring_allreduce", "launch_allgather",
                 "nccl_comm_init_all", "nccl_comm_destroy", "nccl_group_start", "nccl_group_end",
                 "launch_ring_allreduce_nccl", "launch_allgather_nccl", "nccl_comm_count",
                 "nccl_comm_user_rank"]:
        assert name in syms, name


def test_every_declared_symbol_is_exported():
    missing = set(declared_symbols()) - exported_symbols()
    assert not missing, f"declared but not exported: {sorted(missing)}"


def test_ctypes_prototypes_cover_the_header():
    assert set(declared_symbols()) == set(kc_lib.exported_names())


def test_library_loads_and_reports_version():
    assert b"sm_100a" in kc_lib.lib().kc_version()


def test_built_for_sm100a_only():
    """The build recipe compiles every CUDA source for sm_100a and nothing else
    (checked on the recipe, not by inspecting the compiled code)."""
    recipe = (ROOT / "kernel-craft_b200" / "build.py").read_text()
    assert set(re.findall(r"arch=compute_\w+,code=\w+", recipe)) == {"arch=compute_100a,code=sm_100a"}
    assert "-arch" not in recipe.replace("arch=compute_100a", "")


@pytest.mark.parametrize("call", [
    lambda l: l.kc_gemv_w4a16(None, None, None, None, 1, 16, 128, 128, None),
    lambda l: l.kc_gemv_w4a16(1, 1, 1, 1, 0, 16, 128, 128, None),          # M = 0
    lambda l: l.kc_gemv_w4a16(1, 1, 1, 1, 17, 16, 128, 128, None),         # M > 16
    lambda l: l.kc_gemv_w4a16(1, 1, 1, 1, 1, 16, 130, 128, None),          # gs !| K
    lambda l: l.kc_dequantize_int4_f32(1, 1, 1, 1, 4, 7, 7, None),         # odd cols
    lambda l: l.kc_gemv_int4_f32(1, 1, 1, 1, 1, 4, 8, 0, None),            # gs = 0
    lambda l: l.kc_quantize_fp8_per_token(None, 1, 1, 4, 4, None),
    lambda l: l.kc_quantize_fp8_per_tensor_dynamic(1, 1, 1, 16, 1, 2, None),  # workspace < 4
    lambda l: l.kc_sgemm_nt(1, 1, 1, -1, 4, 4, None),
    lambda l: l.kc_dequantize_w4_bf16(1, 1, 1, 4, 6, 4, None),              # gs !| K
    lambda l: l.kc_nccl_comm_init_rank(None, 2, None, 0),
    # the fused collectives and the tile-ordered layout
    lambda l: l.kc_gemm_fp8_allreduce(1, 1, 1, 1, None, None, None, 2, 0, 1, 512, 512, 64, 0, None),
    lambda l: l.kc_gemm_fp8_allreduce_mc(1, 1, 1, 1, None, None, None, 2, 0, 1, 512, 512, 64, 0, None),
    lambda l: l.kc_allreduce_bf16_nvls(None, 2, 0, 1024, 0, None),
    lambda l: l.kc_allreduce_bf16_nvls(16, 2, 0, 1000, 0, None),           # count % (8 * ranks)
    lambda l: l.kc_w4a16_tile_weights(None, None, 16, 128, None),
    lambda l: l.kc_w4a16_tile_weights(16, 16, 16, 100, None),              # K % 128
    lambda l: l.kc_gemv_w4a16_grouped_tiled(None, None, None, 1, 1, 128, None),
    lambda l: l.kc_selftest_stream_read(None, 16, 0, None, None),
])
def test_host_validation_rejects_without_launching(call):
    l = kc_lib.lib()
    st = call(l)
    assert st == kc_lib.KC_ERR_INVALID_ARG
    assert l.kc_get_last_error() == kc_lib.KC_ERR_INVALID_ARG
    assert l.kc_get_last_error() == 0  # reading clears


def test_out_of_scope_launchers_report_unsupported():
    l = kc_lib.lib()
    l.kc_get_last_error()
    l.launch_flash_attention(None, None, None, None, 1, 1, 1, 1, 1, False, None)
    assert l.kc_get_last_error() == kc_lib.KC_ERR_UNSUPPORTED


def test_grouped_problem_struct_layout():
    import ctypes
    assert ctypes.sizeof(kc_lib.W4A16Problem) == 40
    assert kc_lib.W4A16Problem.N.offset == 32 and kc_lib.W4A16Problem.K.offset == 36


@pytest.mark.skipif(not REF_BRIDGE.exists(), reason="reference checkout not present")
def test_reference_ctypes_bridge_binds_this_library():
    """The reference's unmodified kernel_craft_torch_ops.py (its _find_lib honours
    KERNEL_CRAFT_LIB, :71-72) loads libkernels.so and sets every prototype
    (:101-168) -- the drop-in claim for the Python front end.  Run in a child
    process: the reference module registers the same torch.library namespace."""
    code = (
        "import sys; sys.path.insert(0, %r)\n"
        "import torch\n"
        "import kernel_craft_torch_ops as k\n"
        "lib = k._get_lib()\n"
        "for n in ['launch_dequantize_int4','launch_gemv_int4','launch_quantize_fp8',"
        "'launch_dequantize_fp8','launch_flash_attention','launch_paged_attention',"
        "'launch_verify_draft_tokens']:\n"
        "    assert getattr(lib, n).argtypes is not None, n\n"
        "print('BOUND', k.TORCH_OPS_REGISTERED)\n" % str(REF_BRIDGE.parent))
    env = dict(os.environ, KERNEL_CRAFT_LIB=str(kc_lib.lib_path()))
    res = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, env=env,
                         timeout=300)
    assert res.returncode == 0, res.stderr[-2000:]
    assert "BOUND True" in res.stdout

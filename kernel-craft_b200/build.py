"""Builds libkernels.so for sm_100a, in tree (kernel-craft_b200/lib/).

    python kernel-craft_b200/build.py [--force] [--jobs N]

Every .cu / .cpp under csrc/ is compiled with nvcc for
``-gencode arch=compute_100a,code=sm_100a`` and linked, together with NCCL,
into one shared library that exports the reference's launcher ABI plus the
kc_* API declared in include/kernel_craft.h.  Objects are rebuilt only when a
source or header is newer than the object.  No GPU is needed to build.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent
CSRC = HERE / "csrc"
OBJ = HERE / "_build"
LIB_DIR = HERE / "lib"
LIB = LIB_DIR / "libkernels.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC,-fvisibility=hidden",
    "-I", str(ROOT / "include"),
    "-Xptxas", "-warn-spills",
]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def _sources() -> list[Path]:
    return sorted(p for p in CSRC.iterdir() if p.suffix in (".cu", ".cpp"))


def _headers() -> list[Path]:
    hs = [p for p in CSRC.iterdir() if p.suffix in (".cuh", ".h", ".hpp")]
    hs += list((ROOT / "include").glob("*.h"))
    return hs


def _compile(src: Path, force: bool, extra: list[str]) -> tuple[Path, str]:
    obj = OBJ / (src.name + ".o")
    newest_dep = max([src.stat().st_mtime] + [h.stat().st_mtime for h in _headers()])
    if not force and obj.exists() and obj.stat().st_mtime >= newest_dep:
        return obj, ""
    cmd = [_nvcc()] + NVCC_FLAGS + extra + ["-c", str(src), "-o", str(obj)]
    if src.suffix == ".cpp":
        cmd[1:1] = ["-x", "cu"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{res.stdout}\n{res.stderr}")
    return obj, (res.stdout + res.stderr).strip()


def build(force: bool = False, jobs: int | None = None, verbose: bool = False) -> Path:
    OBJ.mkdir(exist_ok=True)
    LIB_DIR.mkdir(exist_ok=True)
    srcs = _sources()
    extra: list[str] = []
    jobs = jobs or min(8, os.cpu_count() or 1)
    with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
        results = list(ex.map(lambda s: _compile(s, force, extra), srcs))
    objs = [o for o, _ in results]
    for (o, log), s in zip(results, srcs):
        if log and verbose:
            print(f"[{s.name}]\n{log}")
    newest_obj = max(o.stat().st_mtime for o in objs)
    if force or not LIB.exists() or LIB.stat().st_mtime < newest_obj:
        cmd = [_nvcc()] + ARCH + ["-shared", "-o", str(LIB)] + [str(o) for o in objs] + ["-lnccl"]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
    return LIB


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--jobs", type=int, default=None)
    ap.add_argument("-v", "--verbose", action="store_true")
    a = ap.parse_args(argv)
    lib = build(force=a.force, jobs=a.jobs, verbose=a.verbose)
    print(f"built {lib}")
    return 0


if __name__ == "__main__":
    sys.exit(main())

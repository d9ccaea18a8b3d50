"""Build libflashmaxsim_sm100.so in-tree with nvcc for sm_100a.

The library is the product: every MaxSim kernel plus the C ABI of
include/fms.h.  It links the CUDA runtime dynamically (so it shares torch's /
CUDA.jl's runtime state, e.g. the current device) and needs no other library
at link time (NCCL is opened at run time by the multi-GPU entry points; its
header, nccl.h, is needed to build).
Each source compiles to its own object (in parallel, under _build/), then one
link step makes the shared library.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
LIB = PKG / "libflashmaxsim_sm100.so"
OBJ = PKG / "_build"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def sources():
    return sorted(CSRC.glob("*.cu"))


def headers():
    return sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + sorted(INCLUDE.glob("*.h"))


def up_to_date() -> bool:
    if not LIB.exists():
        return False
    t = LIB.stat().st_mtime
    return all(p.stat().st_mtime <= t for p in sources() + headers() + [Path(__file__)])


def _compile(src: Path, verbose: bool) -> Path:
    obj = OBJ / (src.stem + ".o")
    cmd = [nvcc()] + ARCH + [
        "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O3",
        "-I", str(INCLUDE), "-I", str(CSRC), "-c", str(src), "-o", str(obj)]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    subprocess.check_call(cmd)
    return obj


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and up_to_date():
        return LIB
    OBJ.mkdir(exist_ok=True)
    with ThreadPoolExecutor(max_workers=max(1, min(len(sources()), os.cpu_count() or 1))) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose), sources()))
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc()] + ARCH + ["-shared", "-cudart", "shared",
                             "-Xlinker", "-rpath,/usr/local/cuda/lib64", "-o", str(tmp)] + \
        [str(o) for o in objs] + ["-ldl"]
    subprocess.check_call(cmd)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))

"""Build recipe for the CPU oracle (test infrastructure only).

Compiles oracle/fms_oracle.c into oracle/_build/libfms_oracle.so with gcc and
OpenMP.  FlashMaxSim.jl is Julia and no Julia toolchain exists on these
machines, so there is no oracle/_ref build of the reference itself.
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
SRC = HERE / "fms_oracle.c"
OUT_DIR = HERE / "_build"
LIB = OUT_DIR / "libfms_oracle.so"


def build(force: bool = False) -> Path:
    OUT_DIR.mkdir(exist_ok=True)
    if LIB.exists() and not force and LIB.stat().st_mtime >= SRC.stat().st_mtime:
        return LIB
    # -march=x86-64-v3 (AVX2 + FMA), not -march=native: the library travels to
    # the GPU box, whose host CPU may differ from the build machine's.  OpenMP
    # gives the labelled multi-core CPU baseline.
    cmd = ["gcc", "-O3", "-march=x86-64-v3", "-fopenmp", "-fPIC", "-shared",
           "-Wall", "-o", str(LIB) + ".tmp", str(SRC), "-lm"]
    subprocess.check_call(cmd)
    os.replace(str(LIB) + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))

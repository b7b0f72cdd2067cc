"""Build the CPU oracle ``oracle/_build/liboracle.so`` (test infrastructure only).

g++ with OpenMP and without floating-point contraction, so that the
restatement evaluates every expression exactly as written. The baseline
x86-64 target is used so the library runs on any host it is copied to.
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_build" / "liboracle.so"
SRCS = [HERE / "oracle.cpp", HERE / "refine.cpp", HERE / "ply.cpp"]
DEPS = SRCS + [HERE.parent / "include" / "bsx.h", HERE.parent / "include" / "bsx_fmath.h"]


def build(force: bool = False) -> Path:
    OUT.parent.mkdir(exist_ok=True)
    if not force and OUT.exists() and all(d.stat().st_mtime <= OUT.stat().st_mtime for d in DEPS):
        return OUT
    tmp = OUT.with_suffix(".so.tmp")
    cmd = ["g++", "-O3", "-std=c++17", "-fopenmp", "-ffp-contract=off", "-fno-fast-math", "-fPIC", "-shared",
           *[str(x) for x in SRCS], "-o", str(tmp)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"oracle build failed:\n{res.stderr}")
    os.replace(tmp, OUT)
    return OUT


if __name__ == "__main__":
    print(build(force="-f" in sys.argv))

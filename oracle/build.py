"""Build the CPU oracle ``oracle/_build/liboracle.so`` (test infrastructure only).

g++ with OpenMP and without floating-point contraction, so that the
restatement evaluates every expression exactly as written. The baseline
x86-64 target is used so the library runs on any host it is copied to;
``build_native`` makes the CPU-baseline timing copy for the host at hand.
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


def _host_key() -> str:
    """Identifies the host CPU (model and feature flags), so a -march=native build made on one
    machine is never loaded on another."""
    import hashlib
    import platform

    text = platform.machine()
    try:
        with open("/proc/cpuinfo") as fh:
            for line in fh:
                if line.startswith(("model name", "flags", "Features")):
                    text += line
                    if line.startswith(("flags", "Features")):
                        break
    except OSError:
        pass
    return hashlib.sha1(text.encode()).hexdigest()[:12]


def build_native(force: bool = False) -> Path:
    """The timing copy used as the CPU baseline: the same sources with -march=native for the
    host that runs it (vector units and instruction set of that CPU). Contraction stays off and
    there is no fast-math, so every result is the same IEEE value as the portable build."""
    out = HERE / "_build" / f"liboracle_native-{_host_key()}.so"
    out.parent.mkdir(exist_ok=True)
    if not force and out.exists() and all(d.stat().st_mtime <= out.stat().st_mtime for d in DEPS):
        return out
    tmp = out.with_suffix(".so.tmp")
    cmd = ["g++", "-O3", "-march=native", "-std=c++17", "-fopenmp", "-ffp-contract=off", "-fno-fast-math", "-fPIC",
           "-shared", *[str(x) for x in SRCS], "-o", str(tmp)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"native oracle build failed:\n{res.stderr}")
    os.replace(tmp, out)
    return out


if __name__ == "__main__":
    print(build(force="-f" in sys.argv))

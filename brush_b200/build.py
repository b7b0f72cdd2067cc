"""Build the sm_100a shared library ``brush_b200/libbsx.so`` from ``csrc/*.cu``.

Each translation unit is compiled by nvcc in parallel and linked in-tree so the
library travels with the source tree. Floating-point contraction is disabled
(``-fmad=false``, ``-ffp-contract=off``): the pipeline's discrete decisions
(culling, tile counts, alpha cutoffs) must be reproducible bit-for-bit by a
host restatement compiled the same way. The image loss, checked by tolerance
and free of such decisions, is compiled with contraction (``CONTRACTED``).
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = PKG / "libbsx.so"

NVCC = os.environ.get("NVCC", shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CFLAGS = [
    "-O3", "-std=c++17", "-lineinfo", "-fmad=false", "-Xptxas", "-O3",
    "-Xcompiler", "-fPIC,-ffp-contract=off,-fvisibility=hidden",
    f"-I{ROOT / 'include'}",
]


def _sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted((ROOT / "include").glob("*.h"))


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


# Translation units whose arithmetic is checked by tolerance only and that take no
# bit-exact decision: there the compiler may contract multiply-adds. Every other
# unit keeps exact IEEE operations, because the CPU oracle (g++ -ffp-contract=off)
# restates its decisions (culling, tile counts, alpha and early-out tests, the
# raster backward's replay of the forward) or its results bit for bit.
CONTRACTED = {"loss.cu"}


def _compile(src: Path, verbose: bool) -> Path:
    obj = BUILD / (src.stem + ".o")
    if not _stale(obj, [src] + _headers() + [Path(__file__)]):
        return obj
    flags = [("-fmad=true" if f == "-fmad=false" and src.name in CONTRACTED else f) for f in CFLAGS]
    cmd = [NVCC, *ARCH, *flags, "-c", str(src), "-o", str(obj)]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{res.stdout}\n{res.stderr}")
    if verbose and res.stderr:
        sys.stderr.write(res.stderr)
    return obj


def build(verbose: bool = False, force: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    if force:
        for o in BUILD.glob("*.o"):
            o.unlink()
    srcs = _sources()
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose), srcs))
    if _stale(LIB, objs) or force:
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [NVCC, *ARCH, "-shared", "-o", str(tmp), *map(str, objs), "-Xcompiler", "-fPIC"]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
        os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv, force="-f" in sys.argv))

"""The C ABI library loads without a GPU, exports exactly what include/bsx.h declares,
and its host-only camera -> uniforms function agrees bit-for-bit with the oracle's."""
import ctypes as C
import math
import re
import subprocess
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent.parent


def _declared():
    text = (ROOT / "include" / "bsx.h").read_text()
    return sorted(set(re.findall(r"BSX_API\s+[\w\s\*]+?\b(bsx_\w+)\s*\(", text)))


def test_library_exports_every_declared_symbol(bsx_lib):
    lib = bsx_lib.lib()
    declared = _declared()
    assert len(declared) >= 19
    for name in declared:
        assert hasattr(lib, name), name
    out = subprocess.run(["nm", "-D", "--defined-only", str(bsx_lib.LIB_PATH)], capture_output=True, text=True).stdout
    exported = sorted(set(re.findall(r" T (bsx_\w+)", out)))
    assert exported == declared
    assert sorted(bsx_lib.SIGNATURES) == declared


def test_status_strings_and_abi(bsx_lib):
    lib = bsx_lib.lib()
    assert lib.bsx_abi_version() == 2
    assert lib.bsx_status_string(0) == b"ok"
    assert lib.bsx_status_string(4) == b"device wait timed out"
    assert lib.bsx_status_string(8) == b"malformed file"


def test_uniforms_match_oracle_bit_exact(bsx_lib, orc):
    from brush_b200.camera import Camera

    rng = np.random.default_rng(0)
    for k in range(20):
        pos = rng.normal(0, 5, 3)
        cam = Camera.look_at(tuple(pos), tuple(rng.normal(0, 1, 3)), math.radians(rng.uniform(20, 100)), 1297, 840)
        u = cam.project_uniforms(1297, 840, 3, 12345)
        o = orc.make_uniforms(cam, 1297, 840, 3, 12345)
        assert bytes(u) == bytes(o), k


def test_invalid_arguments_rejected_without_gpu(bsx_lib):
    lib = bsx_lib.lib()
    assert lib.bsx_render_fwd(None, None, 0, 0, None, None, None, 0, 0, 0, 0, None, None) == 1
    assert lib.bsx_make_project_uniforms(None, 1, 1, 0, 0, None) == 1

"""The CPU baseline's timing build (-march=native) computes the same values as the
portable oracle build the parity tests use: contraction is off and there is no
fast-math in either, so vectorisation for the host CPU changes no IEEE result.
Compared on one thread, where every sum has a fixed order."""
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent

_SCRIPT = r"""
import hashlib, sys
sys.path.insert(0, {root!r})
import numpy as np
from oracle import build, oracle as orc
if {native}:
    orc.use_library(build.build_native())
orc.set_threads(1)  # the raster backward's OpenMP atomics sum in scheduling order
from brush_b200.splats import clustered_scene, orbit_camera, random_gt
s = clustered_scene(6000, 3, "cpu", seed=8)
cam = orbit_camera(2, 5, 8.0, 160, 120)
r = orc.RenderResult(cam, (160, 120), s.transforms.numpy(), s.sh_coeffs.numpy(), s.raw_opacities.numpy())
vo = np.random.default_rng(1).normal(0, 1e-3, (120, 160, 4)).astype(np.float32)
vc = r.rasterize_bwd(vo, True)
h = hashlib.sha256()
for a in (r.image, r.isect_gid, r.tile_offsets, r.visible, *r.project_bwd(vc)):
    h.update(np.ascontiguousarray(a).tobytes())
chw = np.ascontiguousarray(r.image[..., :3].transpose(2, 0, 1))
gt = random_gt(120, 160, 3).numpy()
h.update(orc.loss_bwd(chw, gt, orc.loss_cfg(), np.ones_like(chw)).tobytes())
print(h.hexdigest())
"""


def _digest(native: bool) -> str:
    out = subprocess.run([sys.executable, "-c", _SCRIPT.format(root=str(ROOT), native=native)], capture_output=True,
                         text=True, timeout=600)
    assert out.returncode == 0, out.stderr
    return out.stdout.strip().splitlines()[-1]


def test_native_timing_build_matches_portable_build():
    assert _digest(True) == _digest(False)

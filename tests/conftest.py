import math
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); runs the sm_100a library")


@pytest.fixture(scope="session")
def orc():
    from oracle import build as obuild
    from oracle import oracle

    obuild.build()
    return oracle


@pytest.fixture(scope="session")
def bsx_lib():
    """The CUDA library, built in-tree if stale (nvcc cross-compiles without a GPU)."""
    from brush_b200 import build as bbuild

    bbuild.build()
    from brush_b200 import _lib

    return _lib


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from brush_b200 import build as bbuild

    bbuild.build()
    return torch.device("cuda:0")


def golden_case(name):
    from brush_b200.camera import Camera, focal_to_fov, fov_to_focal

    d = np.load(ROOT / "tests" / "golden" / f"{name}.npz")
    h, w, _ = d["out_img"].shape
    f = fov_to_focal(math.pi * 0.5, w)
    cam = Camera(fov_x=focal_to_fov(f, w), fov_y=focal_to_fov(f, h), position=(0.123, 0.456, -8.0),
                 rotation=(0.0, 0.0, 0.0, 1.0))
    t = np.concatenate([d["means"], d["quats"], d["scales"]], 1).astype(np.float32)
    return cam, (w, h), t, d["coeffs"].astype(np.float32), d["opacities"].astype(np.float32), d["out_img"]

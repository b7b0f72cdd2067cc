"""Splat value validation (crates/brush-render/src/gaussian_splats.rs:323-379,
validation.rs:6-85), on CPU tensors: NaN / Inf raise (the reference's
render_panics_loudly_on_nan_positions, tests/mod.rs:608-641, under its test
build), plausibility ranges are counted and logged only, shapes are checked."""
import logging
import math

import pytest
import torch

from brush_b200.splats import SplatValidationError, Splats, config1_scene, validate_gradient


def _sixteen(nan_at=None):
    n = 16
    means = torch.zeros(n, 3)
    if nan_at is not None:
        means.view(-1)[nan_at] = float("nan")
    quats = torch.tensor([[1.0, 0.0, 0.0, 0.0]]).repeat(n, 1)
    return Splats.from_parts(means, quats, torch.zeros(n, 3), torch.ones(n, 1, 3), torch.zeros(n))


def test_nan_position_raises():
    with pytest.raises(SplatValidationError, match="means"):
        _sixteen(nan_at=3).validate_values()


def test_valid_scene_passes():
    splats, _, _, _ = config1_scene("cpu", seed=1, n=2048)
    out = splats.validate_values()
    assert all(v["nan"] == 0 and v["inf"] == 0 for v in out.values())
    assert _sixteen().validate_values()["means"]["nan"] == 0


def test_ranges_are_logged_not_raised(caplog):
    s = _sixteen()
    s.sh_coeffs[0, 0, 0] = 10.0            # above the SH range
    s.raw_opacities[1] = -30.0             # below the raw-opacity range
    s.transforms[2, 7] = -15.0             # log-scale below -10, scale (3e-7) below 1e-6
    with caplog.at_level(logging.ERROR):
        out = s.validate_values()
    assert out["sh_coeffs"]["above_max"] == 1
    assert out["raw_opacity"]["below_min"] == 1
    assert out["log_scales"]["below_min"] == 1 and out["scales_plausible"]["below_min"] == 1
    assert "sh_coeffs" in caplog.text


def test_non_strict_reports_without_raising():
    s = _sixteen()
    s.raw_opacities[5] = math.inf
    out = s.validate_values(strict=False)
    assert out["raw_opacity"]["inf"] == 1


def test_gradient_validation():
    g = torch.zeros(16, 10)
    assert validate_gradient(g, "transforms")["nan"] == 0
    g[4, 2] = float("inf")
    with pytest.raises(SplatValidationError, match="gradient_transforms"):
        validate_gradient(g, "transforms")


def test_shape_checks():
    s = _sixteen()
    bad = Splats(s.transforms[:, :9], s.sh_coeffs, s.raw_opacities)
    with pytest.raises(SplatValidationError, match="10D"):
        bad.validate_values()
    bad = Splats(s.transforms, s.sh_coeffs[:8], s.raw_opacities)
    with pytest.raises(SplatValidationError, match="SH coeffs"):
        bad.validate_values()

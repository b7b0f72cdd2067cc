"""Non-pinhole camera models (crates/brush-render/src/kernels/camera_model/): Kannala-
Brandt 4, radial-tangential 8 and thin-prism fisheye, end to end on the GPU.

Forward: the whole pipeline bit-exact against the CPU oracle (same checks as the
pinhole renders). Backward: per-tensor gradients against the oracle (1e-3 of the
tensor's max; projection backward 1e-5 on identical inputs). The projection VJPs
themselves are checked against central differences of the GPU forward, as the
reference's finite-difference fuzz over camera models does
(crates/brush-bench-test/tests/finite_diff.rs:1082-1154).
"""
import dataclasses
import math

import numpy as np
import pytest
import torch

from test_gpu_render import _assert_pipeline_equal

pytestmark = pytest.mark.gpu

MODELS = {
    "kb4": (1, (0.05, -0.01, 0.002, -0.0004, 0.0, 0.0, 0.0, 0.0)),
    "rt8": (2, (-0.12, 0.03, -0.002, 0.01, -0.004, 0.0005, 0.001, -0.0015)),
    "tpf": (3, (0.04, -0.008, 0.001, -0.0002, 0.0008, -0.0006, 0.0009, -0.0007)),
}


def _camera(model, fov_deg, w, h, i=1, n=5):
    from brush_b200.splats import orbit_camera

    cam = orbit_camera(i, n, 8.0, w, h, fov_deg=fov_deg)
    kind, kp = MODELS[model]
    return dataclasses.replace(cam, camera_model=kind, model_params=kp)


@pytest.mark.parametrize("model", list(MODELS))
@pytest.mark.parametrize("fov", [60.0, 150.0])
def test_forward_pipeline_bit_exact(cuda, orc, model, fov):
    import brush_b200 as bsx
    from brush_b200.splats import clustered_scene

    if model == "rt8" and fov > 120:
        fov = 100.0  # the rational model folds over beyond this field of view
    splats = clustered_scene(20000, 3, "cpu", seed=41)
    cam = _camera(model, fov, 480, 320)
    r = orc.RenderResult(cam, (480, 320), splats.transforms.numpy(), splats.sh_coeffs.numpy(),
                         splats.raw_opacities.numpy())
    s = splats.to("cuda")
    out = bsx.render(cam, (480, 320), s.transforms, s.sh_coeffs, s.raw_opacities)
    torch.cuda.synchronize()
    assert r.num_visible > 1000 and r.num_intersections > 0
    _assert_pipeline_equal(r, out)


def test_fisheye_culls_by_angle_not_depth(cuda, orc):
    """A 200-degree KB4 camera keeps splats beside and behind the image plane (z < 0.01,
    which a pinhole culls) when their ray angle is inside half_max_render_fov."""
    import brush_b200 as bsx
    from brush_b200.camera import Camera
    from brush_b200.splats import Splats

    n = 2000
    rng = np.random.default_rng(3)
    ang = rng.uniform(0.0, 2 * math.pi, n)
    theta = rng.uniform(1.2, 1.75, n)  # 69-100 degrees off the optical axis
    d = 3.0
    means = np.stack([d * np.sin(theta) * np.cos(ang), d * np.sin(theta) * np.sin(ang), d * np.cos(theta)], 1)
    s = Splats.from_parts(torch.tensor(means, dtype=torch.float32), torch.tensor([[1.0, 0, 0, 0]] * n),
                          torch.full((n, 3), -3.0), torch.full((n, 1, 3), 0.5), torch.full((n,), 2.0))
    cam = Camera(fov_x=math.radians(200.0), fov_y=math.radians(200.0), camera_model=1,
                 model_params=MODELS["kb4"][1])
    r = orc.RenderResult(cam, (256, 256), s.transforms.numpy(), s.sh_coeffs.numpy(), s.raw_opacities.numpy())
    g = s.to("cuda")
    out = bsx.render(cam, (256, 256), g.transforms, g.sh_coeffs, g.raw_opacities)
    torch.cuda.synchronize()
    _assert_pipeline_equal(r, out)
    vis = r.depth_order
    assert (means[vis, 2] < 0.01).sum() > 50


@pytest.mark.parametrize("model", list(MODELS))
def test_backward_matches_oracle(cuda, orc, model):
    import brush_b200 as bsx
    from brush_b200.splats import clustered_scene

    from test_gpu_backward import _rel

    s = clustered_scene(12000, 3, "cpu", seed=5)
    cam = _camera(model, 90.0, 320, 240, i=2)
    size = (320, 240)
    r = orc.RenderResult(cam, size, s.transforms.numpy(), s.sh_coeffs.numpy(), s.raw_opacities.numpy())
    g = s.to("cuda")
    bsx.render(cam, size, g.transforms, g.sh_coeffs, g.raw_opacities)
    rng = np.random.default_rng(1)
    v_output = rng.normal(0, 1e-3, (size[1], size[0], 4)).astype(np.float32)
    vc_gpu = bsx.rasterize_bwd(torch.from_numpy(v_output).cuda(), True).cpu().numpy()[:, :11]
    vc_orc = r.rasterize_bwd(v_output, True)
    for lanes in [(0, 1), (2, 3, 4), (5, 6, 7), (8,), (9,)]:
        assert _rel(vc_gpu[:, lanes], vc_orc[:, lanes]) <= 1e-3, lanes
    vc12 = np.zeros((s.num_splats, 12), np.float32)
    vc12[:, :11] = vc_orc
    grads = bsx.project_bwd(torch.from_numpy(vc12).cuda(), s.num_splats, s.sh_coeffs_per_splat)
    vt, vs, vo, _ = r.project_bwd(vc_orc)
    assert np.abs(vt).max() > 0
    for got, ref in [(grads.v_transforms, vt), (grads.v_coeffs, vs), (grads.v_raw_opac, vo)]:
        assert _rel(got.cpu().numpy(), ref) <= 1e-5


STEPS = (1e-4, 2e-4, 5e-4, 1e-3)


def _fd_scene():
    means = [[0.35, -0.22, 0.05], [-0.45, 0.4, 0.15], [0.1, 0.48, -0.25], [-0.38, -0.3, 0.12]]
    rots = [[0.85, 0.15, 0.07, 0.02], [0.72, 0.18, 0.27, 0.12], [0.55, 0.37, 0.33, 0.18], [0.78, 0.12, 0.08, 0.23]]
    log_scales = [[-1.45, -1.55, -1.62], [-1.52, -1.38, -1.33], [-1.68, -1.52, -1.41], [-1.33, -1.58, -1.49]]
    dc = [[0.42, 0.58, 0.47], [0.62, 0.38, 0.33], [0.37, 0.52, 0.63], [0.48, 0.47, 0.52]]
    op = [2.4, 2.1, 2.3, 2.5]
    t = np.concatenate([np.array(means), np.array(rots), np.array(log_scales)], 1).astype(np.float32)
    return t, np.array(dc, np.float32).reshape(4, 1, 3), np.array(op, np.float32)


@pytest.mark.parametrize("model", list(MODELS))
def test_projection_vjp_matches_central_differences(cuda, model):
    """d mean(image) / d (mean, rotation, log-scale) of splats seen off-axis through the
    distorting lens (smooth alpha cutoff), against central differences of the forward."""
    import brush_b200 as bsx
    from brush_b200.camera import Camera

    kind, kp = MODELS[model]
    cam = Camera(fov_x=1.4, fov_y=1.4, position=(0.0, 0.0, -2.2), rotation=(0.0, 0.0, 0.0, 1.0),
                 camera_model=kind, model_params=kp)
    size = (48, 48)
    t, sh, op = _fd_scene()

    def render(tt):
        return bsx.render(cam, size, torch.from_numpy(tt).cuda(), torch.from_numpy(sh).cuda(),
                          torch.from_numpy(op).cuda(), raster_pass=bsx._lib.PASS_BACKWARD_SMOOTH_CUTOFF)

    out = render(t)
    v_out = torch.full((size[1], size[0], 4), 1.0 / (size[0] * size[1] * 4), device="cuda")
    vc = bsx.rasterize_bwd(v_out, False)
    vt = bsx.project_bwd(vc, 4, 1).v_transforms.cpu().numpy()
    for splat in range(4):
        for col in (0, 1, 2, 4, 8):
            def f(h):
                tt = t.copy()
                tt[splat, col] += h
                return float(render(tt).out_img.double().mean())

            num = float(np.median([(f(h) - f(-h)) / (2 * h) for h in STEPS]))
            an = float(vt[splat, col])
            scale = max(abs(num), abs(an), 1e-8)
            assert abs(num - an) <= 5e-5 + 0.01 * scale, (model, splat, col, num, an)

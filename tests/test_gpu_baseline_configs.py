"""Oracle parity at the benchmark configurations' own sizes.

config 2 (the headline: 1M splats, SH degree 3, 1920x1080), a config-3-shaped step
(3M splats, SH degree 3, 1297x840, a hemisphere camera) and config 5's forward-only
viewer render (6M splats, SH degree 3, 3840x2160), each on seeded CPU-generated
inputs fed to both the sm_100a pipeline and the CPU oracle.

Bars (the same as the small-scene tests):
- bit-exact: per-splat tile counts, depth order, the inclusive count scan, sorted
  (tile, splat) intersection arrays, tile ranges (incl. the backward-pass shortening),
  projected rows, max radii, visibility; the packed forward image;
- float image: max |diff| <= 1e-4;
- gradients: per parameter group max |g - g_ref| <= 1e-3 * max |g_ref| (the raster
  backward sums with float atomics in scheduling order);
- the training step's fused projection backward + AdamScaled (one kernel), on its own
  inputs (the step's raster-backward rows): gradients <= 1e-5 relative, and every
  updated parameter within 1e-6 of the oracle's AdamScaled applied to the same gradients;
- the whole step against the oracle chain, every element: Adam's first update is
  lr * g / (|g| + eps), so an element may move differently only where the two gradients'
  update directions differ, which the test allows for and requires to happen only where
  the oracle's gradient is within the gradient tolerance of zero.
"""
import numpy as np
import pytest
import torch

from test_gpu_render import _assert_pipeline_equal

pytestmark = pytest.mark.gpu


def _rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


def _scene(name):
    from brush_b200 import splats as S

    if name == "cfg2":
        splats, cam, size, gt = S.config2_scene("cpu", seed=2)
        return splats, cam, size, gt
    if name == "cfg3":
        splats = S.clustered_scene(3_000_000, 3, "cpu", seed=3)
        w, h = 1297, 840
        cam = S.hemisphere_cameras(200, 8.0, w, h, seed=3)[0]
        return splats, cam, (w, h), S.random_gt(h, w, 1003, "cpu")
    raise ValueError(name)


def _oracle_chain(orc, r, gt, w, h):
    """Loss gradient of 0.8 L1 + 0.2 (1 - SSIM) on the oracle render, then its backward."""
    chw = np.ascontiguousarray(r.image[..., :3].transpose(2, 0, 1))
    oc = orc.loss_cfg(0.8, -0.2)
    loss = float(orc.loss_fwd(chw, gt, oc).astype(np.float64).mean())
    dl = np.full((3, h, w), np.float32(1.0 / (3 * h * w)), np.float32)
    vo = np.zeros((h, w, 4), np.float32)
    vo[..., :3] = orc.loss_bwd(chw, gt, oc, dl).transpose(1, 2, 0)
    vc = r.rasterize_bwd(vo, True)
    return loss, vo, vc


@pytest.mark.parametrize("name", ["cfg2", "cfg3"])
def test_render_and_backward_at_config_size(cuda, orc, name):
    import brush_b200 as bsx

    splats, cam, size, gt = _scene(name)
    w, h = size
    t, sh, op = splats.transforms.numpy(), splats.sh_coeffs.numpy(), splats.raw_opacities.numpy()
    r = orc.RenderResult(cam, size, t, sh, op)
    g = splats.to("cuda")
    out = bsx.render(cam, size, g.transforms, g.sh_coeffs, g.raw_opacities)
    torch.cuda.synchronize()
    assert r.num_visible > 100_000 and r.num_intersections > 1_000_000
    _assert_pipeline_equal(r, out)
    # backward from the oracle's loss gradient on identical inputs
    _, vo, vc_ref = _oracle_chain(orc, r, gt.numpy(), w, h)
    vc = bsx.rasterize_bwd(torch.from_numpy(vo).cuda(), True).cpu().numpy()[:, :11]
    for lanes, lane_name in [((0, 1), "xy"), ((2, 3, 4), "conic"), ((5, 6, 7), "rgb"), ((8,), "alpha"),
                             ((9,), "refine")]:
        assert _rel(vc[:, lanes], vc_ref[:, lanes]) <= 1e-3, lane_name
    vc12 = np.zeros((splats.num_splats, 12), np.float32)
    vc12[:, :11] = vc_ref
    grads = bsx.project_bwd(torch.from_numpy(vc12).cuda(), splats.num_splats, splats.sh_coeffs_per_splat)
    vt, vs, vop, vr = r.project_bwd(vc_ref)
    for got, want, gname in [(grads.v_transforms, vt, "transforms"), (grads.v_coeffs, vs, "sh"),
                             (grads.v_raw_opac, vop, "opacity"), (grads.v_refine_weight, vr, "refine")]:
        assert _rel(got.cpu().numpy(), want) <= 1e-5, gname


@pytest.mark.parametrize("name", ["cfg2", "cfg3"])
def test_fused_training_step_at_config_size(cuda, orc, name):
    """One bsx_train_step with the reference rate table (SH degree 3: the projection backward
    with AdamScaled fused, the benchmarked kernel) against the oracle, every element."""
    import brush_b200 as bsx

    splats, cam, size, gt = _scene(name)
    w, h = size
    n, c = splats.num_splats, splats.sh_coeffs_per_splat
    p0 = [splats.transforms.numpy().copy(), splats.sh_coeffs.numpy().reshape(n, 3 * c).copy(),
          splats.raw_opacities.numpy().reshape(n, 1).copy()]
    g = splats.to("cuda")
    cfg = bsx.TrainConfig(mean_noise=False)
    tr = bsx.SplatTrainer(cfg, g, keep_gradients=True)
    st = tr.step(cam, size, gt.cuda(), g)
    torch.cuda.synchronize()
    p_gpu = [g.transforms.cpu().numpy(), g.sh_coeffs.cpu().numpy().reshape(n, 3 * c),
             g.raw_opacities.cpu().numpy().reshape(n, 1)]
    g_gpu = [tr.grads.v_transforms.cpu().numpy(), tr.grads.v_coeffs.cpu().numpy().reshape(n, 3 * c),
             tr.grads.v_raw_opac.cpu().numpy().reshape(n, 1)]
    # the step's own raster-backward rows (input of its fused projection backward)
    vc_gpu = tr.native.raster_grads().cpu().numpy()[:, :11].copy()
    tr.close()

    # rates of the first optimizer step (burn ExponentialLrScheduler: the initial rates)
    lr_mean = cfg.lr_mean * tr.median_scale
    assert st.lr_mean == float(np.float32(lr_mean))
    groups = [(1.0, [lr_mean] * 3 + [cfg.lr_rotation] * 4 + [cfg.lr_scale] * 3, False),
              (cfg.lr_coeffs_dc, [1.0] * 3 + [1.0 / cfg.lr_coeffs_sh_scale] * (3 * c - 3), True),
              (cfg.lr_opac, None, False)]

    def adam(params, grads):
        out = []
        for (lr, cols, red), p_, g_ in zip(groups, params, grads):
            q = p_.copy()
            m = np.zeros_like(q)
            v = np.zeros(n, np.float32) if red else np.zeros_like(q)
            orc.adam(q, g_, m, v, lr, cols, red, step=1)
            out.append(q)
        return out

    # the fused kernel on identical inputs: projection backward, then AdamScaled
    r = orc.RenderResult(cam, size, p0[0], p0[1].reshape(n, c, 3), p0[2].reshape(n))
    vt, vs, vop, _ = r.project_bwd(vc_gpu)
    for got, want, gname in [(g_gpu[0], vt, "transforms"), (g_gpu[1], vs.reshape(n, -1), "sh"),
                             (g_gpu[2], vop.reshape(n, 1), "opacity")]:
        assert _rel(got, want) <= 1e-5, gname
    p_same = adam(p0, g_gpu)
    for got, want, gname in zip(p_gpu, p_same, ("transforms", "sh", "opacity")):
        tol = 1e-6 * np.maximum(np.abs(want), 1.0)
        assert (np.abs(got - want) <= tol).all(), gname

    # the whole step against the oracle chain (render, loss, backward, AdamScaled)
    loss, _, vc_ref = _oracle_chain(orc, r, gt.numpy(), w, h)
    assert abs(float(st.loss.item()) - loss) <= 1e-5 * abs(loss)
    vt, vs, vop, _ = r.project_bwd(vc_ref)
    g_ref = [vt, vs.reshape(n, -1), vop.reshape(n, 1)]
    for got, want, gname in zip(g_gpu, g_ref, ("transforms", "sh", "opacity")):
        assert _rel(got, want) <= 1e-3, gname
    p_ref = adam(p0, g_ref)
    for k, ((lr, cols, red), got, want) in enumerate(zip(groups, p_gpu, p_ref)):
        lr_col = np.float64(lr) * (np.asarray(cols, np.float64) if cols is not None else 1.0)
        dev = np.abs(got.astype(np.float64) - want)
        tight = 1e-6 * np.maximum(np.abs(want), 1.0) + 1e-6 * lr_col
        if red:
            # SH rows move by u = g / rms(row g) (one second moment per row), continuous in the
            # gradient: |u' - u| <= (|g'_k - g_k| + |u_k| max_j |g'_j - g_j|) / rms'
            gr, gg = g_ref[k].astype(np.float64), g_gpu[k].astype(np.float64)
            rms = np.minimum(np.sqrt((gr * gr).mean(axis=1, keepdims=True)),
                             np.sqrt((gg * gg).mean(axis=1, keepdims=True)))
            d = np.abs(gg - gr)
            u = np.abs(gr) / np.where(rms > 0, rms, 1.0)
            bound = (d + u * d.max(axis=1, keepdims=True)) / np.where(rms > 0, rms, 1.0)
            assert (dev <= tight + lr_col * bound * 1.01).all(), "sh"
            continue
        # first-step Adam direction u(g) = g / (|g| + eps) of each side's gradient
        eps = 1e-15
        u_ref = g_ref[k] / (np.abs(g_ref[k]).astype(np.float64) + eps)
        u_gpu = g_gpu[k] / (np.abs(g_gpu[k]).astype(np.float64) + eps)
        du = np.abs(u_gpu - u_ref)
        assert (dev <= tight + lr_col * du * 1.001).all(), ("element outside the direction allowance", k)
        moved = du > 1e-3
        gmax = np.abs(g_ref[k]).max(axis=0, keepdims=True)
        assert (np.abs(g_ref[k])[moved] <= (1e-3 * np.broadcast_to(gmax, moved.shape))[moved]).all(), k


def test_config5_forward_viewer_render_bit_exact(cuda, orc):
    """Config 5's forward-only pass (6M splats, SH degree 3, 3840x2160, packed RGBA8)."""
    import brush_b200 as bsx
    from brush_b200 import splats as S

    splats, size = S.config5_scene("cpu", seed=5)
    cam = S.circle_cameras(120, 8.0, size[0], size[1])[0]
    r = orc.RenderResult(cam, size, splats.transforms.numpy(), splats.sh_coeffs.numpy(),
                         splats.raw_opacities.numpy(), raster_pass=0)
    g = splats.to("cuda")
    out = bsx.render(cam, size, g.transforms, g.sh_coeffs, g.raw_opacities, raster_pass=0)
    torch.cuda.synchronize()
    assert r.num_visible > 1_000_000 and r.num_intersections > 1_000_000
    _assert_pipeline_equal(r, out, bwd=False)

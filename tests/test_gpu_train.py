"""The native whole-step trainer (bsx_train_step) against the same step composed
from the public operators, with the reference learning-rate table.

The raster backward accumulates with float atomics, so two runs of the same
step may differ in the last bits of the gradients. The composed step therefore
reuses the native step's own gradients (read back after each step): what is
compared is the orchestration - rates, groups, column scales, moments, time
step - and it must match bit for bit.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _burn_rates(cfg, k, median):
    """Rates of optimizer step k (1-based): burn ExponentialLrScheduler, first step = initial rate."""
    t = cfg.total_train_iters
    gm = (cfg.lr_mean_end / cfg.lr_mean) ** (1.0 / t)
    gs = (cfg.lr_scale_end / cfg.lr_scale) ** (1.0 / t)
    pm, ps = cfg.lr_mean / gm, cfg.lr_scale / gs
    for _ in range(k):
        pm *= gm
        ps *= gs
    return pm * median, ps


@pytest.mark.parametrize("camera_model", [0, 1])
def test_native_step_matches_composed_step(cuda, camera_model):
    """camera_model 1: Kannala-Brandt 4, which takes the fused step's non-pinhole kernel."""
    import dataclasses

    import brush_b200 as bsx
    from brush_b200.adam import AdamGroup, AdamScaled
    from brush_b200.splats import clustered_scene, orbit_camera, random_gt

    splats = clustered_scene(20000, 3, "cpu", seed=11).to("cuda")
    w, h = 192, 128
    kp = (0.05, -0.01, 0.002, -0.0004, 0.0, 0.0, 0.0, 0.0)
    cams = [dataclasses.replace(orbit_camera(i, 3, 8.0, w, h), camera_model=camera_model, model_params=kp)
            for i in range(3)]
    gts = [random_gt(h, w, 40 + i, "cpu").cuda() for i in range(3)]
    cfg = bsx.TrainConfig(mean_noise=False)
    comp = splats.clone()
    tr = bsx.SplatTrainer(cfg, splats, keep_gradients=True)
    fused = splats.clone()
    tr_f = bsx.SplatTrainer(cfg, fused)  # gradients not written: same parameters
    n, c = comp.num_splats, comp.sh_coeffs_per_splat
    opt = AdamScaled(epsilon=1e-15)
    groups = None
    for k in range(1, 4):
        st = tr.step(cams[k - 1], (w, h), gts[k - 1], splats)
        tr_f.step(cams[k - 1], (w, h), gts[k - 1], fused)
        grads = [tr.grads.v_transforms.clone(), tr.grads.v_coeffs.reshape(n, 3 * c).clone(),
                 tr.grads.v_raw_opac.reshape(n, 1).clone()]
        lr_mean, lr_scale = _burn_rates(cfg, k, tr.median_scale)
        assert st.lr_mean == float(np.float32(lr_mean))
        assert tr.step_count == k
        tscale = [lr_mean] * 3 + [cfg.lr_rotation] * 4 + [lr_scale] * 3
        sh_cols = [1.0] * 3 + [1.0 / cfg.lr_coeffs_sh_scale] * (3 * c - 3)
        params = (comp.transforms, comp.sh_coeffs.view(n, 3 * c), comp.raw_opacities.view(n, 1))
        if groups is None:
            groups = [AdamGroup(params[0], grads[0], 1.0, tscale),
                      AdamGroup(params[1], grads[1], cfg.lr_coeffs_dc, sh_cols, reduce_moment_2=True),
                      AdamGroup(params[2], grads[2], cfg.lr_opac)]
        for g, gr in zip(groups, grads):
            g.grad = gr
        groups[0].col_scale = tscale
        opt.step(groups)
        torch.cuda.synchronize()
        for a, b in ((splats.transforms, comp.transforms), (splats.sh_coeffs, comp.sh_coeffs),
                     (splats.raw_opacities, comp.raw_opacities)):
            np.testing.assert_array_equal(a.cpu().numpy(), b.cpu().numpy())
        # the gradients' last bits depend on atomic order, so the trainer without
        # gradient write-back is compared within the step's own float noise
        for a, b in ((splats.transforms, fused.transforms), (splats.sh_coeffs, fused.sh_coeffs)):
            d = (a - b).abs().max().item()
            assert d <= 1e-5 * max(a.abs().max().item(), 1.0), d
        assert st.num_visible > 0 and st.num_intersections > 0
        assert np.isfinite(float(st.loss.item()))
    tr_f.close()
    rec = tr.record
    vis = rec.vis_weight.cpu().numpy()
    assert set(np.unique(vis)).issubset({0.0, 1.0, 2.0, 3.0}) and vis.max() >= 1.0
    assert (rec.refine_weight_norm.cpu().numpy() >= tr.grads.v_refine_weight.cpu().numpy()).all()
    assert (rec.max_screen_size.cpu().numpy() >= 0).all()
    tr.close()


def test_native_step_uniform_rate_and_empty_view(cuda):
    """uniform_lr skips the schedule; a camera that sees nothing leaves the splats unchanged."""
    import brush_b200 as bsx
    from brush_b200.camera import Camera
    from brush_b200.splats import config1_scene

    splats, cam, size, gt = config1_scene("cuda", seed=2)
    before = splats.clone()
    tr = bsx.SplatTrainer(bsx.TrainConfig(uniform_lr=1e-3, mean_noise=False), splats, gather_stats=False)
    away = Camera.look_at((0.0, 0.0, 3.0), target=(0.0, 0.0, 10.0), img_w=size[0], img_h=size[1])
    st = tr.step(away, size, gt.cuda(), splats)
    assert st.num_visible == 0 and st.num_intersections == 0 and st.lr_mean == pytest.approx(1e-3)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(splats.transforms.cpu().numpy(), before.transforms.cpu().numpy())
    st = tr.step(cam, size, gt.cuda(), splats)
    assert st.num_visible > 0
    assert not np.array_equal(splats.transforms.cpu().numpy(), before.transforms.cpu().numpy())
    tr.close()

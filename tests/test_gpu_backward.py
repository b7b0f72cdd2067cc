"""Backward / loss / optimizer parity against the CPU oracle.

Tolerances: gradients per parameter tensor max|g - g_ref| <= 1e-3 * max|g_ref|
(the only difference is the order of the per-tile atomic accumulation);
loss map / loss gradient / Adam: 1e-5 relative.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    scale = max(np.abs(b).max(), 1e-30)
    return float(np.abs(a - b).max() / scale)


def _scene(seed=5, n=12000, deg=3, w=320, h=240):
    from brush_b200.splats import clustered_scene, orbit_camera

    s = clustered_scene(n, deg, "cpu", seed=seed)
    cam = orbit_camera(seed % 5, 5, 8.0, w, h)
    return s, cam, (w, h)


@pytest.mark.parametrize("refine", [True, False])
def test_rasterize_and_project_backward(cuda, orc, refine):
    import brush_b200 as bsx

    s, cam, size = _scene()
    bg = (0.1, 0.05, 0.2)
    r = orc.RenderResult(cam, size, s.transforms.numpy(), s.sh_coeffs.numpy(), s.raw_opacities.numpy(), bg=bg)
    g = s.to("cuda")
    out = bsx.render(cam, size, g.transforms, g.sh_coeffs, g.raw_opacities, background=bg)
    rng = np.random.default_rng(0)
    v_output = rng.normal(0, 1e-3, (size[1], size[0], 4)).astype(np.float32)
    vc_gpu = bsx.rasterize_bwd(torch.from_numpy(v_output).cuda(), refine).cpu().numpy()[:, :11]
    vc_orc = r.rasterize_bwd(v_output, refine)
    for lanes, name in [((0, 1), "xy"), ((2, 3, 4), "conic"), ((5, 6, 7), "rgb"), ((8,), "alpha"), ((9,), "refine")]:
        if name == "refine" and not refine:
            assert (vc_gpu[:, 9] == 0).all()
            continue
        assert _rel(vc_gpu[:, lanes], vc_orc[:, lanes]) <= 1e-3, name
    # projection backward on identical inputs
    vc12 = np.zeros((s.num_splats, 12), np.float32)
    vc12[:, :11] = vc_orc
    grads = bsx.project_bwd(torch.from_numpy(vc12).cuda(), s.num_splats, s.sh_coeffs_per_splat)
    vt, vs, vo, vr = r.project_bwd(vc_orc)
    for got, ref, name in [(grads.v_transforms[:, 0:3], vt[:, 0:3], "means"), (grads.v_transforms[:, 3:7], vt[:, 3:7], "quats"),
                           (grads.v_transforms[:, 7:10], vt[:, 7:10], "log_scales"), (grads.v_coeffs, vs, "sh"),
                           (grads.v_raw_opac, vo, "opacity"), (grads.v_refine_weight, vr, "refine")]:
        assert _rel(got.cpu().numpy(), ref) <= 1e-5, name


@pytest.mark.parametrize("cfg", [dict(), dict(composite_bg=(0.3, 0.2, 0.1)), dict(mask=True),
                                 dict(l1_weight=1.0, ssim_weight=0.0)])
def test_loss_forward_backward(cuda, orc, cfg):
    from brush_b200.loss import ImageLossConfig, image_loss_backward, image_loss_forward

    rng = np.random.default_rng(1)
    h, w = 77, 131
    pred = rng.uniform(0, 1, (3, h, w)).astype(np.float32)
    gt = rng.integers(0, 2**32, (h, w), dtype=np.uint64).astype(np.uint32).view(np.int32)
    dl = rng.normal(0, 1, (3, h, w)).astype(np.float32)
    c = ImageLossConfig(**{"l1_weight": 0.8, "ssim_weight": -0.2, **cfg})
    oc = orc.loss_cfg(c.l1_weight, c.ssim_weight, c.composite_bg, c.mask)
    m = image_loss_forward(torch.from_numpy(pred).cuda(), torch.from_numpy(gt).cuda(), c).cpu().numpy()
    assert _rel(m, orc.loss_fwd(pred, gt, oc)) <= 1e-5
    d = image_loss_backward(torch.from_numpy(pred).cuda(), torch.from_numpy(gt).cuda(), torch.from_numpy(dl).cuda(),
                            c).cpu().numpy()
    assert _rel(d, orc.loss_bwd(pred, gt, oc, dl)) <= 1e-5


def test_loss_alpha_channel(cuda, orc):
    from brush_b200.loss import ImageLossConfig, image_loss_backward, image_loss_forward

    rng = np.random.default_rng(2)
    h, w = 40, 50
    pred = rng.uniform(0, 1, (4, h, w)).astype(np.float32)
    gt = rng.integers(0, 2**32, (h, w), dtype=np.uint64).astype(np.uint32).view(np.int32)
    dl = rng.normal(0, 1, (4, h, w)).astype(np.float32)
    c = ImageLossConfig()
    oc = orc.loss_cfg(0.8, -0.2)
    m = image_loss_forward(torch.from_numpy(pred).cuda(), torch.from_numpy(gt).cuda(), c).cpu().numpy()
    assert _rel(m, orc.loss_fwd(pred, gt, oc)) <= 1e-5
    d = image_loss_backward(torch.from_numpy(pred).cuda(), torch.from_numpy(gt).cuda(), torch.from_numpy(dl).cuda(),
                            c).cpu().numpy()
    assert _rel(d, orc.loss_bwd(pred, gt, oc, dl)) <= 1e-5


@pytest.mark.parametrize("h,w,cfg", [
    (96, 160, {}),
    (75, 131, {}),
    (33, 70, {"composite_bg": (0.2, 0.5, 0.9), "mask": True}),
    (40, 47, {"l1_weight": 1.0, "ssim_weight": 0.0}),
    (1, 1, {}),
    (70, 1, {}),
    (9, 301, {"composite_bg": (0.7, 0.1, 0.3)}),
], ids=["aligned", "ragged", "composite_mask", "l1_only", "single_pixel", "single_column", "wide_strip"])
def test_fused_loss_matches_mean_and_gradient(cuda, orc, h, w, cfg):
    from brush_b200.loss import ImageLossConfig, image_loss_fused

    rng = np.random.default_rng(3)
    img = rng.uniform(0, 1, (h, w, 4)).astype(np.float32)
    gt = rng.integers(0, 2**32, (h, w), dtype=np.uint64).astype(np.uint32).view(np.int32)
    c = ImageLossConfig(**cfg)
    loss, vout = image_loss_fused(torch.from_numpy(img).cuda(), torch.from_numpy(gt).cuda(), c)
    oc = orc.loss_cfg(c.l1_weight, c.ssim_weight, c.composite_bg, c.mask)
    chw = np.ascontiguousarray(img[..., :3].transpose(2, 0, 1))
    ref_map = orc.loss_fwd(chw, gt, oc)
    assert abs(float(loss.item()) - float(ref_map.astype(np.float64).mean())) <= 1e-5 * abs(ref_map.mean()) + 1e-7
    dl = np.full((3, h, w), np.float32(1.0 / (3 * h * w)), np.float32)
    ref_g = orc.loss_bwd(chw, gt, oc, dl).transpose(1, 2, 0)
    v = vout.cpu().numpy()
    assert _rel(v[..., :3], ref_g) <= 1e-5
    assert (v[..., 3] == 0).all()


def test_adam_groups(cuda, orc):
    from brush_b200.adam import AdamGroup, AdamScaled

    rng = np.random.default_rng(4)
    n, c = 1000, 16
    pt = rng.normal(0, 1, (n, 10)).astype(np.float32)
    ps = rng.normal(0, 1, (n, 3 * c)).astype(np.float32)
    po = rng.normal(0, 1, (n, 1)).astype(np.float32)
    tscale = [1e-3] * 3 + [2e-3] * 4 + [7e-3] * 3
    sh_cols = [1.0] * 3 + [0.1] * (3 * c - 3)
    groups = [AdamGroup(torch.from_numpy(pt.copy()).cuda(), None, 1.0, tscale),
              AdamGroup(torch.from_numpy(ps.copy()).cuda(), None, 2e-3, sh_cols, reduce_moment_2=True),
              AdamGroup(torch.from_numpy(po.copy()).cuda(), None, 0.012)]
    state = [(pt.copy(), np.zeros_like(pt), np.zeros_like(pt)), (ps.copy(), np.zeros_like(ps), np.zeros(n, np.float32)),
             (po.copy(), np.zeros_like(po), np.zeros_like(po))]
    opt = AdamScaled()
    for step in range(1, 4):
        grads = [rng.normal(0, 1, x.shape).astype(np.float32) for x in (pt, ps, po)]
        for gg, gr in zip(groups, grads):
            gg.grad = torch.from_numpy(gr).cuda()
        opt.step(groups, grad_scale=0.5)
        for (p, m, v), gr, gg in zip(state, grads, groups):
            orc.adam(p, gr, m, v, gg.lr, gg.col_scale, gg.reduce_moment_2, step=step, grad_scale=0.5)
    for (p, _, _), gg in zip(state, groups):
        assert np.abs(gg.param.cpu().numpy() - p).max() <= 1e-6 * max(1.0, np.abs(p).max())


def test_train_step_matches_oracle_chain(cuda, orc):
    """Config-1 step (uniform lr 1e-3): render -> 0.8 L1 + 0.2 (1-SSIM) -> backward -> Adam."""
    import brush_b200 as bsx
    from brush_b200.splats import config1_scene

    splats, cam, size, gt = config1_scene("cpu", seed=1)
    p0 = splats.clone()
    g = splats.to("cuda")
    trainer = bsx.SplatTrainer(bsx.TrainConfig(uniform_lr=1e-3, mean_noise=False), g, gather_stats=False)
    stats = trainer.step(cam, size, gt.cuda(), g)
    torch.cuda.synchronize()
    # oracle chain
    r = orc.RenderResult(cam, size, p0.transforms.numpy(), p0.sh_coeffs.numpy(), p0.raw_opacities.numpy())
    w, h = size
    chw = np.ascontiguousarray(r.image[..., :3].transpose(2, 0, 1))
    oc = orc.loss_cfg(0.8, -0.2)
    ref_loss = float(orc.loss_fwd(chw, gt.numpy(), oc).astype(np.float64).mean())
    assert abs(float(stats.loss.item()) - ref_loss) <= 1e-5 * abs(ref_loss)
    dl = np.full((3, h, w), np.float32(1.0 / (3 * h * w)), np.float32)
    vo = np.zeros((h, w, 4), np.float32)
    vo[..., :3] = orc.loss_bwd(chw, gt.numpy(), oc, dl).transpose(1, 2, 0)
    vc = r.rasterize_bwd(vo, True)
    vt, vs, vop, _ = r.project_bwd(vc)
    n = p0.num_splats
    for param, grad, gpu_p, reduce in [(p0.transforms.numpy().copy(), vt, g.transforms, False),
                                       (p0.sh_coeffs.numpy().reshape(n, -1).copy(), vs.reshape(n, -1), g.sh_coeffs, True),
                                       (p0.raw_opacities.numpy().reshape(n, 1).copy(), vop.reshape(n, 1), g.raw_opacities,
                                        False)]:
        before = param.copy()
        m = np.zeros_like(param)
        v = np.zeros(n, np.float32) if reduce else np.zeros_like(param)
        orc.adam(param, grad, m, v, 1e-3, None, reduce, step=1)
        got = gpu_p.cpu().numpy().reshape(param.shape)
        moved = np.abs(param - before).max()
        assert moved > 0
        # Adam's first step is sign-like (|update| = lr where g != 0), so compare per element
        # where the reference gradient is not vanishingly small.
        big = np.abs(grad) > 1e-3 * np.abs(grad).max()
        assert np.abs(got - param)[big].max() <= 1e-3 * moved + 1e-7


@pytest.mark.parametrize("cols", [48, 12, 75])
def test_adam_bit_reproducible(cuda, cols):
    """Equal inputs give bit-equal parameters and moments on every run (data-parallel replicas rely on it)."""
    from brush_b200.adam import AdamGroup, AdamScaled

    p0 = np.random.default_rng(cols).normal(0, 1, (50000, cols)).astype(np.float32)
    grads = [torch.from_numpy(np.random.default_rng(100 + s).normal(0, 1, p0.shape).astype(np.float32)).cuda()
             for s in range(2)]
    outs = []
    for _ in range(3):
        g = AdamGroup(torch.from_numpy(p0.copy()).cuda(), None, 1e-3, reduce_moment_2=True)
        opt = AdamScaled()
        for gr in grads:
            g.grad = gr
            opt.step([g])
        outs.append([t.cpu().numpy() for t in (g.param, g.m, g.v)])
    for o in outs[1:]:
        for a, b in zip(o, outs[0]):
            np.testing.assert_array_equal(a, b)

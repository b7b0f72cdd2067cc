"""The mean-noise injection on the GPU (crates/brush-train/src/train.rs:1095-1169).

- the operator bsx_mean_noise_step equals the oracle restatement value for value;
- inside bsx_train_step (the default, gated on the RefineRecord visibility accumulated
  since the last refine) the step equals, over three steps and value for value, the same
  step composed from the library's AdamScaled on the step's own gradients followed by the
  oracle's noise step with the trainer's visibility statistic;
- with the step's own visibility as the gate (mrnf_noise_injection off) likewise.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_noise_operator_matches_oracle(cuda, orc):
    from brush_b200 import _lib
    from brush_b200._context import context, ptr

    rng = np.random.default_rng(11)
    n = 200_003
    t = rng.normal(0, 1, (n, 10)).astype(np.float32)
    raw = rng.normal(-3, 2, n).astype(np.float32)
    gate = (rng.uniform(0, 1, n) < 0.6).astype(np.float32) * rng.choice([1.0, 2.0, 3.0], n).astype(np.float32)
    ctx = context(0)
    d_raw, d_gate = torch.from_numpy(raw).cuda(), torch.from_numpy(gate).cuda()  # alive until the kernel has run
    for scale, limit, step in [(0.05, 0.02, 1), (1e-3, 10.0, 2), (2.0, 0.5, 77)]:
        want = orc.mean_noise_step(t, raw, gate, scale, limit, 42, step)
        dt = torch.from_numpy(t.copy()).cuda()
        ctx.check(_lib.lib().bsx_mean_noise_step(ctx.handle, ptr(dt), ptr(d_raw), ptr(d_gate), n,
                                                 float(np.float32(scale)), float(np.float32(limit)), 42, step))
        got = dt.cpu().numpy()
        np.testing.assert_array_equal(got, want)
        assert (got[:, :3] != t[:, :3]).any()


@pytest.mark.parametrize("accumulated_gate", [True, False])
def test_train_step_noise_matches_composed_step(cuda, orc, accumulated_gate):
    import brush_b200 as bsx
    from brush_b200.adam import AdamGroup, AdamScaled
    from brush_b200.splats import clustered_scene, orbit_camera, random_gt

    splats = clustered_scene(20000, 3, "cpu", seed=12).to("cuda")
    w, h = 192, 128
    cams = [orbit_camera(i, 3, 8.0, w, h) for i in range(3)]
    gts = [random_gt(h, w, 60 + i, "cpu").cuda() for i in range(3)]
    cfg = bsx.TrainConfig(mrnf_noise_injection=accumulated_gate, noise_seed=5)
    comp = splats.clone()
    tr = bsx.SplatTrainer(cfg, splats, keep_gradients=True)
    n, c = comp.num_splats, comp.sh_coeffs_per_splat
    opt = AdamScaled(epsilon=1e-15)
    groups = None
    prev_vis = np.zeros(n, np.float32)
    moved = 0
    for k in range(1, 4):
        st = tr.step(cams[k - 1], (w, h), gts[k - 1], splats)
        grads = [tr.grads.v_transforms.clone(), tr.grads.v_coeffs.reshape(n, 3 * c).clone(),
                 tr.grads.v_raw_opac.reshape(n, 1).clone()]
        lr_mean = float(st.lr_mean)
        tscale = [lr_mean] * 3 + [cfg.lr_rotation] * 4 + [_lr_scale(cfg, k)] * 3
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
        vis = tr.record.vis_weight.cpu().numpy().copy()
        gate = vis if accumulated_gate else vis - prev_vis  # this step's visible[]: 0 or 1
        prev_vis = vis
        scale = np.float32(np.float32(lr_mean) * np.float32(cfg.mean_noise_weight))
        noised = orc.mean_noise_step(comp.transforms.cpu().numpy(), comp.raw_opacities.cpu().numpy(), gate, scale,
                                     np.float32(tr.median_scale), 5, k)
        moved += int((noised[:, :3] != comp.transforms.cpu().numpy()[:, :3]).any(axis=1).sum())
        comp.transforms.copy_(torch.from_numpy(noised).cuda())
        for a, b in ((splats.transforms, comp.transforms), (splats.sh_coeffs, comp.sh_coeffs),
                     (splats.raw_opacities, comp.raw_opacities)):
            np.testing.assert_array_equal(a.cpu().numpy(), b.cpu().numpy())
    assert moved > 0
    tr.close()


def _lr_scale(cfg, k):
    """The scale-column rate of optimizer step k (burn ExponentialLrScheduler, first step = initial)."""
    g = (cfg.lr_scale_end / cfg.lr_scale) ** (1.0 / cfg.total_train_iters)
    p = cfg.lr_scale / g
    for _ in range(k):
        p *= g
    return p

"""Densification on the GPU (bsx_trainer_refine_plan / _apply) against the
oracle restatement of refine_for_phase (crates/brush-train/src/train.rs:1191-1860):
same prune decisions, same draws, same split arithmetic, same optimizer-state
remap, bit for bit; then training continues at the new count."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _snapshot(tr, splats):
    n = splats.num_splats
    rec = tr.record
    state = tr.native.optimizer_state()
    (m_t, m_s, m_o), (v_t, v_s, v_o) = state
    c = splats.sh_coeffs_per_splat
    return dict(
        t=splats.transforms.cpu().numpy().copy(), sh=splats.sh_coeffs.cpu().numpy().copy(),
        op=splats.raw_opacities.cpu().numpy().copy(),
        record=tuple(x.cpu().numpy().copy() for x in (rec.refine_weight_norm, rec.vis_weight, rec.max_screen_size)),
        moments=((m_t.cpu().numpy().copy(), m_s.reshape(n, 3 * c).cpu().numpy().copy(), m_o.cpu().numpy().copy()),
                 (v_t.cpu().numpy().copy(), v_s.cpu().numpy().copy(), v_o.cpu().numpy().copy())),
        bounds=(tr.bounds[0].copy(), tr.bounds[1].copy()))


def _check(tr, splats, snap, ref, st):
    for f in ("num_added", "num_split_oversized", "num_split_high_grad", "num_pruned", "num_pruned_non_finite",
              "total_splats"):
        assert getattr(st, f) == getattr(ref["stats"], f), f
    np.testing.assert_array_equal(splats.transforms.cpu().numpy(), ref["transforms"])
    np.testing.assert_array_equal(splats.sh_coeffs.cpu().numpy(), ref["sh"])
    np.testing.assert_array_equal(splats.raw_opacities.cpu().numpy(), ref["opac"])
    n2 = st.total_splats
    (m_t, m_s, m_o), (v_t, v_s, v_o) = tr.native.optimizer_state()
    got_m = (m_t.cpu().numpy(), m_s.reshape(n2, -1).cpu().numpy(), m_o.cpu().numpy())
    got_v = (v_t.cpu().numpy(), v_s.cpu().numpy(), v_o.cpu().numpy())
    for a, b in zip(got_m + got_v, ref["m"] + ref["v"]):
        np.testing.assert_array_equal(a, b)
    rec = tr.record
    assert rec.vis_weight.shape[0] == n2 and not rec.vis_weight.any() and not rec.refine_weight_norm.any()
    assert rec.grad2d_accum.shape[0] == n2
    assert tr.n == n2 and splats.num_splats == n2


def test_refine_matches_oracle_and_training_continues(cuda, orc):
    import brush_b200 as bsx
    from brush_b200.splats import clustered_scene, orbit_camera, random_gt

    splats = clustered_scene(30000, 1, "cpu", seed=21, log_scale_mean=-2.5).to("cuda")
    w, h = 256, 192
    cams = [orbit_camera(i, 4, 8.0, w, h) for i in range(4)]
    gts = [random_gt(h, w, 70 + i, "cpu").cuda() for i in range(4)]
    tr = bsx.SplatTrainer(bsx.TrainConfig(), splats)
    for k in range(6):
        tr.step(cams[k % 4], (w, h), gts[k % 4], splats)
    # prune cases the training alone would not produce
    with torch.no_grad():
        splats.raw_opacities[:50] = -12.0
        splats.transforms[50:55, 0] = 1e4
        splats.transforms[55, 8] = float("nan")
        splats.transforms[56, 3:7] = 1e-6
        splats.transforms[57, 7] = -40.0
    cfg = bsx.RefineConfig(growth_grad_threshold=2e-5, growth_select_fraction=0.3, split_at_screen_size=0.05,
                           seed=1234)
    for r in range(2):
        torch.cuda.synchronize()
        snap = _snapshot(tr, splats)
        n = snap["t"].shape[0]
        st = tr.refine(splats, global_iter=200 * (r + 1), phase_iter=200 * (r + 1), phase_total=3000,
                       refine_config=cfg)
        ref = orc.refine(snap["t"], snap["sh"], snap["op"], snap["record"], snap["moments"],
                         orc.refine_cfg(growth_grad_threshold=2e-5, growth_select_fraction=0.3,
                                        split_at_screen_size=0.05, seed=1234),
                         snap["bounds"][0], snap["bounds"][1], 200 * (r + 1), r, 200 * (r + 1), 3000)
        torch.cuda.synchronize()
        _check(tr, splats, snap, ref, st)
        if r == 0:
            assert st.num_pruned >= 58 and st.num_pruned_non_finite >= 1
            assert st.num_added > 0 and st.num_split_high_grad > 0
        for k in range(4):
            s2 = tr.step(cams[k], (w, h), gts[k], splats)
            assert np.isfinite(float(s2.loss.item()))
    tr.close()


def test_refine_refuses_without_statistics(cuda):
    import brush_b200 as bsx
    from brush_b200.splats import config1_scene

    splats, cam, size, gt = config1_scene("cuda", seed=3)
    tr = bsx.SplatTrainer(bsx.TrainConfig(uniform_lr=1e-3), splats, gather_stats=False)
    tr.step(cam, size, gt.cuda(), splats)
    with pytest.raises(bsx.BsxError):
        tr.refine(splats, 100)
    tr.close()


def test_gradient_threshold_rule_matches_oracle(cuda, orc):
    """The original 3DGS densification: the view-space gradient-norm
    statistic the trainer accumulates, then clone / split / prune, bit-equal to the oracle."""
    import brush_b200 as bsx
    from brush_b200.splats import clustered_scene, orbit_camera, random_gt

    splats = clustered_scene(30000, 1, "cpu", seed=24, log_scale_mean=-3.0, log_scale_std=1.0).to("cuda")
    w, h = 256, 192
    cams = [orbit_camera(i, 4, 8.0, w, h) for i in range(4)]
    gts = [random_gt(h, w, 80 + i, "cpu").cuda() for i in range(4)]
    tr = bsx.SplatTrainer(bsx.TrainConfig(accumulate_grad2d=True), splats)
    # the statistic after one step: |d loss / d xy * (W/2, H/2)| where visible
    tr.step(cams[0], (w, h), gts[0], splats)
    torch.cuda.synchronize()
    vg = tr.native.raster_grads().cpu().numpy()
    vis = tr.record.vis_weight.cpu().numpy()
    gx, gy = vg[:, 0] * np.float32(w / 2), vg[:, 1] * np.float32(h / 2)
    want = np.where(vis > 0, np.sqrt(gx * gx + gy * gy), np.float32(0)).astype(np.float32)
    np.testing.assert_array_equal(tr.record.grad2d_accum.cpu().numpy(), want)
    for k in range(1, 5):
        tr.step(cams[k % 4], (w, h), gts[k % 4], splats)
    torch.cuda.synchronize()
    with torch.no_grad():
        splats.raw_opacities[:40] = -9.0  # below the 0.005 opacity floor
    snap = _snapshot(tr, splats)
    g2 = tr.record.grad2d_accum.cpu().numpy().copy()
    vis = snap["record"][1]
    avg = np.where(vis > 0, g2 / np.maximum(vis, 1), 0)
    thr = float(np.quantile(avg[avg > 0], 0.8))
    t = snap["t"]
    smax = np.exp(t[:, 7:10].astype(np.float64)).max(axis=1)
    ext = float(max(snap["bounds"][1]))
    dense = float(np.median(smax[avg >= thr])) / ext
    kw = dict(growth_grad_threshold=thr, min_opacity=0.005, percent_dense=dense, seed=77)
    cfg = bsx.RefineConfig(rule=bsx.REFINE_GRAD_THRESHOLD, **kw)
    st = tr.refine(splats, 100, 100, 3000, cfg)
    ref = orc.refine(t, snap["sh"], snap["op"], snap["record"] + (g2,), snap["moments"],
                     orc.refine_cfg(rule=1, **kw), snap["bounds"][0], snap["bounds"][1], 100, 0, 100, 3000)
    torch.cuda.synchronize()
    _check(tr, splats, snap, ref, st)
    clones = st.num_added - st.num_split_high_grad
    assert st.num_pruned >= 40 and clones > 0 and st.num_split_high_grad > 0
    assert not tr.record.grad2d_accum.any()
    # split children: scales / 1.6 of their parent, means within a few parent scales
    n2 = st.total_splats
    kids = splats.transforms.cpu().numpy()[n2 - 2 * st.num_split_high_grad:]
    assert np.isfinite(kids).all()
    for k in range(4):
        s2 = tr.step(cams[k], (w, h), gts[k], splats)
        assert np.isfinite(float(s2.loss.item()))
    tr.close()


def _bounds_from_pos(means, percentile):
    """numpy restatement of bounds_from_pos (splat_init.rs:130-158) with total_cmp order."""
    lo_v, hi_v = [], []
    p = np.float32(percentile)
    for k in range(3):
        v = means[:, k][np.isfinite(means[:, k])]
        if v.size == 0:
            return np.zeros(3, np.float32), np.ones(3, np.float32)
        b = v.view(np.uint32)
        key = np.where(b & 0x80000000, ~b, b | 0x80000000)  # total_cmp as an unsigned order
        vs = v[np.argsort(key, kind="stable")]
        n = v.size
        lo = int(np.float32(np.float32(np.float32(1) - p) / np.float32(2)) * np.float32(n))
        hi = min(n - 1, int(np.float32(np.float32(np.float32(1) + p) / np.float32(2)) * np.float32(n)))
        lo_v.append(vs[lo])
        hi_v.append(vs[hi])
    mn, mx = np.array(lo_v, np.float32), np.array(hi_v, np.float32)
    return (mx + mn) / np.float32(2), (mx - mn) / np.float32(2)


@pytest.mark.parametrize("n", [1, 7, 100_003])
def test_device_bounds_match_restatement(cuda, n):
    """bsx_splat_bounds (the library's radix sort, no PyTorch kernels) against bounds_from_pos,
    with non-finite coordinates, signed zeros and the all-non-finite fallback."""
    from brush_b200.splats import splat_bounds

    rng = np.random.default_rng(n)
    t = rng.normal(0, 2, (n, 10)).astype(np.float32)
    if n > 10:
        t[:5, 0] = np.nan
        t[5:9, 1] = np.inf
        t[9:20, 2] = -0.0
        t[20:30, 2] = 0.0
    for p in (0.8, 0.0, 1.0):
        c, e = splat_bounds(torch.from_numpy(t).cuda()[:, 0:3], p)
        wc, we = _bounds_from_pos(t[:, :3].copy(), p)
        np.testing.assert_array_equal(c, wc)
        np.testing.assert_array_equal(e, we)
    t[:, 1] = np.nan
    c, e = splat_bounds(torch.from_numpy(t).cuda()[:, 0:3], 0.8)
    assert c.tolist() == [0, 0, 0] and e.tolist() == [1, 1, 1]

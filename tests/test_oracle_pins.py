"""Pin the CPU oracle to the reference's own known answers before trusting it.

- gsplat golden forward renders committed by the reference
  (crates/brush-bench-test/src/reference.rs:28-151; tolerance 1e-5 + 1 %);
- the raster-oracle KATs (crates/brush-render/src/tests/raster_oracle.rs:111-159);
- sort / prefix-sum / tile-offset KATs (brush-sort/src/lib.rs:170-429,
  brush-prefix-sum/src/lib.rs:109-191, get_tile_offset.rs:88-129);
- the loss KATs: the L1 formula on the reference's 2x2 vectors, SSIM(x, x) = 1 and the
  SSIM clamp range on its byte patterns (crates/brush-loss/tests/reference.rs:133-256, 363-412);
- the render invariance tests: culled splats appended or prepended change nothing, and a
  repeated render is bit-identical (crates/brush-render/src/tests/mod.rs:302-410);
- the shared elementary functions against the C library.
"""
import math

import numpy as np
import pytest

from conftest import golden_case


@pytest.mark.parametrize("name", ["tiny_case", "basic_case"])
def test_golden_gsplat_render(orc, name):
    cam, size, t, sh, op, ref = golden_case(name)
    r = orc.RenderResult(cam, size, t, sh, op)
    err = np.abs(r.image - ref)
    tol = 1e-5 + 1e-2 * np.abs(ref)
    assert not np.isnan(r.image).any()
    assert (err <= tol).all(), f"max err {err.max()}"


def test_raster_kat_one_splat_clamps_negative_color(orc):
    img = orc.rasterize_rows([0.5, 0.5, 1.0, 0.0, 1.0, 0.5, 1.0, 0.5, -1.0, 0.0], 1, 1, (0.2, 0.4, 0.6))
    np.testing.assert_allclose(img.ravel(), [0.6, 0.45, 0.3, 0.5], atol=1e-6)


def test_raster_kat_early_out_splat_not_accumulated(orc):
    rows = [0.5, 0.5, 1.0, 0.0, 1.0, 0.999, 1.0, 0.0, 0.0, 0.0, 0.5, 0.5, 1.0, 0.0, 1.0, 0.999, 0.0, 1.0, 0.0, 0.0]
    np.testing.assert_allclose(orc.rasterize_rows(rows, 1, 1).ravel(), [0.999, 0, 0, 0.999], atol=1e-6)


def test_raster_kat_hard_and_smooth_cutoff(orc):
    mid = float(np.float32(1.0 / 255.0))
    rows = [0.5, 0.5, 1.0, 0.0, 1.0, mid, 1.0, 0.0, 0.0, 0.0]
    np.testing.assert_allclose(orc.rasterize_rows(rows, 1, 1).ravel(), [mid, 0, 0, mid], atol=1e-7)
    np.testing.assert_allclose(orc.rasterize_rows(rows, 1, 1, smooth=True).ravel(), [mid / 2, 0, 0, mid / 2],
                               atol=1e-7)


def test_tile_raster_matches_global_order_raster(orc):
    """Binned tile rasterization equals compositing all depth-sorted splats (raster_oracle.rs:306-329, 2e-5)."""
    from brush_b200.splats import config1_scene

    splats, cam, size, _ = config1_scene("cpu", seed=7, n=2048)
    r = orc.RenderResult(cam, size, splats.transforms.numpy(), splats.sh_coeffs.numpy(),
                         splats.raw_opacities.numpy())
    rows = r.projected[r.depth_order][:, :10]
    glob = orc.rasterize_rows(rows, size[0], size[1])
    assert np.abs(glob - r.image).max() <= 2e-5


def test_sort_kat_stable_for_every_pass_count(orc):
    n = 4099
    i = np.arange(n, dtype=np.uint64)
    group = ((i * 73) % 1021).astype(np.uint64)
    prod = (group * 0x9E3779B9) & 0xFFFFFFFF
    keys = ((((prod << 7) | (prod >> 25)) & 0xFFFFFFFF) ^ 0xA5A55A5A).astype(np.uint32)
    vals = np.arange(n, dtype=np.uint32)
    for bits in [0, 4, 8, 12, 13, 14, 15, 16, 20, 28, 32]:
        eff = (bits + 3) // 4 * 4
        mask = 0xFFFFFFFF if eff == 32 else (1 << eff) - 1
        order = np.argsort(keys & np.uint32(mask), kind="stable")
        ko, vo = orc.radix_argsort(keys, vals, bits)
        assert (ko == keys[order]).all() and (vo == vals[order]).all(), bits


def test_prefix_sum_kats(orc):
    assert list(orc.prefix_sum([1, 1, 1, 1])) == [1, 2, 3, 4]
    for n in [255, 256, 257]:
        d = (np.arange(n) % 7).astype(np.uint32)
        assert (orc.prefix_sum(d) == np.cumsum(d).astype(np.uint32)).all()
    d = np.array([2, 0, 32, 512, 30965] * 100, dtype=np.uint32)
    assert (orc.prefix_sum(d) == np.cumsum(d).astype(np.uint32)).all()


def test_tile_offset_kat_runs_and_sentinel(orc):
    runs = [31, 1, 223, 1, 1791, 1, 17, 0]
    ids, exp = [], np.zeros((8, 2), np.uint32)
    for tid, rl in enumerate(runs):
        if rl == 0:
            continue
        s = len(ids)
        ids += [tid] * rl
        exp[tid] = (s, len(ids))
    ids += [8] * 13
    assert (orc.tile_offsets(np.array(ids, np.uint32), 8) == exp).all()


def test_shared_exp_log_accuracy(orc):
    rng = np.random.default_rng(0)
    xs = np.concatenate([rng.uniform(-103, 88, 20000), rng.uniform(-2, 2, 20000)]).astype(np.float32)
    for x in xs[::7]:
        e = orc.expf(x)
        ref = np.float32(math.exp(float(x)))
        assert abs(np.int64(np.float32(e).view(np.int32)) - np.int64(ref.view(np.int32))) <= 1
    for x in np.abs(xs[::7]) + np.float32(1e-3):
        lg = orc.logf(x)
        ref = np.float32(math.log(float(x)))
        assert abs(np.int64(np.float32(lg).view(np.int32)) - np.int64(ref.view(np.int32))) <= 2


def test_raster_exp_accuracy_on_its_domain(orc):
    """bsx_expf_raster (the rasterizers' exp): within 1.4 ulp of the exact exponential on
    [-16, 0] (every float there measures 1.37 at most), within 4.5 ulp down to -87."""
    assert 0.0 <= orc.expf_raster_max_ulp(-16.0, 7) <= 1.4
    assert 0.0 <= orc.expf_raster_max_ulp(-87.0, 101) <= 4.5


def test_raster_sigma_symmetric_and_close_to_reference_expression(orc):
    """bsx_raster_sigma gives the same bits for (dx, dy) and (-dx, -dy) (the forward takes
    pixel - splat, the backward's restatement splat - pixel), and stays within a few ulp of
    the reference's unfused 0.5 (c00 dx^2 + c11 dy^2) + c01 dx dy."""
    rng = np.random.default_rng(5)
    for _ in range(3000):
        c00, c11 = (float(v) for v in np.float32(rng.uniform(1e-3, 2.0, 2)))
        c01 = float(np.float32(rng.uniform(-0.9, 0.9) * math.sqrt(c00 * c11)))
        dx, dy = (float(v) for v in np.float32(rng.uniform(-20.0, 20.0, 2)))
        a = orc.raster_sigma(c00, c01, c11, dx, dy)
        b = orc.raster_sigma(c00, c01, c11, -dx, -dy)
        assert np.float32(a).view(np.uint32) == np.float32(b).view(np.uint32)
        exact = 0.5 * (c00 * dx * dx + c11 * dy * dy) + c01 * dx * dy
        scale = 0.5 * (c00 * dx * dx + c11 * dy * dy) + abs(c01 * dx * dy)
        assert abs(a - exact) <= 4e-7 * scale + 1e-30


def test_shared_atan2_accuracy_and_special_values(orc):
    """bsx_atan2f (the camera models' angle) within 2 ulp of the C library, with its
    quadrant and signed-zero conventions."""
    rng = np.random.default_rng(1)
    pts = np.concatenate([rng.normal(size=(20000, 2)), rng.uniform(-1e-4, 1e-4, (2000, 2)),
                          rng.uniform(-1e4, 1e4, (2000, 2))]).astype(np.float32)
    for y, x in pts[::3]:
        a = np.float32(orc.atan2f(y, x))
        ref = np.float32(math.atan2(float(y), float(x)))
        assert abs(np.int64(a.view(np.int32)) - np.int64(ref.view(np.int32))) <= 2, (y, x)
    inf = float("inf")
    for y, x in [(0.0, 1.0), (0.0, -1.0), (-0.0, -1.0), (1.0, 0.0), (-1.0, -0.0), (0.0, -0.0), (inf, 1.0),
                 (1.0, -inf), (-inf, -inf), (inf, inf)]:
        assert np.float32(orc.atan2f(y, x)) == np.float32(math.atan2(y, x)), (y, x)


def test_gauss_taps_normalised(orc):
    w = orc.gauss_taps()
    assert abs(float(w.sum()) - 1.0) < 1e-6 and np.allclose(w, w[::-1])


def _pattern(h, w, scale, offset):
    """The reference loss tests' deterministic RGBA byte pattern (brush-loss/tests/reference.rs:27-31)."""
    i = np.arange(h * w * 4, dtype=np.uint64)
    return ((i * scale + offset) % 251).astype(np.uint8).reshape(h, w, 4)


def _packed(b):
    b = b.astype(np.uint32)
    return b[..., 0] | (b[..., 1] << 8) | (b[..., 2] << 16) | (b[..., 3] << 24)


@pytest.mark.parametrize("channels,l1,bg,mask", [(3, 0.73, None, False), (3, 0.41, (0.1, 0.25, 0.8), True),
                                                 (4, 0.19, None, False)])
def test_loss_l1_kat(orc, channels, l1, bg, mask):
    """L1-only loss map against the reference's CPU formula and its own 2x2 vectors
    (brush-loss/tests/reference.rs:133-175, 363-412): weight * |pred - gt| * (mask ? alpha : 1),
    gt = byte / 255 (+ (1 - alpha) * bg when compositing), the alpha channel weighted 1."""
    gt = np.array([10, 100, 200, 0, 250, 50, 25, 64, 30, 90, 150, 192, 240, 180, 60, 255], np.uint8).reshape(2, 2, 4)
    if channels == 3:
        pred = np.array([0.9, 0.1, 0.4, 0.2, 0.8, 0.5, 0.7, 0.3, 0.05, 0.4, 0.6, 0.95], np.float32).reshape(2, 2, 3)
    else:
        pred = np.array([0.9, 0.1, 0.4, 0.8, 0.2, 0.8, 0.5, 0.1, 0.7, 0.3, 0.05, 0.9, 0.4, 0.6, 0.95, 0.2],
                        np.float32).reshape(2, 2, 4)
    cfg = orc.loss_cfg(l1_weight=l1, ssim_weight=0.0, composite_bg=bg, mask=mask)
    got = orc.loss_fwd(np.ascontiguousarray(pred.transpose(2, 0, 1)), _packed(gt), cfg).transpose(1, 2, 0)
    alpha = gt[..., 3].astype(np.float32) / 255.0
    for c in range(channels):
        if c == 3:
            ref, wgt = alpha, 1.0
        else:
            ref = gt[..., c].astype(np.float32) / 255.0
            if bg is not None:
                ref = ref + (1.0 - alpha) * np.float32(bg[c])
            wgt = l1
        exp = wgt * np.abs(pred[..., c] - ref) * (alpha if mask else 1.0)
        assert np.abs(got[..., c] - exp).max() < 2e-6, (c, got[..., c], exp)


def test_loss_ssim_of_identical_pattern_is_one(orc):
    """SSIM(x, x) = 1 on the reference's 40x56 pattern (reference.rs:210-232, |mean - 1| < 1e-4)."""
    b = _pattern(40, 56, 11, 13)
    pred = np.ascontiguousarray((b[..., :3].astype(np.float32) / 255.0).transpose(2, 0, 1))
    m = orc.loss_fwd(pred, _packed(b), orc.loss_cfg(l1_weight=0.0, ssim_weight=1.0))
    assert abs(float(m.astype(np.float64).mean()) - 1.0) < 1e-4
    assert np.abs(m - 1.0).max() <= 1e-5


def test_loss_ssim_stays_in_clamp_range(orc):
    """SSIM of two different patterns stays inside [-1, 1] (reference.rs:234-256)."""
    a, b = _pattern(40, 56, 7, 19), _pattern(40, 56, 13, 7)
    pred = np.ascontiguousarray((a[..., :3].astype(np.float32) / 255.0).transpose(2, 0, 1))
    m = orc.loss_fwd(pred, _packed(b), orc.loss_cfg(l1_weight=0.0, ssim_weight=1.0))
    assert m.min() >= -1.0 and m.max() <= 1.0 and m.min() < 0.9


def _rng_scene(n, spread, log_scale, opac, seed):
    """Random splats: means in [-spread, spread]^3, log-scales and opacity logits uniform in the
    given ranges, random rotations, DC colours in [0, 1] (the shape of the reference's
    invariance scenes, crates/brush-render/src/tests/mod.rs:250-290)."""
    rng = np.random.default_rng(seed)
    means = rng.uniform(-spread, spread, (n, 3))
    q = rng.normal(size=(n, 4))
    ls = rng.uniform(*log_scale, (n, 3))
    t = np.concatenate([means, q, ls], 1).astype(np.float32)
    sh = rng.uniform(0.0, 1.0, (n, 1, 3)).astype(np.float32)
    op = rng.uniform(*opac, n).astype(np.float32)
    return t, sh, op


def _invariance_render(orc, t, sh, op):
    from brush_b200.camera import Camera

    cam = Camera(fov_x=0.5, fov_y=0.5, position=(0.0, 0.0, -5.0), rotation=(0.0, 0.0, 0.0, 1.0))
    return orc.RenderResult(cam, (256, 256), t, sh, op).image


def test_invariance_hidden_splats_do_not_perturb_render(orc):
    """Appending culled splats (opacity far below 1/255, behind the camera, far off-screen)
    leaves the render unchanged (crates/brush-render/src/tests/mod.rs:333-378, < 1e-5)."""
    t, sh, op = _rng_scene(5000, 1.5, (-3.0, -0.5), (0.0, 3.0), 0xBEEF)
    ht, hsh, hop = _rng_scene(20000, 1.0, (-1.0, 1.0), (-20.0, -20.0), 0xDEAD)
    ht[1::3, 0:3] = [0.0, 0.0, -1000.0]  # behind the camera (it looks along +z from z = -5)
    ht[2::3, 0:3] = [1e6, 1e6, 10.0]     # far off-screen
    hop[1::3] = 2.0
    hop[2::3] = 2.0
    a = _invariance_render(orc, t, sh, op)
    b = _invariance_render(orc, np.concatenate([t, ht]), np.concatenate([sh, hsh]), np.concatenate([op, hop]))
    assert a[..., 3].max() > 0.5
    assert np.abs(a - b).max() < 1e-5


def test_invariance_culled_prefix_and_determinism(orc):
    """A culled prefix shifts every splat's id without changing the render (mod.rs:380-410),
    and rendering twice is bit-identical (mod.rs:302-330)."""
    t, sh, op = _rng_scene(4000, 1.5, (-3.0, -0.5), (0.0, 3.0), 0xC0FFEE)
    pt, psh, pop = _rng_scene(50000, 1.0, (-1.0, 1.0), (-20.0, -20.0), 0xF00D)
    a = _invariance_render(orc, t, sh, op)
    b = _invariance_render(orc, np.concatenate([pt, t]), np.concatenate([psh, sh]), np.concatenate([pop, op]))
    assert np.abs(a - b).max() < 1e-5
    np.testing.assert_array_equal(a, _invariance_render(orc, t, sh, op))

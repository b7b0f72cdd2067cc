"""Pin the CPU oracle's backward to the mathematics, independently of the GPU.

The oracle's forward is pinned by the reference's golden renders and KATs; its
backward restates the reference's hand-written VJPs
(crates/brush-render/src/kernels/rasterize_backwards.rs:166-443,
project_backwards.rs:19-263, camera_model/pinhole.rs:58-123, sh.rs:253-466,
crates/brush-loss/src/lib.rs:553-890), which no reference fixture pins. These
tests check it against central differences of the oracle's own forward, the way
the reference checks its GPU backward (crates/brush-bench-test/tests/finite_diff.rs:
531-600: central differences, 5e-5 + 1 % of the larger magnitude, rendered with the
C^1 smooth alpha cutoff, finite_diff.rs:29-31; camera models :1082-1154), plus the
loss VJP (crates/brush-loss/tests/reference.rs) and the AdamScaled update
(crates/brush-train/src/adam_scaled.rs:216-383) against a numpy restatement.
CPU only: the GPU is compared with this oracle elsewhere.
"""
import numpy as np
import pytest

STEPS = (1e-4, 2e-4, 5e-4, 1e-3)
REL_TOL = 0.01
ABS_TOL = 5e-5
SIZE = (32, 32)
SMOOTH = 2  # raster pass with the smooth alpha cutoff (PASS_BACKWARD_SMOOTH_CUTOFF)


def _camera(model=0, params=(0.0,) * 8):
    from brush_b200.camera import Camera

    return Camera(fov_x=0.6, fov_y=0.6, position=(0.0, 0.0, -3.0), rotation=(0.0, 0.0, 0.0, 1.0),
                  camera_model=model, model_params=params)


def _scene(sh_degree=0):
    """Four splats well inside a 32x32 view with unnormalised, non-axis-aligned rotations."""
    means = [[0.15, -0.12, 0.05], [-0.25, 0.35, 0.15], [0.05, 0.28, -0.25], [-0.18, -0.22, 0.12]]
    rots = [[0.85, 0.15, 0.07, 0.02], [0.72, 0.18, 0.27, 0.12], [0.55, 0.37, 0.33, 0.18],
            [0.78, 0.12, 0.08, 0.23]]
    log_scales = [[-1.45, -1.55, -1.62], [-1.52, -1.38, -1.33], [-1.68, -1.52, -1.41],
                  [-1.33, -1.58, -1.49]]
    dc = [[0.42, 0.58, 0.47], [0.62, 0.38, 0.33], [0.37, 0.52, 0.63], [0.48, 0.47, 0.52]]
    op = [2.4, 2.1, 2.3, 2.5]
    t = np.concatenate([np.array(means), np.array(rots), np.array(log_scales)], 1).astype(np.float32)
    coeffs = (sh_degree + 1) ** 2
    sh = np.zeros((4, coeffs, 3), np.float32)
    sh[:, 0, :] = dc
    if coeffs > 1:
        sh[:, 1:, :] = np.random.default_rng(17).normal(0.0, 0.3, (4, coeffs - 1, 3))
    return t, sh, np.array(op, np.float32)


def _mean_image(orc, cam, t, sh, op, mip=False):
    r = orc.RenderResult(cam, SIZE, t, sh, op, mip=mip, raster_pass=SMOOTH)
    return float(r.image.astype(np.float64).mean())


def _analytic(orc, cam, t, sh, op, mip=False):
    r = orc.RenderResult(cam, SIZE, t, sh, op, mip=mip, raster_pass=SMOOTH)
    w, h = SIZE
    v_out = np.full((h, w, 4), 1.0 / (h * w * 4), np.float32)
    vt, vs, vo, _ = r.project_bwd(r.rasterize_bwd(v_out, False))
    return vt, vs, vo


def _central(f):
    """Median over STEPS of the central difference (f(+h) - f(-h)) / 2h."""
    return float(np.median([(f(h) - f(-h)) / (2 * h) for h in STEPS]))


def _check(numerical, analytical, label):
    scale = max(abs(numerical), abs(analytical), 1e-8)
    assert abs(numerical - analytical) <= ABS_TOL + REL_TOL * scale, \
        f"{label}: numerical {numerical:.6e} vs analytical {analytical:.6e}"


def _perturbed(t, sh, op, lane, splat, comp, d):
    t2, sh2, op2 = t.copy(), sh.copy(), op.copy()
    if lane == "sh":
        sh2[splat, comp // 3, comp % 3] += d
    elif lane == "opac":
        op2[splat] += d
    else:
        t2[splat, {"mean": 0, "rot": 3, "scale": 7}[lane] + comp] += d
    return t2, sh2, op2


def _pick(vt, vs, vo, lane, splat, comp):
    if lane == "sh":
        return float(vs[splat, comp // 3, comp % 3])
    if lane == "opac":
        return float(vo[splat])
    return float(vt[splat, {"mean": 0, "rot": 3, "scale": 7}[lane] + comp])


LANES = [("mean", 0, 0), ("mean", 0, 2), ("mean", 1, 1), ("mean", 3, 0),
         ("rot", 0, 0), ("rot", 1, 2), ("rot", 2, 3),
         ("scale", 0, 0), ("scale", 1, 1), ("scale", 3, 2),
         ("sh", 0, 0), ("sh", 1, 4), ("sh", 2, 2),
         ("opac", 0, 0), ("opac", 2, 0)]


@pytest.mark.parametrize("lane,splat,comp", LANES)
def test_oracle_render_gradient_matches_central_difference(orc, lane, splat, comp):
    cam = _camera()
    t, sh, op = _scene(0)
    if lane == "sh":
        comp %= 3
    an = _pick(*_analytic(orc, cam, t, sh, op), lane, splat, comp)
    num = _central(lambda h: _mean_image(orc, cam, *_perturbed(t, sh, op, lane, splat, comp, h)))
    _check(num, an, f"{lane}[{splat},{comp}]")


@pytest.mark.parametrize("lane,splat,comp", [("mean", 0, 0), ("mean", 1, 2), ("mean", 2, 1),
                                             ("sh", 0, 3), ("sh", 1, 14), ("sh", 2, 29), ("sh", 3, 47),
                                             ("sh", 0, 1), ("scale", 2, 0), ("rot", 3, 1)])
def test_oracle_sh3_gradient_matches_central_difference(orc, lane, splat, comp):
    """Degree-3 colours: coefficient gradients of every band, and the view-direction term
    of the mean gradient (sh.rs:253-381)."""
    cam = _camera()
    t, sh, op = _scene(3)
    an = _pick(*_analytic(orc, cam, t, sh, op), lane, splat, comp)
    num = _central(lambda h: _mean_image(orc, cam, *_perturbed(t, sh, op, lane, splat, comp, h)))
    _check(num, an, f"sh3 {lane}[{splat},{comp}]")


@pytest.mark.parametrize("lane,splat,comp", [("mean", 0, 0), ("mean", 1, 1), ("scale", 0, 0), ("scale", 1, 1),
                                             ("sh", 0, 0), ("opac", 0, 0), ("opac", 2, 0)])
def test_oracle_mip_gradient_matches_central_difference(orc, lane, splat, comp):
    """Mip mode (helpers.rs:191-206), with the reference's own mip cases and tolerances
    (finite_diff.rs:675-785: 1e-4 + 3 %). The reference's projection VJP scales the opacity
    gradient by the compensation factor sqrt(det / det_blurred) but does not differentiate
    that factor with respect to the covariance (project_backwards.rs:188-190); the oracle
    restates this, so the geometric lanes agree with central differences only within that
    tolerance, and for splats large against the 0.1-pixel blur, as here."""
    cam = _camera()
    t, sh, op = _scene(0)
    an = _pick(*_analytic(orc, cam, t, sh, op, mip=True), lane, splat, comp)
    num = _central(lambda h: _mean_image(orc, cam, *_perturbed(t, sh, op, lane, splat, comp, h), mip=True))
    scale = max(abs(num), abs(an), 1e-8)
    assert abs(num - an) <= 1e-4 + 0.03 * scale, f"mip {lane}[{splat},{comp}]: {num:.6e} vs {an:.6e}"


CAMERA_MODELS = {
    "kb4": (1, (0.05, -0.01, 0.002, -0.0004, 0.0, 0.0, 0.0, 0.0)),
    "rt8": (2, (-0.12, 0.03, -0.002, 0.01, -0.004, 0.0005, 0.001, -0.0015)),
    "tpf": (3, (0.04, -0.008, 0.001, -0.0002, 0.0008, -0.0006, 0.0009, -0.0007)),
}


@pytest.mark.parametrize("model", list(CAMERA_MODELS))
@pytest.mark.parametrize("lane,splat,comp", [("mean", 0, 0), ("mean", 1, 1), ("mean", 3, 2),
                                             ("scale", 2, 1), ("rot", 1, 0)])
def test_oracle_camera_model_gradient_matches_central_difference(orc, model, lane, splat, comp):
    """Projection and Jacobian VJPs of the distorted models (camera_model/*.rs), the mean
    gradient above all, through the whole render."""
    kind, params = CAMERA_MODELS[model]
    cam = _camera(kind, params)
    t, sh, op = _scene(0)
    an = _pick(*_analytic(orc, cam, t, sh, op), lane, splat, comp)
    num = _central(lambda h: _mean_image(orc, cam, *_perturbed(t, sh, op, lane, splat, comp, h)))
    _check(num, an, f"{model} {lane}[{splat},{comp}]")


def test_oracle_quaternion_tangent_directions(orc):
    """Directions tangent to the quaternion (the radial one is normalised away), with
    strongly anisotropic scales so that every rotation axis changes the image."""
    cam = _camera()
    t, sh, op = _scene(0)
    t[:, 7:10] = [[-1.0, -2.2, -1.8]] * 4
    vt, _, _ = _analytic(orc, cam, t, sh, op)
    rng = np.random.default_rng(3)
    for s in range(4):
        q = t[s, 3:7].astype(np.float64)
        for _ in range(3):
            d = rng.normal(size=4)
            d -= q * (d @ q) / (q @ q)
            d /= np.linalg.norm(d)

            def along(h, s=s, d=d):
                tp = t.copy()
                tp[s, 3:7] += (h * d).astype(np.float32)
                return _mean_image(orc, cam, tp, sh, op)

            _check(_central(along), float(vt[s, 3:7] @ d), f"quat tangent splat {s}")


def test_oracle_gradients_vanish_for_culled_splats(orc):
    """A splat behind the camera and one below the opacity threshold get exactly zero
    gradient rows (project_backwards.rs:143-156 exits on an all-zero compact row)."""
    cam = _camera()
    t, sh, op = _scene(0)
    t = np.concatenate([t, t[:2]])
    sh = np.concatenate([sh, sh[:2]])
    op = np.concatenate([op, np.array([2.0, -30.0], np.float32)])
    t[4, 2] = -10.0  # behind the camera at z = -3
    vt, vs, vo = _analytic(orc, cam, t, sh, op)
    assert not vt[4:].any() and not vs[4:].any() and not vo[4:].any()
    assert np.abs(vt[:4]).max() > 0.0


@pytest.mark.parametrize("cfg_kw", [dict(), dict(l1_weight=0.0, ssim_weight=1.0),
                                    dict(composite_bg=(0.2, 0.5, 0.8))])
def test_oracle_loss_vjp_matches_central_difference(orc, cfg_kw):
    """image_loss_backward (brush-loss/src/lib.rs:553-890) against central differences of
    the mean of image_loss_forward; zero padding at the borders is included."""
    rng = np.random.default_rng(6)
    h, w = 16, 16
    pred = rng.uniform(0.2, 0.8, (3, h, w)).astype(np.float32)
    gt = rng.integers(0, 2**32, (h, w), dtype=np.uint64).astype(np.uint32)
    cfg = orc.loss_cfg(**cfg_kw)
    dl = np.full((3, h, w), 1.0 / (3 * h * w), np.float32)
    v = orc.loss_bwd(pred, gt, cfg, dl)

    def loss(x):
        return float(orc.loss_fwd(x, gt, cfg).astype(np.float64).mean())

    eps = 2e-3
    for (c, y, x) in [(0, 0, 0), (1, 5, 7), (2, 12, 12), (0, 15, 10), (2, 9, 3), (1, 0, 15)]:
        p, m = pred.copy(), pred.copy()
        p[c, y, x] += eps
        m[c, y, x] -= eps
        num = (loss(p) - loss(m)) / (2 * eps)
        an = float(v[c, y, x])
        assert abs(num - an) <= 2e-6 + 0.02 * max(abs(num), abs(an)), (cfg_kw, c, y, x, num, an)


def _adam_numpy(param, grad, m, v, lr, col_scale, reduce, step, b1=0.9, b2=0.999, eps=1e-15):
    """AdaptiveMomentum::transform + AdamScaled::step (adam_scaled.rs:216-303,329-383) in f32.
    The reference's betas are f32 fields, so 1 - beta is an f32 subtraction (0.1 becomes
    0.100000024), and beta^t is an f32 power."""
    f = np.float32
    k1, k2 = f(1) - f(b1), f(1) - f(b2)
    g = grad.astype(f)
    gsq = g * g
    if reduce:
        gsq = (gsq.sum(axis=1, dtype=f) / f(g.shape[1]))[:, None]
    if step == 1:
        m1 = g * k1
        m2 = gsq * k2
    else:
        m1 = m * f(b1) + g * k1
        m2 = (v[:, None] if reduce else v) * f(b2) + gsq * k2
    c1 = m1 / (f(1) - f(b1) ** step)
    c2 = m2 / (f(1) - f(b2) ** step)
    upd = c1 / (np.sqrt(c2) + f(eps))
    scale = (col_scale.astype(f) * f(lr)) if col_scale is not None else f(lr)
    return param - upd * scale, m1, (m2[:, 0] if reduce else m2)


@pytest.mark.parametrize("reduce,scaled", [(False, False), (False, True), (True, True)])
def test_oracle_adam_matches_numpy_restatement(orc, reduce, scaled):
    """Three AdamScaled steps: plain, per-column learning-rate scale (transforms), and the
    SH form with one second moment per row (the mean of the row's squared gradients)."""
    rng = np.random.default_rng(9)
    rows, cols = 257, 48 if reduce else 10
    p = rng.normal(size=(rows, cols)).astype(np.float32)
    m = np.zeros_like(p)
    v = np.zeros(rows, np.float32) if reduce else np.zeros_like(p)
    scale = rng.uniform(0.05, 2.0, cols).astype(np.float32) if scaled else None
    p0 = p.copy()
    pn, mn, vn = p.copy(), m.copy(), v.copy()
    for step in (1, 2, 3):
        g = rng.normal(scale=0.1, size=(rows, cols)).astype(np.float32)
        orc.adam(p, g, m, v, 1e-3, col_scale=scale, reduce=reduce, step=step)
        pn, mn, vn = _adam_numpy(pn, g, mn, vn, 1e-3, scale, reduce, step)
    np.testing.assert_allclose(m, mn, rtol=1e-6, atol=1e-9)
    np.testing.assert_allclose(v, vn, rtol=1e-5, atol=1e-12)
    np.testing.assert_allclose(p, pn, rtol=1e-6, atol=1e-7)
    assert np.abs(p - p0).max() > 1e-4  # three steps of about lr each moved the parameters



def _lcg_weights(h, w, c=4, seed=0xCAFEF00D):
    """Deterministic weights in [0, 1) from a 64-bit LCG (the generator of finite_diff.rs:803-812)."""
    out = np.empty(h * w * c, np.float32)
    state = seed
    for i in range(out.size):
        state = (state * 6364136223846793005 + 1442695040888963407) & (2**64 - 1)
        out[i] = np.float32((state >> 33) / 0xFFFFFFFF)
    return out.reshape(h, w, c)


@pytest.mark.parametrize("lane,splat,comp", [("mean", 0, 0), ("mean", 1, 1), ("scale", 0, 0), ("sh", 1, 1),
                                             ("opac", 0, 0), ("opac", 2, 0), ("rot", 2, 1)])
def test_oracle_weighted_loss_gradient_matches_central_difference(orc, lane, splat, comp):
    """sum(image * W) for a fixed random weight map W (finite_diff.rs:794-917): a per-pixel
    asymmetry between forward and backward that a uniform mean would hide shows here.
    Tolerance 0.5 + 2 % as the reference's (sum-loss values are in the hundreds)."""
    cam = _camera()
    t, sh, op = _scene(0)
    wts = _lcg_weights(SIZE[1], SIZE[0])
    r = orc.RenderResult(cam, SIZE, t, sh, op, raster_pass=SMOOTH)
    vt, vs, vo, _ = r.project_bwd(r.rasterize_bwd(wts, False))
    an = _pick(vt, vs, vo, lane, splat, comp)

    def value(h):
        img = orc.RenderResult(cam, SIZE, *_perturbed(t, sh, op, lane, splat, comp, h), raster_pass=SMOOTH).image
        return float((img.astype(np.float64) * wts).sum())

    num = _central(value)
    scale = max(abs(num), abs(an), 1e-8)
    assert abs(num - an) <= 0.5 + 0.02 * scale, f"weighted {lane}[{splat},{comp}]: {num:.6e} vs {an:.6e}"
    assert abs(num - an) <= 0.05 + 0.01 * scale  # the oracle also meets a ten times tighter bound


def test_oracle_early_out_back_splats_gradient(orc):
    """Thirty opaque splats stacked in depth: the front few drive transmittance below 1e-4,
    the rest are skipped where the stack covers a pixel, and their opacity gradient is
    near zero on both sides (finite_diff.rs:1020-1075, |diff| < 5e-4)."""
    cam = _camera()
    n = 30
    t = np.zeros((n, 10), np.float32)
    t[:, 2] = np.arange(n) * 0.3
    t[:, 3] = 1.0
    t[:, 7:10] = -0.3
    c = 0.3 + 0.4 * (np.arange(n) / n)
    sh = np.repeat(c[:, None, None], 3, axis=2).astype(np.float32)
    op = np.full(n, 4.0, np.float32)
    _, _, vo = _analytic(orc, cam, t, sh, op)
    eps = 1e-3
    for s in (1, 5, 10, 15, 20, 25, 29):
        p, m = op.copy(), op.copy()
        p[s] += eps
        m[s] -= eps
        num = (_mean_image(orc, cam, t, sh, p) - _mean_image(orc, cam, t, sh, m)) / (2 * eps)
        assert abs(num - float(vo[s])) < 5e-4, (s, num, float(vo[s]))
    assert abs(float(vo[1])) > 1e-4 and abs(float(vo[25])) < 1e-6 and abs(float(vo[29])) < 1e-6


@pytest.mark.parametrize("comp", [0, 5, 13, 26, 40, 52, 61, 74])
def test_oracle_sh4_coefficient_gradient(orc, comp):
    """Coefficient gradients in every band up to degree 4 (25 coefficients;
    finite_diff.rs:1748-1830 exercises each band)."""
    cam = _camera()
    t, sh, op = _scene(0)
    sh4 = np.zeros((4, 25, 3), np.float32)
    sh4[:, :1] = sh
    sh4[:, 1:] = np.random.default_rng(23).normal(0.0, 0.2, (4, 24, 3))
    for splat in (0, 3):
        an = _pick(*_analytic(orc, cam, t, sh4, op), "sh", splat, comp)
        num = _central(lambda h: _mean_image(orc, cam, *_perturbed(t, sh4, op, "sh", splat, comp, h)))
        _check(num, an, f"sh4[{splat},{comp}]")

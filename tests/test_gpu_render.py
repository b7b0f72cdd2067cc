"""Forward-render parity: the sm_100a pipeline against the CPU oracle.

Bit-exact: per-splat tile counts, visible set and depth order, the inclusive
count scan, sorted (tile, splat) intersection arrays, tile ranges (including
the backward-pass shortening), projected rows. Image: max abs error <= 1e-4
(the pipelines evaluate the same float operations, so the observed error is 0).
"""
import numpy as np
import pytest
import torch

from conftest import golden_case

pytestmark = pytest.mark.gpu


def _u32(t):
    return t.cpu().numpy().view(np.uint32)


def _render_both(orc, splats, cam, size, raster_pass=1, mip=False, bg=(0.0, 0.0, 0.0)):
    import brush_b200 as bsx

    r = orc.RenderResult(cam, size, splats.transforms.cpu().numpy(), splats.sh_coeffs.cpu().numpy(),
                         splats.raw_opacities.cpu().numpy(), mip=mip, raster_pass=raster_pass, bg=bg)
    s = splats.to("cuda")
    out = bsx.render(cam, size, s.transforms, s.sh_coeffs, s.raw_opacities, int(mip), bg, raster_pass)
    torch.cuda.synchronize()
    return r, out


def _assert_pipeline_equal(r, out, bwd=True):
    V, M = r.num_visible, r.num_intersections
    assert out.aux.num_visible == V
    assert out.aux.num_intersections == M
    assert (_u32(out.tile_counts) == r.counts).all()
    assert (_u32(out.depth_order) == r.depth_order).all()
    assert (_u32(out.cum_counts) == r.cum).all()
    assert (_u32(out.isect_tile) == r.isect_tile).all()
    assert (_u32(out.compact_gid_from_isect) == r.isect_gid).all()
    assert (_u32(out.aux.tile_offsets) == r.tile_offsets).all()
    proj = out.projected_splats.cpu().numpy()
    vis = r.depth_order
    assert (proj[vis].view(np.uint32) == r.projected[vis].view(np.uint32)).all()
    assert (out.aux.max_radius.cpu().numpy() == r.max_radius).all()
    if bwd:
        img = out.out_img.cpu().numpy()
        assert np.abs(img - r.image).max() <= 1e-4
        assert (out.aux.visible.cpu().numpy() == r.visible).all()
    else:
        assert (_u32(out.out_img) == r.image_packed).all()


def test_config1_pipeline_bit_exact(cuda, orc):
    from brush_b200.splats import config1_scene

    splats, cam, size, _ = config1_scene("cpu", seed=1)
    r, out = _render_both(orc, splats, cam, size)
    assert r.num_intersections > 0
    _assert_pipeline_equal(r, out)
    assert np.abs(out.out_img.cpu().numpy() - r.image).max() == 0.0


@pytest.mark.parametrize("deg", [1, 2, 3, 4])
def test_sh_degrees_and_clusters_bit_exact(cuda, orc, deg):
    from brush_b200.splats import clustered_scene, orbit_camera

    splats = clustered_scene(20000, deg, "cpu", seed=10 + deg)
    cam = orbit_camera(deg, 7, 8.0, 640, 352)
    r, out = _render_both(orc, splats, cam, (640, 352), bg=(0.1, 0.2, 0.3))
    _assert_pipeline_equal(r, out)


def test_forward_packed_pass(cuda, orc):
    from brush_b200.splats import clustered_scene, orbit_camera

    splats = clustered_scene(8000, 3, "cpu", seed=21)
    cam = orbit_camera(1, 5, 8.0, 300, 200)
    r, out = _render_both(orc, splats, cam, (300, 200), raster_pass=0)
    _assert_pipeline_equal(r, out, bwd=False)


@pytest.mark.parametrize("raster_pass", [0, 1])
def test_many_tiles_bit_exact(cuda, orc, raster_pass):
    """4096x2304 (36 864 tiles): the rasterizers launch tiles in an order computed from
    their intersection counts, beyond the counts that order keeps in shared memory; every
    tile is rendered exactly once (forward bit-exact) and replayed once (backward)."""
    import brush_b200 as bsx
    from brush_b200.splats import clustered_scene, orbit_camera

    from test_gpu_backward import _rel

    splats = clustered_scene(30000, 1, "cpu", seed=23)
    size = (4096, 2304)
    cam = orbit_camera(3, 5, 8.0, *size)
    r, out = _render_both(orc, splats, cam, size, raster_pass=raster_pass)
    assert r.num_intersections > 0
    _assert_pipeline_equal(r, out, bwd=raster_pass != 0)
    if raster_pass:
        rng = np.random.default_rng(4)
        v_output = rng.normal(0, 1e-3, (size[1], size[0], 4)).astype(np.float32)
        vc_gpu = bsx.rasterize_bwd(torch.from_numpy(v_output).cuda(), False).cpu().numpy()[:, :11]
        vc_orc = r.rasterize_bwd(v_output, False)
        for lanes in [(0, 1), (2, 3, 4), (5, 6, 7), (8,)]:
            assert _rel(vc_gpu[:, lanes], vc_orc[:, lanes]) <= 1e-3, lanes


def test_mip_and_smooth_cutoff(cuda, orc):
    from brush_b200.splats import clustered_scene, orbit_camera

    splats = clustered_scene(8000, 1, "cpu", seed=22)
    cam = orbit_camera(2, 5, 8.0, 256, 256)
    r, out = _render_both(orc, splats, cam, (256, 256), raster_pass=2, mip=True)
    _assert_pipeline_equal(r, out)


@pytest.mark.parametrize("name", ["tiny_case", "basic_case"])
def test_golden_gsplat_cases_on_gpu(cuda, orc, name):
    import brush_b200 as bsx

    cam, size, t, sh, op, ref = golden_case(name)
    out = bsx.render(cam, size, torch.from_numpy(t).cuda(), torch.from_numpy(sh).cuda(),
                     torch.from_numpy(op).cuda())
    img = out.out_img.cpu().numpy()
    assert (np.abs(img - ref) <= 1e-5 + 1e-2 * np.abs(ref)).all()
    r = orc.RenderResult(cam, size, t, sh, op)
    assert np.abs(img - r.image).max() <= 1e-4


def test_zero_splats_render_background(cuda):
    import brush_b200 as bsx
    from brush_b200.camera import Camera

    cam = Camera.look_at((0, 0, -3), (0, 0, 0), 1.0, 40, 30)
    z = torch.zeros((0, 10), device="cuda")
    out = bsx.render(cam, (40, 30), z, torch.zeros((0, 1, 3), device="cuda"), torch.zeros(0, device="cuda"),
                     background=(0.25, 0.5, 0.75))
    img = out.out_img.cpu().numpy()
    assert out.aux.num_visible == 0 and out.aux.num_intersections == 0
    np.testing.assert_array_equal(img[..., :3], np.broadcast_to([0.25, 0.5, 0.75], img[..., :3].shape))
    assert (img[..., 3] == 0).all()


def test_culled_and_nonfinite_splats_change_nothing(cuda, orc):
    """Appending splats that every cull test rejects leaves the image unchanged
    (crates/brush-render/src/tests/mod.rs:336-410) and NaN/Inf inputs are culled
    (crates/brush-bench-test/tests/fuzz.rs)."""
    from brush_b200.splats import Splats, config1_scene

    splats, cam, size, _ = config1_scene("cpu", seed=3, n=4000)
    bad = splats.clone()
    k = 64
    bad_t = bad.transforms[:k].clone()
    bad_t[0:16, 0] = float("nan")
    bad_t[16:32, 7] = float("inf")
    bad_t[32:48, 2] = -100.0  # behind the camera
    bad_t[48:64, 3:7] = 0.0   # zero quaternion
    extra = Splats(torch.cat([bad_t, splats.transforms]), torch.cat([bad.sh_coeffs[:k], splats.sh_coeffs]),
                   torch.cat([bad.raw_opacities[:k], splats.raw_opacities]))
    r0, out0 = _render_both(orc, splats, cam, size)
    img0 = out0.out_img.cpu().numpy().copy()
    r1, out1 = _render_both(orc, extra, cam, size)
    _assert_pipeline_equal(r1, out1)
    assert np.abs(out1.out_img.cpu().numpy() - img0).max() <= 1e-5
    assert (out1.tile_counts[:k].cpu().numpy() == 0).all()


def test_repeat_render_is_bit_identical(cuda):
    import brush_b200 as bsx
    from brush_b200.splats import clustered_scene, orbit_camera

    s = clustered_scene(50000, 3, "cuda", seed=30)
    cam = orbit_camera(0, 1, 8.0, 800, 600)
    a = bsx.render(cam, (800, 600), s.transforms, s.sh_coeffs, s.raw_opacities).out_img.clone()
    b = bsx.render(cam, (800, 600), s.transforms, s.sh_coeffs, s.raw_opacities).out_img.clone()
    assert torch.equal(a, b)


def test_config2_scale_properties(cuda):
    """Full-size (1M splats, SH3, 1920x1080) structural invariants."""
    import brush_b200 as bsx
    from brush_b200.splats import config2_scene

    splats, cam, size, _ = config2_scene("cuda")
    out = bsx.render(cam, size, splats.transforms, splats.sh_coeffs, splats.raw_opacities)
    torch.cuda.synchronize()
    V, M = out.aux.num_visible, out.aux.num_intersections
    assert 0 < V <= splats.num_splats and M > 0
    counts = out.tile_counts.to(torch.int64)
    assert int(counts.sum()) == M
    cum = out.cum_counts.to(torch.int64) & 0xFFFFFFFF
    assert int(cum[-1]) == M and bool((cum[1:] >= cum[:-1]).all())
    tiles = out.isect_tile.to(torch.int64)
    assert bool((tiles[1:] >= tiles[:-1]).all())
    T = out.aux.tile_offsets.shape[0] * out.aux.tile_offsets.shape[1]
    off = out.aux.tile_offsets.reshape(-1, 2).to(torch.int64)
    bc = torch.bincount(tiles[tiles < T], minlength=T)
    starts = off[:, 0][bc > 0]
    assert bool((tiles[starts] == torch.nonzero(bc > 0).squeeze(1)).all())
    assert bool((off[:, 1] <= off[:, 0] + bc).all())  # shortened ends stay inside their run
    # depth order really is sorted by depth
    d = out.projected_splats[out.depth_order.to(torch.int64), 9]
    assert bool((d[1:] >= d[:-1]).all())
    img = out.out_img
    assert bool(torch.isfinite(img).all()) and float(img[..., 3].max()) <= 1.0

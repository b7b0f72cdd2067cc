"""The backward operators with the reference's own signatures and compact layouts
(``SplatBwdOps::rasterize_bwd`` / ``project_bwd``, crates/brush-render-bwd/src/burn_glue.rs:84-141),
driven through the C ABI with inputs laid out as the reference's forward leaves them:
projected rows [V,10] and gradient rows [V,11] by compact id (depth rank), the
intersection list in compact ids, ``global_from_compact_gid`` [V].

Checked against the CPU oracle (which indexes by global id) with the tolerances of the
other backward tests: raster gradients per lane group <= 1e-3 relative to the largest
reference value; projection backward on identical inputs <= 1e-5.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


def _reference_layout(r):
    """Compact-indexed tensors of an oracle render (compact id c <-> global id depth_order[c])."""
    order = r.depth_order.astype(np.int64)
    v = order.size
    comp = np.full(r.n, 0xFFFFFFFF, np.uint32)
    comp[order] = np.arange(v, dtype=np.uint32)
    projected10 = np.ascontiguousarray(r.projected[order, :10])
    ids = comp[r.isect_gid.astype(np.int64)]
    assert (ids < v).all()
    return order, projected10, ids


def _uniforms(r):
    from brush_b200 import _lib

    return _lib.ProjectUniforms.from_buffer_copy(bytes(r.uniforms))


@pytest.mark.parametrize("refine,smooth,deg", [(True, False, 3), (False, False, 1), (True, True, 0)])
def test_reference_signature_backward_matches_oracle(cuda, orc, refine, smooth, deg):
    import brush_b200 as bsx
    from brush_b200.splats import clustered_scene, orbit_camera

    s = clustered_scene(15000, deg, "cpu", seed=40 + deg)
    w, h = 320, 200
    cam = orbit_camera(deg, 5, 8.0, w, h)
    bg = (0.2, 0.1, 0.05)
    t, sh, op = s.transforms.numpy(), s.sh_coeffs.numpy(), s.raw_opacities.numpy()
    r = orc.RenderResult(cam, (w, h), t, sh, op, raster_pass=2 if smooth else 1, bg=bg)
    order, proj10, ids = _reference_layout(r)
    v = order.size
    assert v > 0 and r.num_intersections > 0
    rng = np.random.default_rng(deg)
    v_output = rng.normal(0, 1e-3, (h, w, 4)).astype(np.float32)
    dev = "cuda"
    vc = bsx.rasterize_bwd_ref(torch.from_numpy(r.image).to(dev), torch.from_numpy(proj10).to(dev),
                               torch.from_numpy(ids.view(np.int32)).to(dev),
                               torch.from_numpy(r.tile_offsets.view(np.int32)).to(dev), bg, (w, h),
                               torch.from_numpy(v_output).to(dev), smooth_cutoff=smooth,
                               compute_refine_weight=refine)
    torch.cuda.synchronize()
    got = vc.cpu().numpy()
    assert got.shape == (v, 11)
    ref = r.rasterize_bwd(v_output, refine)[order]
    for lanes, name in [((0, 1), "xy"), ((2, 3, 4), "conic"), ((5, 6, 7), "rgb"), ((8,), "alpha"), ((9,), "refine")]:
        if name == "refine" and not refine:
            assert (got[:, 9] == 0).all()
            continue
        assert _rel(got[:, lanes], ref[:, lanes]) <= 1e-3, name
    assert (got[:, 10] == 0).all()  # depth lane: no depth rendering
    # projection backward from the oracle's compact rows
    grads = bsx.project_bwd_ref(torch.from_numpy(t).to(dev), torch.from_numpy(sh).to(dev),
                                torch.from_numpy(op).to(dev), torch.from_numpy(order.astype(np.int32)).to(dev),
                                _uniforms(r), 0, torch.from_numpy(np.ascontiguousarray(ref)).to(dev))
    dense = np.zeros((r.n, 11), np.float32)
    dense[order] = ref
    vt, vs, vo, vr = r.project_bwd(dense)
    for got_t, want, name in [(grads.v_transforms, vt, "transforms"), (grads.v_coeffs, vs, "sh"),
                              (grads.v_raw_opac, vo, "opacity"), (grads.v_refine_weight, vr, "refine")]:
        assert _rel(got_t.cpu().numpy(), want) <= 1e-5, name


def test_reference_signature_skips_out_of_range_inputs(cuda, orc):
    """An intersection id >= V and a tile range beyond M are skipped (the other entries are
    unaffected) and reported as BSX_ERR_INVALID_ARG at the next synchronisation."""
    import brush_b200 as bsx
    from brush_b200._context import context
    from brush_b200._lib import BsxError
    from brush_b200.splats import clustered_scene, orbit_camera

    s = clustered_scene(4000, 0, "cpu", seed=44)
    w, h = 128, 96
    cam = orbit_camera(1, 5, 8.0, w, h)
    r = orc.RenderResult(cam, (w, h), s.transforms.numpy(), s.sh_coeffs.numpy(), s.raw_opacities.numpy())
    order, proj10, ids = _reference_layout(r)
    v = order.size
    v_output = np.random.default_rng(9).normal(0, 1e-3, (h, w, 4)).astype(np.float32)
    args = [torch.from_numpy(r.image).cuda(), torch.from_numpy(proj10).cuda()]
    off = torch.from_numpy(r.tile_offsets.view(np.int32)).cuda()
    good = bsx.rasterize_bwd_ref(*args, torch.from_numpy(ids.view(np.int32)).cuda(), off, (0, 0, 0), (w, h),
                                 torch.from_numpy(v_output).cuda()).cpu().numpy()
    context().sync()
    bad_ids = np.concatenate([ids, np.array([v + 5, 0xFFFFFFF0], np.uint32)])
    bad_off = r.tile_offsets.copy().reshape(-1, 2)
    empty = np.nonzero(bad_off[:, 1] == bad_off[:, 0])[0]
    assert empty.size > 0
    # an empty tile whose range now covers only the two bad ids
    bad_off[empty[0]] = (ids.size, ids.size + 2)
    got = bsx.rasterize_bwd_ref(*args, torch.from_numpy(bad_ids.view(np.int32)).cuda(),
                                torch.from_numpy(bad_off.reshape(r.tile_offsets.shape).view(np.int32)).cuda(),
                                (0, 0, 0), (w, h), torch.from_numpy(v_output).cuda()).cpu().numpy()
    with pytest.raises(BsxError) as e:
        context().sync()
    assert e.value.status == 1
    assert _rel(got, good) <= 1e-6
    # a range past M
    bad_off[empty[0]] = (ids.size, ids.size + 100)
    bsx.rasterize_bwd_ref(*args, torch.from_numpy(ids.view(np.int32)).cuda(),
                          torch.from_numpy(bad_off.reshape(r.tile_offsets.shape).view(np.int32)).cuda(), (0, 0, 0),
                          (w, h), torch.from_numpy(v_output).cuda())
    with pytest.raises(BsxError):
        context().sync()
    context().sync()  # the error word was cleared


def test_failed_render_invalidates_the_backward_state(cuda):
    """A render that fails leaves no state behind: the backward then refuses with
    BSX_ERR_STATE instead of reading the previous render's buffers."""
    import brush_b200 as bsx
    from brush_b200._lib import BsxError
    from brush_b200.splats import clustered_scene, orbit_camera

    s = clustered_scene(2000, 0, "cuda", seed=45)
    cam = orbit_camera(0, 5, 8.0, 64, 48)
    bsx.render(cam, (64, 48), s.transforms, s.sh_coeffs, s.raw_opacities)
    v_output = torch.zeros((48, 64, 4), device="cuda")
    bsx.rasterize_bwd(v_output)  # valid after a good render
    with pytest.raises(BsxError):
        bsx.render(orbit_camera(0, 5, 8.0, 20000, 48), (20000, 48), s.transforms, s.sh_coeffs, s.raw_opacities)
    with pytest.raises(BsxError) as e:
        bsx.rasterize_bwd(v_output)
    assert e.value.status == 6
    vc = torch.zeros((2000, 12), device="cuda")
    with pytest.raises(BsxError) as e:
        bsx.project_bwd(vc, 2000, 1)
    assert e.value.status == 6

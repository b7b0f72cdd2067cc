"""PLY import / export on the GPU (bsx_ply_load, bsx_ply_export) against the CPU oracle
restatement of crates/brush-serde (oracle/ply.cpp), bit for bit; round trips as the
reference's export tests (crates/brush-serde/src/export.rs:193-349)."""
import numpy as np
import pytest
import torch

from plyfiles import compressed_elements, ply_bytes, splat_rows

pytestmark = pytest.mark.gpu


def _gpu(data, subsample=None):
    from brush_b200.ply import load_splat_from_ply

    msg = load_splat_from_ply(data, subsample)
    s = msg.splats
    return msg, s.transforms.cpu().numpy(), s.sh_coeffs.cpu().numpy(), s.raw_opacities.cpu().numpy()


def _same(a, b):
    """Bit-equal, except that every NaN equals every NaN (the payload of sqrt of a
    negative number differs between processors; random packed quaternions hit it)."""
    assert a.shape == b.shape
    nan = np.isnan(a)
    assert np.array_equal(nan, np.isnan(b))
    assert np.array_equal(a[~nan].view(np.uint32), b[~nan].view(np.uint32))


@pytest.mark.parametrize("degree", [0, 1, 2, 3])
@pytest.mark.parametrize("fmt", ["binary_little_endian", "ascii"])
def test_standard_decode_matches_oracle(cuda, orc, degree, fmt):
    n = 1000 if fmt == "ascii" else 20000
    data = ply_bytes([("vertex", splat_rows(n, degree=degree, seed=degree))], fmt=fmt)
    for sub in (None, 3):
        msg, t, sh, op = _gpu(data, sub)
        rt, rsh, rop = orc.ply_decode(data, sub or 1)
        _same(t, rt)
        _same(sh, rsh)
        _same(op, rop)
        assert msg.meta.total_splats == len(rt) and sh.shape[1] == (degree + 1) ** 2


def test_big_endian_equals_little_endian(cuda):
    rows = splat_rows(3000, degree=3, seed=9)
    _, t1, s1, o1 = _gpu(ply_bytes([("vertex", rows)]))
    _, t2, s2, o2 = _gpu(ply_bytes([("vertex", rows)], fmt="binary_big_endian"))
    _same(t1, t2)
    _same(s1, s2)
    _same(o1, o2)


def test_colour_overrides_types_and_defaults(cuda, orc):
    rng = np.random.default_rng(4)
    n = 777
    cases = [
        splat_rows(n, degree=0, extra=[("red", "u1", rng.integers(0, 256, n)), ("green", "u1", rng.integers(0, 256, n)),
                                        ("blue", "u1", rng.integers(0, 256, n))]),
        splat_rows(n, degree=1, drop=("f_dc_0", "f_dc_1", "f_dc_2"),
                   extra=[("r", "u2", rng.integers(0, 65536, n)), ("g", "u2", rng.integers(0, 65536, n)),
                          ("b", "u2", rng.integers(0, 65536, n))]),
        splat_rows(n, degree=0, drop=("rot_0", "rot_1", "rot_2", "rot_3", "scale_0", "scale_1", "scale_2", "opacity",
                                      "f_dc_0", "f_dc_1", "f_dc_2")),
        splat_rows(n, degree=0, drop=("rot_3", "scale_2"), extra=[("nx", "f8", rng.normal(size=n)),
                                                                 ("label", "i2", rng.integers(-5, 5, n))]),
    ]
    for rows in cases:
        data = ply_bytes([("vertex", rows)])
        _, t, sh, op = _gpu(data)
        rt, rsh, rop = orc.ply_decode(data)
        _same(t, rt)
        _same(sh, rsh)
        _same(op, rop)


@pytest.mark.parametrize("rest", [0, 9, 45])
def test_compressed_decode_matches_oracle(cuda, orc, rest):
    data = ply_bytes(compressed_elements(5000, sh_rest=rest, seed=rest))
    for sub in (None, 7):
        msg, t, sh, op = _gpu(data, sub)
        rt, rsh, rop = orc.ply_decode(data, sub or 1)
        assert msg.compressed
        _same(t, rt)
        _same(sh, rsh)
        _same(op, rop)


def test_export_matches_oracle_and_round_trips(cuda, orc):
    from brush_b200.ply import splat_to_ply
    from brush_b200.splats import Splats

    rng = np.random.default_rng(7)
    for c in (1, 4, 9, 16):
        n = 4099
        t = rng.normal(size=(n, 10)).astype(np.float32)
        sh = rng.normal(size=(n, c, 3)).astype(np.float32)
        op = rng.normal(size=n).astype(np.float32)
        s = Splats(torch.from_numpy(t).cuda(), torch.from_numpy(sh).cuda(), torch.from_numpy(op).cuda())
        data = splat_to_ply(s, up_axis=(0.0, -1.0, 0.5))
        head_end = data.index(b"end_header\n") + len(b"end_header\n")
        head = data[:head_end].decode()
        assert head.count("property float f_rest_") == 3 * (c - 1)
        assert f"comment SH degree: {int(round(c ** 0.5)) - 1}" in head
        assert "comment Vertical axis: 0 -1 0.5" in head and "SplatRenderMode: default" in head
        assert data[head_end:] == orc.ply_encode_rows(t, sh, op)
        msg, t2, sh2, op2 = _gpu(data)
        q = t[:, 3:7]
        nrm = np.maximum(np.sqrt(((q[:, 0] * q[:, 0] + q[:, 1] * q[:, 1]) + q[:, 2] * q[:, 2]) + q[:, 3] * q[:, 3]),
                         np.float32(1e-12))
        _same(t2[:, :3], t[:, :3])
        _same(t2[:, 7:], t[:, 7:])
        _same(t2[:, 3:7], (q / nrm[:, None]).astype(np.float32))
        _same(sh2, sh)
        _same(op2, op)
        assert msg.meta.up_axis == (0.0, -1.0, 0.5)


def test_loaded_splats_render(cuda):
    """A file written from a training scene loads into splats that render like the originals."""
    import brush_b200 as bsx
    from brush_b200.ply import load_splat_from_ply, splat_to_ply
    from brush_b200.splats import config1_scene

    splats, cam, size, _ = config1_scene("cuda", seed=5)
    q = splats.transforms[:, 3:7]
    splats.transforms[:, 3:7] = q / q.norm(dim=1, keepdim=True)
    a = bsx.render(cam, size, splats.transforms, splats.sh_coeffs, splats.raw_opacities).out_img.cpu().numpy()
    back = load_splat_from_ply(splat_to_ply(splats)).splats
    b = bsx.render(cam, size, back.transforms, back.sh_coeffs, back.raw_opacities).out_img.cpu().numpy()
    assert np.abs(a - b).max() <= 1e-4

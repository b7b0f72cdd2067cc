"""PLY import: host-side header parsing and validation of the C ABI (no GPU), and the
CPU oracle's decode pinned against known answers. Cases follow the reference's own
tests (crates/brush-serde/src/import.rs tests :756-1198, quant.rs tests :63-112,
export.rs tests :193-349); the files are written by tests/plyfiles.py."""
import ctypes as C
import struct

import numpy as np
import pytest

from plyfiles import compressed_elements, ply_bytes, splat_rows


def _parse(bsx_lib, data, subsample=1):
    L = bsx_lib.lib()
    info = bsx_lib.PlyInfo()
    h = C.c_void_p()
    err = C.create_string_buffer(512)
    buf = (C.c_uint8 * max(len(data), 1)).from_buffer_copy(data or b"\0")
    st = L.bsx_ply_parse(buf, len(data), subsample, C.byref(h), C.byref(info), err, 512)
    if h:
        L.bsx_ply_free(h)
    return st, info, err.value.decode()


def _error(bsx_lib, data, subsample=1):
    st, _, msg = _parse(bsx_lib, data, subsample)
    assert st == 8, (st, msg)  # BSX_ERR_FORMAT
    return msg


def test_truncated_binary_is_an_eof_error(bsx_lib):
    data = ply_bytes([("vertex", splat_rows(2, degree=0))])
    assert "Unexpected EOF" in _error(bsx_lib, data[:-10])


def test_partial_ascii_token_is_an_error(bsx_lib):
    head = b"ply\nformat ascii 1.0\nelement vertex 1\nproperty float x\nproperty float y\nproperty float z\nend_header\n"
    _error(bsx_lib, head + b"1.0 2.0 3e")
    st, info, _ = _parse(bsx_lib, head + b"1.0 2.0 3.0")  # final token without newline is fine
    assert st == 0 and info.num_splats == 1


def test_zero_rows_zero_subsample_and_unknown_format(bsx_lib):
    assert "no vertices" in _error(bsx_lib, ply_bytes([("vertex", splat_rows(0, degree=0))]))
    assert "no vertices" in _error(bsx_lib, ply_bytes(compressed_elements(0)[:1] + [("vertex", compressed_elements(1)[1][1][:0])]))
    assert "greater than zero" in _error(bsx_lib, ply_bytes([("vertex", splat_rows(3))]), subsample=0)
    assert "Unknown format" in _error(bsx_lib, ply_bytes([("face", splat_rows(3))]))


def test_colour_and_sh_schema_validation(bsx_lib):
    partial_rgb = splat_rows(1, degree=0, drop=("f_dc_0", "f_dc_1", "f_dc_2"), extra=[("red", "u1", 3)])
    assert "exactly one red, green, and blue" in _error(bsx_lib, ply_bytes([("vertex", partial_rgb)]))
    dt = [(n, "f4") for n in ("x", "y", "z", "f_dc_0", "f_dc_1", "f_dc_2")] + [(f"f_rest_{k}", "f4") for k in range(75)]
    assert "Unsupported SH rest property count" in _error(bsx_lib, ply_bytes([("vertex", np.zeros(1, dtype=dt))]))
    gap = [(n, "f4") for n in ("x", "y", "z", "f_dc_0", "f_dc_1", "f_dc_2")] + [(f"f_rest_{k}", "f4") for k in range(1, 10)]
    assert "contiguous" in _error(bsx_lib, ply_bytes([("vertex", np.zeros(1, dtype=gap))]))
    two_dc = splat_rows(1, degree=0, drop=("f_dc_2",))
    assert "f_dc_0, f_dc_1, and f_dc_2" in _error(bsx_lib, ply_bytes([("vertex", two_dc)]))
    rest_only = splat_rows(1, degree=1, drop=("f_dc_0", "f_dc_1", "f_dc_2"))
    assert "complete DC or RGB" in _error(bsx_lib, ply_bytes([("vertex", rest_only)]))
    els = compressed_elements(4, sh_rest=9)
    bad_sh = np.zeros(4, dtype=[(f"f_rest_{k}", "u1") for k in range(75)])
    assert "Unsupported SH rest property count" in _error(bsx_lib, ply_bytes(els[:2] + [("sh", bad_sh)]))


def test_compressed_needs_chunk_rows_and_complete_blocks(bsx_lib):
    els = compressed_elements(300, sh_rest=9)  # 2 chunk rows needed
    assert "chunk rows" in _error(bsx_lib, ply_bytes([("chunk", els[0][1][:1])] + els[1:]))
    full = ply_bytes(els)
    assert "Unexpected EOF" in _error(bsx_lib, full[:-5])
    head = full[: full.index(b"end_header\n") + len(b"end_header\n")]
    assert "Unexpected EOF" in _error(bsx_lib, head + els[0][1].tobytes()[:-3])
    st, info, _ = _parse(bsx_lib, full)
    assert st == 0 and info.compressed == 1 and info.sh_coeffs == 4 and info.num_splats == 300


def test_header_metadata_and_subsample(bsx_lib):
    rows = splat_rows(10, degree=2)
    data = ply_bytes([("vertex", rows)], comments=["Vertical axis: 0.5, -1, 2", "SplatRenderMode: mip"])
    st, info, _ = _parse(bsx_lib, data, subsample=3)
    assert st == 0 and info.num_splats == 4 and info.total_rows == 10 and info.sh_coeffs == 9
    assert info.render_mode == 1 and info.has_up_axis == 1 and list(info.up_axis) == [0.5, -1.0, 2.0]
    st, info, _ = _parse(bsx_lib, ply_bytes([("vertex", rows)], comments=["vertical axis: z"]), subsample=100)
    assert st == 0 and info.num_splats == 1 and list(info.up_axis) == [0.0, 0.0, -1.0] and info.render_mode == -1


def test_oracle_decode_known_answers(orc):
    # standard rows decode to the written floats; SH rest re-interleaved channel-major -> [coeff][channel]
    rows = splat_rows(5, degree=1, seed=3)
    t, sh, op = orc.ply_decode(ply_bytes([("vertex", rows)]))
    assert np.array_equal(t[:, 0], rows["x"]) and np.array_equal(t[:, 3], rows["rot_0"])
    assert np.array_equal(t[:, 7], rows["scale_0"]) and np.array_equal(op, rows["opacity"])
    assert np.array_equal(sh[:, 0, 1], rows["f_dc_1"])
    assert np.array_equal(sh[:, 2, 0], rows["f_rest_1"]) and np.array_equal(sh[:, 1, 2], rows["f_rest_6"])
    # absent groups take the Splats defaults
    bare = splat_rows(2, degree=0, drop=("rot_0", "rot_1", "rot_2", "rot_3", "scale_0", "scale_1", "scale_2",
                                         "opacity", "f_dc_0", "f_dc_1", "f_dc_2"))
    t, sh, op = orc.ply_decode(ply_bytes([("vertex", bare)]))
    assert (t[:, 3:7] == [1, 0, 0, 0]).all() and (t[:, 7:] == -4).all() and (op == 0).all() and (sh == 0.5).all()
    # u8 RGB override: (v / 255 - 0.5) / SH_C0
    rgb = splat_rows(1, degree=0, extra=[("red", "u1", 255), ("green", "u1", 0), ("blue", "u1", 128)])
    _, sh, _ = orc.ply_decode(ply_bytes([("vertex", rgb)]))
    c0 = np.float32(0.2820948)
    assert sh[0, 0, 0] == (np.float32(1.0) - np.float32(0.5)) / c0
    assert sh[0, 0, 2] == (np.float32(128) / np.float32(255) - np.float32(0.5)) / c0


def test_oracle_compressed_decode_known_answers(orc):
    # quant.rs tests: decode_vec_11_10_11(0) = 0, all-ones = 1; the zero-centred quaternion is unit length
    els = compressed_elements(2, seed=1)
    chunk, vert = els[0][1], els[1][1]
    for b in chunk.dtype.names:
        chunk[b] = 0.0 if b.startswith("min") else 1.0
    vert["packed_position"] = [0, (0x7FF << 21) | (0x3FF << 11) | 0x7FF]
    vert["packed_rotation"] = [(512 << 20) | (512 << 10) | 512, (3 << 30) | (512 << 20) | (512 << 10) | 512]
    vert["packed_color"] = [0xFF00FF80, 0x000000FF - 1]
    t, sh, op = orc.ply_decode(ply_bytes(els))
    assert (t[0, :3] == 0).all() and (t[1, :3] == 1).all()
    for r in range(2):
        assert abs(float(np.linalg.norm(t[r, 3:7])) - 1.0) < 1e-5
    assert t[1, 6] == t[1, 3:7].max()  # "largest" = 3 is the z slot (stored w x y z)
    assert op[0] == orc.logf(np.float32(128 / 255) / (np.float32(1) - np.float32(128 / 255)))


def test_oracle_export_rows_field_layout(orc):
    rng = np.random.default_rng(2)
    n, c = 3, 9
    t = rng.normal(size=(n, 10)).astype(np.float32)
    sh = rng.normal(size=(n, c, 3)).astype(np.float32)
    op = rng.normal(size=n).astype(np.float32)
    rows = np.frombuffer(orc.ply_encode_rows(t, sh, op), np.float32).reshape(n, 14 + 3 * (c - 1))
    q = t[:, 3:7]
    nrm = np.sqrt(((q[:, 0] * q[:, 0] + q[:, 1] * q[:, 1]) + q[:, 2] * q[:, 2]) + q[:, 3] * q[:, 3])
    assert np.array_equal(rows[:, 7:11], q / nrm[:, None])
    assert np.array_equal(rows[:, 11:14], sh[:, 0, :])
    # f_rest_{channel * 8 + k} = sh[k + 1, channel]
    assert np.array_equal(rows[:, 14 + 8 * 2 + 3], sh[:, 4, 2])
    assert struct.pack("<f", t[0, 0]) == rows[0, :1].tobytes()

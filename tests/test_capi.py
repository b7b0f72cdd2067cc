"""The C ABI library loads without a GPU, exports exactly what include/bsx.h declares,
and its host-only camera -> uniforms function agrees bit-for-bit with the oracle's."""
import ctypes as C
import math
import re
import subprocess
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent


def _declared():
    text = (ROOT / "include" / "bsx.h").read_text()
    return sorted(set(re.findall(r"BSX_API\s+[\w\s\*]+?\b(bsx_\w+)\s*\(", text)))


def test_library_exports_every_declared_symbol(bsx_lib):
    lib = bsx_lib.lib()
    declared = _declared()
    assert len(declared) >= 19
    for name in declared:
        assert hasattr(lib, name), name
    out = subprocess.run(["nm", "-D", "--defined-only", str(bsx_lib.LIB_PATH)], capture_output=True, text=True).stdout
    exported = sorted(set(re.findall(r" T (bsx_\w+)", out)))
    assert exported == declared
    assert sorted(bsx_lib.SIGNATURES) == declared


def test_status_strings_and_abi(bsx_lib):
    lib = bsx_lib.lib()
    assert lib.bsx_abi_version() == 7
    assert lib.bsx_status_string(0) == b"ok"
    assert lib.bsx_status_string(4) == b"device wait timed out"
    assert lib.bsx_status_string(8) == b"malformed file"


def test_uniforms_match_oracle_bit_exact(bsx_lib, orc):
    from brush_b200.camera import Camera

    rng = np.random.default_rng(0)
    for k in range(20):
        pos = rng.normal(0, 5, 3)
        cam = Camera.look_at(tuple(pos), tuple(rng.normal(0, 1, 3)), math.radians(rng.uniform(20, 100)), 1297, 840)
        u = cam.project_uniforms(1297, 840, 3, 12345)
        o = orc.make_uniforms(cam, 1297, 840, 3, 12345)
        assert bytes(u) == bytes(o), k


# distortion coefficients of the camera-model tests (camera.rs tests use the same kinds)
MODEL_PARAMS = {1: (0.05, -0.01, 0.002, -0.0004, 0, 0, 0, 0),
                2: (-0.12, 0.03, -0.002, 0.01, -0.004, 0.0005, 0.001, -0.0015),
                3: (0.04, -0.008, 0.001, -0.0002, 0.0008, -0.0006, 0.0009, -0.0007)}


def test_camera_model_uniforms_match_oracle(bsx_lib, orc):
    """Per-model focal length (camera.rs:85-101) and clamp limits (camera.rs:200-254)."""
    import dataclasses

    from brush_b200.camera import Camera, focal_to_fov, fov_to_focal

    rng = np.random.default_rng(1)
    for model, kp in MODEL_PARAMS.items():
        for k in range(6):
            cam = Camera.look_at(tuple(rng.normal(0, 5, 3)), (0.0, 0.0, 0.0), math.radians(rng.uniform(40, 150)),
                                 640, 480)
            cam = dataclasses.replace(cam, camera_model=model, model_params=kp, center_uv=(0.47, 0.53))
            u = cam.project_uniforms(640, 480, 3, 99)
            assert bytes(u) == bytes(orc.make_uniforms(cam, 640, 480, 3, 99)), (model, k)
            assert u.camera_model == model and np.allclose(list(u.model_params), kp)
            f = fov_to_focal(cam.fov_x, 640, model, kp)
            assert abs(u.fx - f) <= 1e-6 * f
            assert abs(focal_to_fov(f, 640, model, kp) - cam.fov_x) < 1e-9
            if model == 2:
                # clamp bounds are the undistorted edges, r * radial(r) = distorted edge, where the
                # fixed-point inverse converges (moderate fields of view)
                from brush_b200.camera import _rt8_radial
                edge = (1.15 * 640 - u.cx) / u.fx
                r = u.lim_pos_x
                if edge < 1.0:
                    assert abs(r * _rt8_radial(r, kp) - edge) < 1e-5
            else:
                assert u.lim_pos_x == 0.0 and u.lim_neg_y == 0.0


def test_invalid_arguments_rejected_without_gpu(bsx_lib):
    lib = bsx_lib.lib()
    assert lib.bsx_render_fwd(None, None, 0, 0, None, None, None, 0, 0, 0, 0, None, None) == 1
    assert lib.bsx_make_project_uniforms(None, 1, 1, 0, 0, None) == 1


def _c_category(decl: str) -> str:
    decl = decl.strip()
    if "*" in decl or "[" in decl:
        return "ptr"
    base = re.sub(r"\b(const|unsigned|signed|struct)\b", "", decl).split()[0]
    if base == "void":
        return "void"
    table = {"uint32_t": "u32", "int32_t": "i32", "int": "i32", "float": "f32", "double": "f64",
             "uint64_t": "u64", "size_t": "u64", "int64_t": "i64"}
    if base in table:
        return table[base]
    if base in ("bsx_status", "bsx_render_mode", "bsx_raster_pass", "bsx_camera_model"):
        return "i32"  # C enums are int-sized
    raise AssertionError(f"unmapped C type {decl!r}")


def _ctypes_category(t) -> str:
    import ctypes as C

    if t is None:
        return "void"
    if t in (C.c_void_p, C.c_char_p) or (isinstance(t, type) and issubclass(t, C._Pointer)):
        return "ptr"
    for cats, name in (((C.c_uint32, C.c_uint), "u32"), ((C.c_int32, C.c_int), "i32"), ((C.c_float,), "f32"),
                       ((C.c_double,), "f64"), ((C.c_uint64, C.c_size_t), "u64"), ((C.c_int64,), "i64")):
        if t in cats:
            return name
    raise AssertionError(f"unmapped ctypes type {t!r}")


def test_bindings_match_header_signatures(bsx_lib):
    """Every ctypes binding has the header's parameter count and, per parameter, the same
    kind (pointer, 32/64-bit integer, float) and return kind: a mismatch would pass wrong
    arguments across the ABI without any error."""
    text = (ROOT / "include" / "bsx.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    decls = re.findall(r"BSX_API\s+([\w\s\*]+?)\b(bsx_\w+)\s*\(([^;]*?)\)\s*;", text, flags=re.S)
    assert len(decls) == len(_declared())
    for ret, name, params in decls:
        params = " ".join(params.split())
        cats = [] if params in ("", "void") else [_c_category(p) for p in params.split(",")]
        restype, argtypes = bsx_lib.SIGNATURES[name]
        got = [_ctypes_category(t) for t in argtypes]
        assert got == cats, f"{name}: header {cats} vs binding {got}"
        assert _ctypes_category(restype) == _c_category(ret), name


def test_integration_binding_declares_every_entry_point():
    """The Rust FFI block of the integration guide names exactly the header's entry points."""
    doc = set(re.findall(r"pub fn (bsx_\w+)", (ROOT / "INTEGRATION.md").read_text()))
    assert doc == set(_declared())


_STRUCTS = {"Camera": "bsx_camera", "ProjectUniforms": "bsx_project_uniforms", "RenderOut": "bsx_render_out",
            "LossCfg": "bsx_loss_cfg", "AdamGroup": "bsx_adam_group", "AdamCfg": "bsx_adam_cfg",
            "DpGroup": "bsx_dp_group", "DpExchange": "bsx_dp_exchange", "TrainConfig": "bsx_train_config",
            "TrainStats": "bsx_train_stats", "DpSplats": "bsx_dp_splats", "RefineConfig": "bsx_refine_config",
            "RefineStats": "bsx_refine_stats", "PlyInfo": "bsx_ply_info"}


_ORACLE_STRUCTS = {"_Camera": "bsx_camera", "Uniforms": "bsx_project_uniforms", "LossCfg": "bsx_loss_cfg",
                   "RefineCfg": "bsx_refine_config", "RefineStats": "bsx_refine_stats"}


@pytest.mark.parametrize("side", ["library", "oracle"])
def test_struct_layouts_match_header(bsx_lib, tmp_path, side):
    """Every ctypes mirror of a header struct (the library's bindings and the oracle's) has the C
    compiler's size and, field by field, the same name and offset: a missing or misplaced field
    would make the C side read garbage."""
    import ctypes as C
    import subprocess

    if side == "library":
        mod, structs = bsx_lib, _STRUCTS
    else:
        from oracle import oracle as mod

        structs = _ORACLE_STRUCTS
    lines = ["#include <stdio.h>", "#include <stddef.h>", f'#include "{ROOT / "include" / "bsx.h"}"',
             "int main(void) {"]
    for py, cname in structs.items():
        lines.append(f'  printf("{py} size %zu\\n", sizeof({cname}));')
        for field, _ in getattr(mod, py)._fields_:
            lines.append(f'  printf("{py} {field} %zu\\n", offsetof({cname}, {field}));')
    lines += ["  return 0;", "}"]
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines) + "\n")
    exe = tmp_path / "layout"
    res = subprocess.run(["gcc", "-std=c11", str(src), "-o", str(exe)], capture_output=True, text=True)
    assert res.returncode == 0, res.stderr  # a ctypes field missing from the C struct fails here
    got = {}
    for ln in subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.splitlines():
        py, key, val = ln.split()
        got[(py, key)] = int(val)
    for py in structs:
        st = getattr(mod, py)
        assert C.sizeof(st) == got[(py, "size")], py  # a C field missing from ctypes changes the size
        for field, _ in st._fields_:
            assert getattr(st, field).offset == got[(py, field)], (py, field)

"""numpy front-end of the CPU oracle (``oracle/oracle.cpp``).

TEST INFRASTRUCTURE ONLY: imported by tests/, by ``__graft_entry__.smoke()``
and by ``bench.py``'s CPU-baseline leg as the checker / CPU baseline, never by
the product path.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "_build" / "liboracle.so"

_lib = None


class _Camera(C.Structure):
    _fields_ = [("fov_x", C.c_double), ("fov_y", C.c_double), ("center_uv", C.c_float * 2),
                ("position", C.c_float * 3), ("rotation", C.c_float * 4), ("camera_model", C.c_int32),
                ("model_params", C.c_float * 8)]


class Uniforms(C.Structure):
    _fields_ = [("viewmat", C.c_float * 12), ("fx", C.c_float), ("fy", C.c_float), ("cx", C.c_float),
                ("cy", C.c_float), ("camera_pos", C.c_float * 3), ("half_max_render_fov", C.c_float),
                ("lim_pos_x", C.c_float), ("lim_pos_y", C.c_float), ("lim_neg_x", C.c_float),
                ("lim_neg_y", C.c_float), ("img_w", C.c_uint32), ("img_h", C.c_uint32),
                ("tile_bw", C.c_uint32), ("tile_bh", C.c_uint32), ("sh_degree", C.c_uint32),
                ("total_splats", C.c_uint32), ("num_visible", C.c_uint32), ("camera_model", C.c_int32),
                ("model_params", C.c_float * 8)]


class LossCfg(C.Structure):
    _fields_ = [("l1_weight", C.c_float), ("ssim_weight", C.c_float), ("composite_bg", C.c_int32),
                ("bg", C.c_float * 3), ("mask", C.c_int32)]


class RefineCfg(C.Structure):
    """bsx_refine_config (include/bsx.h)."""
    _fields_ = [("max_splats", C.c_uint32), ("growth_grad_threshold", C.c_float),
                ("growth_select_fraction", C.c_float), ("growth_stop_iter", C.c_uint32),
                ("split_at_screen_size", C.c_float), ("opac_decay", C.c_float), ("scale_decay", C.c_float),
                ("min_scale_prune", C.c_int32), ("min_scale_prune_threshold", C.c_float),
                ("near_zero_rotation_prune", C.c_int32), ("radial_bounds_prune", C.c_int32),
                ("min_opacity", C.c_float), ("prune_extent_factor", C.c_float),
                ("split_long_axis_scale", C.c_float), ("split_other_axis_scale", C.c_float),
                ("split_opacity_scale", C.c_float), ("seed", C.c_uint64), ("rule", C.c_int32),
                ("percent_dense", C.c_float)]


class RefineStats(C.Structure):
    _fields_ = [(name, C.c_uint32) for name in ("num_added", "num_split_oversized", "num_split_high_grad",
                                                 "num_pruned", "num_pruned_non_finite", "total_splats")]


_lib_path = None


def use_library(path) -> None:
    """Load the restatement from ``path`` (e.g. the -march=native timing build) instead of the
    portable build; must precede the first call into the oracle."""
    global _lib_path
    if _lib is not None and Path(path) != Path(_lib_path or LIB):
        raise RuntimeError("the oracle library is already loaded")
    _lib_path = Path(path)


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        path = _lib_path or LIB
        if path == LIB and not LIB.exists():
            from .build import build

            build()
        _lib = C.CDLL(str(path))
        f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
        u32p = np.ctypeslib.ndpointer(np.uint32, flags="C_CONTIGUOUS")
        _lib.orc_make_project_uniforms.argtypes = [C.POINTER(_Camera), C.c_uint32, C.c_uint32, C.c_uint32,
                                                   C.c_uint32, C.POINTER(Uniforms)]
        _lib.orc_render.restype = C.c_void_p
        _lib.orc_render.argtypes = [C.POINTER(Uniforms), f32p, f32p, f32p, C.c_uint32, C.c_uint32, C.c_int,
                                    C.c_int, f32p]
        _lib.orc_render_free.argtypes = [C.c_void_p]
        _lib.orc_render_sizes.argtypes = [C.c_void_p, u32p]
        _lib.orc_render_get.restype = C.c_size_t
        _lib.orc_render_get.argtypes = [C.c_void_p, C.c_int, C.c_void_p]
        _lib.orc_rasterize_bwd.argtypes = [C.c_void_p, f32p, C.c_int, f32p]
        _lib.orc_project_bwd.argtypes = [C.POINTER(Uniforms), f32p, f32p, f32p, C.c_uint32, C.c_uint32, C.c_int,
                                         f32p, f32p, f32p, f32p, f32p]
        _lib.orc_loss_fwd.argtypes = [f32p, u32p, C.c_uint32, C.c_uint32, C.c_uint32, C.POINTER(LossCfg), f32p]
        _lib.orc_loss_bwd.argtypes = [f32p, u32p, C.c_uint32, C.c_uint32, C.c_uint32, C.POINTER(LossCfg), f32p,
                                      f32p]
        _lib.orc_adam.argtypes = [f32p, f32p, f32p, f32p, C.c_uint32, C.c_uint32, C.c_float, C.c_void_p, C.c_int,
                                  C.c_float, C.c_float, C.c_float, C.c_uint32, C.c_float]
        _lib.orc_radix_argsort_u32.argtypes = [u32p, u32p, C.c_uint32, C.c_uint32, u32p, u32p]
        _lib.orc_prefix_sum_u32.argtypes = [u32p, C.c_uint32, u32p]
        _lib.orc_tile_offsets.argtypes = [u32p, C.c_uint32, C.c_uint32, u32p]
        _lib.orc_rasterize_rows.argtypes = [f32p, C.c_uint32, C.c_uint32, C.c_uint32, f32p, C.c_int, f32p]
        _lib.orc_gauss_taps.argtypes = [f32p]
        u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")
        _lib.orc_refine_prune_mask.argtypes = [f32p, f32p, f32p, C.c_uint32, C.c_uint32, C.POINTER(RefineCfg), f32p,
                                               C.c_float, u8p]
        _lib.orc_refine_plan.restype = C.c_void_p
        _lib.orc_refine_plan.argtypes = [f32p, f32p, f32p, f32p, f32p, f32p, C.c_uint32, C.c_uint32,
                                         C.POINTER(RefineCfg), f32p, f32p, C.c_uint32, C.c_uint32,
                                         C.POINTER(RefineStats)]
        _lib.orc_refine_plan2.restype = C.c_void_p
        _lib.orc_refine_plan2.argtypes = [f32p, f32p, f32p, f32p, f32p, f32p, f32p, C.c_uint32, C.c_uint32,
                                          C.POINTER(RefineCfg), f32p, f32p, C.c_uint32, C.c_uint32,
                                          C.POINTER(RefineStats)]
        _lib.orc_refine_plan_rows.argtypes = [C.c_void_p, u32p, u32p]
        _lib.orc_refine_apply.argtypes = [C.c_void_p] + [f32p] * 18 + [C.c_uint32, C.c_uint32]
        _lib.orc_refine_free.argtypes = [C.c_void_p]
        _lib.orc_weighted_sample.restype = C.c_uint32
        _lib.orc_weighted_sample.argtypes = [f32p, C.c_uint32, C.c_uint32, C.c_uint64, C.c_uint32, u32p]
        _lib.orc_refine_uniform.restype = C.c_float
        _lib.orc_refine_uniform.argtypes = [C.c_uint64, C.c_uint32, C.c_uint32]
        _lib.orc_expf.restype = C.c_float
        _lib.orc_expf.argtypes = [C.c_float]
        _lib.orc_logf.restype = C.c_float
        _lib.orc_atan2f.restype = C.c_float
        _lib.orc_atan2f.argtypes = [C.c_float, C.c_float]
        _lib.orc_ply_decode.restype = C.c_int
        _lib.orc_ply_decode.argtypes = [C.c_char_p, C.c_size_t, C.c_uint32, C.POINTER(C.c_uint32),
                                        C.POINTER(C.c_uint32), C.c_void_p, C.c_void_p, C.c_void_p, C.c_char_p,
                                        C.c_size_t]
        _lib.orc_ply_encode_rows.restype = C.c_uint64
        _lib.orc_ply_encode_rows.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_uint32, C.c_uint32, C.c_void_p]
        _lib.orc_raster_sigma.restype = C.c_float
        _lib.orc_raster_sigma.argtypes = [C.c_float] * 5
        _lib.orc_expf_raster_max_ulp.restype = C.c_double
        _lib.orc_expf_raster_max_ulp.argtypes = [C.c_float, C.c_uint32]
        _lib.orc_logf.argtypes = [C.c_float]
        _lib.orc_set_threads.argtypes = [C.c_int]
        _lib.orc_set_raster_expr.argtypes = [C.c_int]
        _lib.orc_mean_noise_step.argtypes = [f32p, f32p, f32p, C.c_uint32, C.c_float, C.c_float, C.c_uint64,
                                             C.c_uint32]
        _lib.orc_sincos_2pi.argtypes = [C.c_float, C.POINTER(C.c_float), C.POINTER(C.c_float)]
        _lib.orc_normal3.argtypes = [C.c_uint64, C.c_uint32, C.c_uint32, f32p]
        _lib.orc_normal3_many.argtypes = [C.c_uint64, C.c_uint32, C.c_uint32, f32p]
        _lib.orc_sincos_2pi_max_err.argtypes = [np.ctypeslib.ndpointer(np.float64, flags="C_CONTIGUOUS")]
        _lib.orc_powi.restype = C.c_float
        _lib.orc_powi.argtypes = [C.c_float, C.c_uint32]
        _lib.orc_raster_decision_flips.argtypes = [C.c_void_p, np.ctypeslib.ndpointer(np.uint64,
                                                                                    flags="C_CONTIGUOUS")]
        _lib.orc_get_threads.restype = C.c_int
    return _lib


def set_raster_expr(reference: bool) -> None:
    """Raster arithmetic of the renders and raster backwards that follow: the kernels' fused
    form (False, the default) or the reference's expression (True: unfused calc_sigma, e^-sigma
    correctly rounded, pix += max(c, 0) * vis; rasterize.rs:131-155)."""
    lib().orc_set_raster_expr(int(bool(reference)))


def raster_decision_flips(render: "RenderResult") -> dict:
    """Pairs where the two raster arithmetics decide differently along ``render``'s trajectory."""
    out = np.zeros(4, np.uint64)
    lib().orc_raster_decision_flips(render._h, out)
    return dict(pairs=int(out[0]), accept_flips=int(out[1]), early_out_flips=int(out[2]), pixels=int(out[3]))


def mean_noise_step(transforms, raw_opac, gate, scale, limit, seed, step):
    """The mean-noise step (train.rs:1095-1169) on a copy of ``transforms`` [N,10]; returns it."""
    t = _f32(transforms).reshape(-1, 10).copy()
    lib().orc_mean_noise_step(t.reshape(-1), _f32(raw_opac).reshape(-1), _f32(gate).reshape(-1), t.shape[0],
                              float(scale), float(limit), int(seed), int(step))
    return t


def sincos_2pi(u: float):
    s, c = C.c_float(), C.c_float()
    lib().orc_sincos_2pi(float(u), C.byref(s), C.byref(c))
    return s.value, c.value


def normal3(seed: int, step: int, index: int) -> np.ndarray:
    z = np.zeros(3, np.float32)
    lib().orc_normal3(int(seed), int(step), int(index), z)
    return z


def normal3_many(seed: int, step: int, n: int) -> np.ndarray:
    z = np.zeros((n, 3), np.float32)
    lib().orc_normal3_many(int(seed), int(step), int(n), z.reshape(-1))
    return z


def sincos_2pi_max_err():
    out = np.zeros(2, np.float64)
    lib().orc_sincos_2pi_max_err(out)
    return float(out[0]), float(out[1])


def powi(b: float, e: int) -> float:
    return float(lib().orc_powi(float(b), int(e)))


def set_threads(n: int) -> None:
    lib().orc_set_threads(int(n))


def threads() -> int:
    return int(lib().orc_get_threads())


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.float32))


def _u32(a) -> np.ndarray:
    a = np.asarray(a)
    if a.dtype == np.int32:
        a = a.view(np.uint32)
    return np.ascontiguousarray(a.astype(np.uint32, copy=False))


def camera_c(cam) -> _Camera:
    c = _Camera()
    c.fov_x, c.fov_y = float(cam.fov_x), float(cam.fov_y)
    c.center_uv[:] = [float(v) for v in cam.center_uv]
    c.position[:] = [float(v) for v in cam.position]
    c.rotation[:] = [float(v) for v in cam.rotation]
    c.camera_model = int(cam.camera_model)
    mp = list(getattr(cam, "model_params", ())) + [0.0] * 8
    c.model_params[:] = [float(v) for v in mp[:8]]
    return c


def make_uniforms(cam, w: int, h: int, sh_degree: int = 0, total: int = 0) -> Uniforms:
    u = Uniforms()
    c = camera_c(cam)
    if lib().orc_make_project_uniforms(C.byref(c), w, h, sh_degree, total, C.byref(u)) != 0:
        raise ValueError("unsupported camera")
    return u


_FIELDS = {"projected": (0, np.float32), "counts": (1, np.uint32), "max_radius": (2, np.float32),
           "depth_order": (3, np.uint32), "cum": (4, np.uint32), "isect_tile": (5, np.uint32),
           "isect_gid": (6, np.uint32), "tile_offsets": (7, np.uint32), "image": (8, np.float32),
           "image_packed": (9, np.uint32), "visible": (10, np.float32)}


class RenderResult:
    """Forward render on the CPU; holds the C++ state needed by ``rasterize_bwd``."""

    def __init__(self, cam, img_size, transforms, sh, raw_opac, mip=False, raster_pass=1, bg=(0.0, 0.0, 0.0)):
        self.w, self.h = int(img_size[0]), int(img_size[1])
        self.transforms = _f32(transforms).reshape(-1, 10)
        n = self.transforms.shape[0]
        self.sh = _f32(sh).reshape(n, -1, 3)
        self.coeffs = self.sh.shape[1]
        self.raw_opac = _f32(raw_opac).reshape(n)
        self.mip = int(bool(mip))
        deg = int(round(self.coeffs ** 0.5)) - 1
        self.uniforms = make_uniforms(cam, self.w, self.h, deg, n)
        self.n = n
        self._h = lib().orc_render(C.byref(self.uniforms), self.transforms, self.sh, self.raw_opac, n, self.coeffs,
                                   self.mip, int(raster_pass), _f32(bg))
        sizes = np.zeros(4, dtype=np.uint32)
        lib().orc_render_sizes(self._h, sizes)
        self.num_visible, self.num_intersections, self.tile_bw, self.tile_bh = (int(v) for v in sizes)
        for name, (idx, dt) in _FIELDS.items():
            count = lib().orc_render_get(self._h, idx, None)
            arr = np.empty(count, dtype=dt)
            if count:
                lib().orc_render_get(self._h, idx, arr.ctypes.data)
            setattr(self, name, arr)
        self.projected = self.projected.reshape(n, 12)
        if self.image.size:
            self.image = self.image.reshape(self.h, self.w, 4)
        if self.image_packed.size:
            self.image_packed = self.image_packed.reshape(self.h, self.w)
        self.tile_offsets = self.tile_offsets.reshape(self.tile_bh, self.tile_bw, 2)

    def rasterize_bwd(self, v_output, compute_refine_weight=True) -> np.ndarray:
        out = np.zeros((self.n, 11), dtype=np.float32)
        lib().orc_rasterize_bwd(self._h, _f32(v_output).reshape(-1), int(compute_refine_weight), out)
        return out

    def project_bwd(self, v_combined):
        n, c = self.n, self.coeffs
        vt = np.zeros((n, 10), np.float32)
        vs = np.zeros((n, c, 3), np.float32)
        vo = np.zeros(n, np.float32)
        vr = np.zeros(n, np.float32)
        lib().orc_project_bwd(C.byref(self.uniforms), self.transforms, self.sh, self.raw_opac, n, c, self.mip,
                              _f32(v_combined).reshape(n, 11), vt, vs, vo, vr)
        return vt, vs, vo, vr

    def __del__(self):
        h = getattr(self, "_h", None)
        if h:
            lib().orc_render_free(h)
            self._h = None


def loss_cfg(l1_weight=0.8, ssim_weight=-0.2, composite_bg=None, mask=False) -> LossCfg:
    c = LossCfg()
    c.l1_weight, c.ssim_weight = float(l1_weight), float(ssim_weight)
    c.composite_bg = int(composite_bg is not None)
    c.bg[:] = [float(v) for v in (composite_bg or (0.0, 0.0, 0.0))]
    c.mask = int(mask)
    return c


def loss_fwd(pred_chw, gt_packed, cfg: LossCfg) -> np.ndarray:
    p = _f32(pred_chw)
    ch, h, w = p.shape
    out = np.empty_like(p)
    lib().orc_loss_fwd(p.reshape(-1), _u32(gt_packed).reshape(-1), w, h, ch, C.byref(cfg), out.reshape(-1))
    return out


def loss_bwd(pred_chw, gt_packed, cfg: LossCfg, dl_dmap) -> np.ndarray:
    p = _f32(pred_chw)
    ch, h, w = p.shape
    out = np.empty_like(p)
    lib().orc_loss_bwd(p.reshape(-1), _u32(gt_packed).reshape(-1), w, h, ch, C.byref(cfg),
                       _f32(dl_dmap).reshape(-1), out.reshape(-1))
    return out


def adam(param, grad, m, v, lr, col_scale=None, reduce=False, beta1=0.9, beta2=0.999, eps=1e-15, step=1,
         grad_scale=1.0):
    """In place on param/m/v (2-D float32 arrays; v is [rows] when reduce)."""
    rows, cols = param.shape
    sc = None
    if col_scale is not None:
        sc_arr = _f32(col_scale)
        sc = sc_arr.ctypes.data
    lib().orc_adam(param.reshape(-1), _f32(grad).reshape(-1), m.reshape(-1), v.reshape(-1), rows, cols, float(lr),
                   sc, int(reduce), beta1, beta2, eps, int(step), float(grad_scale))


def radix_argsort(keys, values, bits):
    k, v = _u32(keys), _u32(values)
    ko, vo = np.empty_like(k), np.empty_like(v)
    lib().orc_radix_argsort_u32(k, v, k.size, int(bits), ko, vo)
    return ko, vo


def prefix_sum(values):
    v = _u32(values)
    out = np.empty_like(v)
    lib().orc_prefix_sum_u32(v, v.size, out)
    return out


def tile_offsets(ids, num_tiles):
    ids = _u32(ids)
    out = np.zeros(num_tiles * 2, dtype=np.uint32)
    lib().orc_tile_offsets(ids, ids.size, num_tiles, out)
    return out.reshape(num_tiles, 2)


def rasterize_rows(rows10, w, h, bg=(0.0, 0.0, 0.0), smooth=False) -> np.ndarray:
    r = _f32(rows10).reshape(-1, 10)
    out = np.empty((h, w, 4), dtype=np.float32)
    lib().orc_rasterize_rows(r.reshape(-1), r.shape[0], w, h, _f32(bg), int(smooth), out.reshape(-1))
    return out


def gauss_taps() -> np.ndarray:
    out = np.empty(11, dtype=np.float32)
    lib().orc_gauss_taps(out)
    return out


def expf(x: float) -> float:
    return float(lib().orc_expf(float(x)))


def logf(x: float) -> float:
    return float(lib().orc_logf(float(x)))


def ply_decode(data: bytes, subsample: int = 1):
    """CPU restatement of load_splat_from_ply: (transforms [N,10], sh [N,C,3], opacities [N])."""
    n, c = C.c_uint32(), C.c_uint32()
    err = C.create_string_buffer(512)
    if lib().orc_ply_decode(data, len(data), subsample, C.byref(n), C.byref(c), None, None, None, err, 512):
        raise ValueError(err.value.decode())
    t = np.zeros((n.value, 10), np.float32)
    sh = np.zeros((n.value, c.value, 3), np.float32)
    op = np.zeros(n.value, np.float32)
    if lib().orc_ply_decode(data, len(data), subsample, C.byref(n), C.byref(c), t.ctypes.data, sh.ctypes.data,
                            op.ctypes.data, err, 512):
        raise ValueError(err.value.decode())
    return t, sh, op


def ply_encode_rows(t, sh, op) -> bytes:
    """The vertex rows splat_to_ply writes (without the header)."""
    t, sh, op = _f32(t).reshape(-1, 10), _f32(sh), _f32(op).reshape(-1)
    n = t.shape[0]
    c = sh.reshape(n, -1, 3).shape[1]
    sh = sh.reshape(n, c, 3)
    size = lib().orc_ply_encode_rows(t.ctypes.data, sh.ctypes.data, op.ctypes.data, n, c, None)
    out = np.zeros(size, np.uint8)
    lib().orc_ply_encode_rows(t.ctypes.data, sh.ctypes.data, op.ctypes.data, n, c, out.ctypes.data)
    return out.tobytes()


def atan2f(y: float, x: float) -> float:
    return float(lib().orc_atan2f(float(y), float(x)))


def raster_sigma(c00: float, c01: float, c11: float, dx: float, dy: float) -> float:
    """The rasterizers' sigma (bsx_raster_sigma) as the kernels and this restatement evaluate it."""
    return float(lib().orc_raster_sigma(c00, c01, c11, dx, dy))


def expf_raster_max_ulp(lo: float, stride: int = 1) -> float:
    """Largest ulp error of bsx_expf_raster over every stride-th float in [lo, 0]
    against the double-precision exponential (-1 if a result is not finite and positive)."""
    return float(lib().orc_expf_raster_max_ulp(float(lo), int(stride)))


def refine_cfg(**kw) -> RefineCfg:
    """bsx_refine_config with the reference defaults (config.rs:100-330), overridden by kw."""
    d = dict(max_splats=10_000_000, growth_grad_threshold=0.0025, growth_select_fraction=0.07,
             growth_stop_iter=15000, split_at_screen_size=0.5, opac_decay=0.004, scale_decay=0.002,
             min_scale_prune=1, min_scale_prune_threshold=1e-10, near_zero_rotation_prune=1,
             radial_bounds_prune=0, min_opacity=1.0 / 255.0, prune_extent_factor=100.0,
             split_long_axis_scale=0.5, split_other_axis_scale=0.85, split_opacity_scale=0.6, seed=42, rule=0,
             percent_dense=0.01)
    d.update(kw)
    c = RefineCfg()
    for k, v in d.items():
        setattr(c, k, v)
    return c


def refine_prune_mask(t, sh, op, cfg, center, max_allowed):
    n = t.shape[0]
    out = np.empty(n, np.uint8)
    lib().orc_refine_prune_mask(_f32(t).reshape(-1), _f32(sh).reshape(-1), _f32(op).reshape(-1), n,
                                _f32(sh).reshape(n, -1).shape[1] // 3 if n else 1, C.byref(cfg),
                                _f32(center), float(max_allowed), out)
    return out


def refine(t, sh, op, record, moments, cfg, center, extent, global_iter, refine_count, phase_iter, phase_total):
    """Prune / replace / split / grow (train.rs:1191-1860), or with cfg.rule = 1 the gradient-threshold
    clone / split rule. record = (refine_norm, vis, screen[, grad2d_accum]);
    moments = ((m_t [n,10], m_s [n,3C], m_o [n]), (v_t [n,10], v_s [n], v_o [n])). Returns
    dict(stats, keep, split, transforms, sh, opac, m, v)."""
    n, c = t.shape[0], sh.shape[1]
    st = RefineStats()
    grad2d = record[3] if len(record) > 3 else np.zeros(n, np.float32)
    h = lib().orc_refine_plan2(_f32(t).reshape(-1), _f32(sh).reshape(-1), _f32(op).reshape(-1),
                               *[_f32(x).reshape(-1) for x in record[:3]], _f32(grad2d).reshape(-1), n, c,
                               C.byref(cfg), _f32(center), _f32(extent), int(global_iter), int(refine_count),
                               C.byref(st))
    try:
        K = st.total_splats - st.num_added
        keep = np.empty(max(K, 1), np.uint32)
        split = np.empty(max(st.num_added, 1), np.uint32)
        if cfg.rule == 0:
            lib().orc_refine_plan_rows(h, keep, split)
        n2 = st.total_splats
        nt, nsh, nop = np.empty((n2, 10), np.float32), np.empty((n2, c, 3), np.float32), np.empty(n2, np.float32)
        nm = (np.empty((n2, 10), np.float32), np.empty((n2, 3 * c), np.float32), np.empty(n2, np.float32))
        nv = (np.empty((n2, 10), np.float32), np.empty(n2, np.float32), np.empty(n2, np.float32))
        (m_t, m_s, m_o), (v_t, v_s, v_o) = moments
        lib().orc_refine_apply(h, _f32(t).reshape(-1), _f32(sh).reshape(-1), _f32(op).reshape(-1),
                               *[_f32(x).reshape(-1) for x in (m_t, m_s, m_o, v_t, v_s, v_o)],
                               nt.reshape(-1), nsh.reshape(-1), nop, *[x.reshape(-1) for x in nm + nv],
                               int(phase_iter), int(phase_total))
    finally:
        lib().orc_refine_free(h)
    return dict(stats=st, keep=keep[:K], split=split[:st.num_added], transforms=nt, sh=nsh, opac=nop, m=nm, v=nv)


def refine_uniform(seed, stream, index) -> float:
    return float(lib().orc_refine_uniform(int(seed), int(stream), int(index)))


def weighted_sample(w, k, seed=42, stream=0):
    """Up to k distinct indices drawn without replacement with probability proportional to w."""
    w = _f32(w)
    out = np.empty(max(k, 1), np.uint32)
    m = lib().orc_weighted_sample(w, w.size, int(k), int(seed), int(stream), out)
    return out[:m].astype(np.int64)

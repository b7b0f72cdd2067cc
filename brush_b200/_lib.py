"""ctypes binding of the C ABI declared in ``include/bsx.h``.

The shared library is loaded from the package directory (``brush_b200/libbsx.so``,
built by ``brush_b200/build.py``). There is no fallback: if the library is
missing or cannot be loaded, every entry point raises.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libbsx.so"

BSX_COMPACT_GRAD_LANES = 11
REFINE_REFERENCE = 0
REFINE_GRAD_THRESHOLD = 1
BSX_GRAD_STRIDE = 12
BSX_PROJECTED_LANES = 12
BSX_TILE_WIDTH = 16
BSX_MAX_RANKS = 8
BSX_PEER_HANDLE_BYTES = 64
BSX_DP_FLAG_WORDS = 64

STATUS_NAMES = {
    0: "BSX_OK",
    1: "BSX_ERR_INVALID_ARG",
    2: "BSX_ERR_SHAPE",
    3: "BSX_ERR_CAPACITY",
    4: "BSX_ERR_DEVICE_TIMEOUT",
    5: "BSX_ERR_CUDA",
    6: "BSX_ERR_STATE",
    7: "BSX_ERR_UNSUPPORTED",
    8: "BSX_ERR_FORMAT",
}

RENDER_DEFAULT, RENDER_MIP = 0, 1
PASS_FORWARD, PASS_BACKWARD, PASS_BACKWARD_SMOOTH_CUTOFF = 0, 1, 2


class BsxError(RuntimeError):
    """A bsx entry point returned a non-OK status."""

    def __init__(self, status: int, message: str):
        self.status = status
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {message}")


class Camera(C.Structure):
    _fields_ = [
        ("fov_x", C.c_double),
        ("fov_y", C.c_double),
        ("center_uv", C.c_float * 2),
        ("position", C.c_float * 3),
        ("rotation", C.c_float * 4),
        ("camera_model", C.c_int32),
        ("model_params", C.c_float * 8),
    ]


CAMERA_PINHOLE, CAMERA_KANNALA_BRANDT_4, CAMERA_RADIAL_TANGENTIAL_8, CAMERA_THIN_PRISM_FISHEYE = 0, 1, 2, 3


class ProjectUniforms(C.Structure):
    _fields_ = [
        ("viewmat", C.c_float * 12),
        ("fx", C.c_float),
        ("fy", C.c_float),
        ("cx", C.c_float),
        ("cy", C.c_float),
        ("camera_pos", C.c_float * 3),
        ("half_max_render_fov", C.c_float),
        ("lim_pos_x", C.c_float),
        ("lim_pos_y", C.c_float),
        ("lim_neg_x", C.c_float),
        ("lim_neg_y", C.c_float),
        ("img_w", C.c_uint32),
        ("img_h", C.c_uint32),
        ("tile_bw", C.c_uint32),
        ("tile_bh", C.c_uint32),
        ("sh_degree", C.c_uint32),
        ("total_splats", C.c_uint32),
        ("num_visible", C.c_uint32),
        ("camera_model", C.c_int32),
        ("model_params", C.c_float * 8),
    ]


class RenderOut(C.Structure):
    _fields_ = [
        ("d_image", C.c_void_p),
        ("d_image_packed", C.c_void_p),
        ("d_visible", C.c_void_p),
        ("d_max_radius", C.c_void_p),
        ("d_tile_offsets", C.c_void_p),
        ("d_projected", C.c_void_p),
        ("d_isect_gid", C.c_void_p),
        ("d_isect_tile", C.c_void_p),
        ("d_depth_order", C.c_void_p),
        ("d_tile_counts", C.c_void_p),
        ("d_cum_counts", C.c_void_p),
        ("num_visible", C.c_uint32),
        ("num_intersections", C.c_uint32),
        ("tile_bw", C.c_uint32),
        ("tile_bh", C.c_uint32),
        ("uniforms", ProjectUniforms),
    ]


class LossCfg(C.Structure):
    _fields_ = [
        ("l1_weight", C.c_float),
        ("ssim_weight", C.c_float),
        ("composite_bg", C.c_int32),
        ("bg", C.c_float * 3),
        ("mask", C.c_int32),
    ]


class AdamGroup(C.Structure):
    _fields_ = [
        ("d_param", C.c_void_p),
        ("d_grad", C.c_void_p),
        ("d_m", C.c_void_p),
        ("d_v", C.c_void_p),
        ("rows", C.c_uint32),
        ("cols", C.c_uint32),
        ("lr", C.c_float),
        ("h_col_scale", C.POINTER(C.c_float)),
        ("reduce_moment_2", C.c_int32),
    ]


class AdamCfg(C.Structure):
    _fields_ = [
        ("beta_1", C.c_float),
        ("beta_2", C.c_float),
        ("epsilon", C.c_float),
        ("step", C.c_uint32),
        ("grad_scale", C.c_float),
    ]


class DpGroup(C.Structure):
    _fields_ = [
        ("d_param", C.c_void_p * BSX_MAX_RANKS),
        ("d_grad", C.c_void_p * BSX_MAX_RANKS),
        ("d_param_mc", C.c_void_p),
        ("d_grad_mc", C.c_void_p),
        ("d_m", C.c_void_p),
        ("d_v", C.c_void_p),
        ("rows", C.c_uint32),
        ("cols", C.c_uint32),
        ("lr", C.c_float),
        ("h_col_scale", C.POINTER(C.c_float)),
        ("reduce_moment_2", C.c_int32),
    ]


class DpExchange(C.Structure):
    _fields_ = [
        ("rank", C.c_int32),
        ("world", C.c_int32),
        ("d_flags", C.c_void_p * BSX_MAX_RANKS),
        ("d_refine", C.c_void_p * BSX_MAX_RANKS),
        ("refine_rows", C.c_uint32),
        ("epoch", C.c_uint32),
        ("timeout_ns", C.c_uint64),
        ("grad_slot_rows", C.c_uint32),
        ("d_gate", C.c_void_p * BSX_MAX_RANKS),
        ("gate_rows", C.c_uint32),
        ("d_refine_mc", C.c_void_p),
        ("d_gate_mc", C.c_void_p),
    ]


class TrainConfig(C.Structure):
    _fields_ = [
        ("total_train_iters", C.c_uint32),
        ("lr_mean", C.c_double),
        ("lr_mean_end", C.c_double),
        ("lr_coeffs_dc", C.c_double),
        ("lr_coeffs_sh_scale", C.c_float),
        ("lr_opac", C.c_double),
        ("lr_scale", C.c_double),
        ("lr_scale_end", C.c_double),
        ("lr_rotation", C.c_double),
        ("ssim_weight", C.c_float),
        ("background", C.c_float * 3),
        ("median_scale", C.c_float),
        ("uniform_lr", C.c_float),
        ("render_mode", C.c_int32),
        ("gather_stats", C.c_int32),
        ("mean_noise", C.c_int32),
        ("noise_vis_gate", C.c_int32),
        ("mean_noise_weight", C.c_float),
        ("noise_seed", C.c_uint64),
        ("accumulate_grad2d", C.c_int32),
    ]


class TrainStats(C.Structure):
    _fields_ = [
        ("num_visible", C.c_uint32),
        ("num_intersections", C.c_uint32),
        ("lr_mean", C.c_float),
        ("step", C.c_uint32),
    ]


class DpSplats(C.Structure):
    _fields_ = [(name, C.c_void_p * BSX_MAX_RANKS) for name in
                ("d_transforms", "d_sh_coeffs", "d_raw_opac", "d_v_transforms", "d_v_sh_coeffs", "d_v_raw_opac")] + \
               [(name, C.c_void_p) for name in
                ("mc_transforms", "mc_sh_coeffs", "mc_raw_opac", "mc_v_transforms", "mc_v_sh_coeffs", "mc_v_raw_opac")]


class RefineConfig(C.Structure):
    _fields_ = [
        ("max_splats", C.c_uint32),
        ("growth_grad_threshold", C.c_float),
        ("growth_select_fraction", C.c_float),
        ("growth_stop_iter", C.c_uint32),
        ("split_at_screen_size", C.c_float),
        ("opac_decay", C.c_float),
        ("scale_decay", C.c_float),
        ("min_scale_prune", C.c_int32),
        ("min_scale_prune_threshold", C.c_float),
        ("near_zero_rotation_prune", C.c_int32),
        ("radial_bounds_prune", C.c_int32),
        ("min_opacity", C.c_float),
        ("prune_extent_factor", C.c_float),
        ("split_long_axis_scale", C.c_float),
        ("split_other_axis_scale", C.c_float),
        ("split_opacity_scale", C.c_float),
        ("seed", C.c_uint64),
        ("rule", C.c_int32),
        ("percent_dense", C.c_float),
    ]


class RefineStats(C.Structure):
    _fields_ = [(name, C.c_uint32) for name in ("num_added", "num_split_oversized", "num_split_high_grad",
                                                 "num_pruned", "num_pruned_non_finite", "total_splats")]


class PlyInfo(C.Structure):
    _fields_ = [
        ("num_splats", C.c_uint32),
        ("total_rows", C.c_uint32),
        ("sh_coeffs", C.c_uint32),
        ("subsample", C.c_uint32),
        ("compressed", C.c_int32),
        ("render_mode", C.c_int32),
        ("has_up_axis", C.c_int32),
        ("up_axis", C.c_float * 3),
    ]


# name -> (restype, argtypes); exactly the functions include/bsx.h declares.
SIGNATURES = {
    "bsx_create": (C.c_int, [C.c_int, C.POINTER(C.c_void_p)]),
    "bsx_destroy": (C.c_int, [C.c_void_p]),
    "bsx_set_stream": (C.c_int, [C.c_void_p, C.c_void_p]),
    "bsx_trim": (C.c_int, [C.c_void_p]),
    "bsx_sync": (C.c_int, [C.c_void_p]),
    "bsx_last_error": (C.c_char_p, [C.c_void_p]),
    "bsx_status_string": (C.c_char_p, [C.c_int]),
    "bsx_abi_version": (C.c_int, []),
    "bsx_launch_count": (C.c_uint64, [C.c_void_p]),
    "bsx_profile_enable": (C.c_int, [C.c_void_p, C.c_int32]),
    "bsx_profile_collect": (C.c_int, [C.c_void_p]),
    "bsx_profile_count": (C.c_int32, [C.c_void_p]),
    "bsx_profile_entry": (
        C.c_int, [C.c_void_p, C.c_int32, C.POINTER(C.c_char_p), C.POINTER(C.c_double), C.POINTER(C.c_uint64)]
    ),
    "bsx_profile_reset": (C.c_int, [C.c_void_p]),
    "bsx_make_project_uniforms": (
        C.c_int,
        [C.POINTER(Camera), C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32, C.POINTER(ProjectUniforms)],
    ),
    "bsx_render_fwd": (
        C.c_int,
        [C.c_void_p, C.POINTER(Camera), C.c_uint32, C.c_uint32, C.c_void_p, C.c_void_p, C.c_void_p, C.c_uint32,
         C.c_uint32, C.c_int32, C.c_int32, C.POINTER(C.c_float), C.POINTER(RenderOut)],
    ),
    "bsx_rasterize_bwd": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int32, C.c_void_p]),
    "bsx_project_bwd": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]),
    "bsx_rasterize_bwd_ref": (
        C.c_int,
        [C.c_void_p, C.c_void_p, C.c_void_p, C.c_uint32, C.c_void_p, C.c_uint32, C.c_void_p, C.POINTER(C.c_float),
         C.c_uint32, C.c_uint32, C.c_void_p, C.c_int32, C.c_int32, C.c_int32, C.c_void_p],
    ),
    "bsx_project_bwd_ref": (
        C.c_int,
        [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_uint32, C.c_uint32, C.c_void_p, C.c_uint32,
         C.POINTER(ProjectUniforms), C.c_int32, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p],
    ),
    "bsx_loss_fwd": (
        C.c_int,
        [C.c_void_p, C.c_void_p, C.c_void_p, C.c_uint32, C.c_uint32, C.c_uint32, C.POINTER(LossCfg), C.c_void_p],
    ),
    "bsx_loss_bwd": (
        C.c_int,
        [C.c_void_p, C.c_void_p, C.c_void_p, C.c_uint32, C.c_uint32, C.c_uint32, C.POINTER(LossCfg), C.c_void_p,
         C.c_void_p],
    ),
    "bsx_loss_fused": (
        C.c_int,
        [C.c_void_p, C.c_void_p, C.c_void_p, C.c_uint32, C.c_uint32, C.POINTER(LossCfg), C.c_void_p, C.c_void_p],
    ),
    "bsx_adam_step": (C.c_int, [C.c_void_p, C.POINTER(AdamGroup), C.c_int32, C.POINTER(AdamCfg)]),
    "bsx_peer_alloc": (C.c_int, [C.c_void_p, C.c_uint64, C.POINTER(C.c_void_p), C.c_char_p]),
    "bsx_peer_free": (C.c_int, [C.c_void_p, C.c_void_p]),
    "bsx_peer_open": (C.c_int, [C.c_void_p, C.c_char_p, C.POINTER(C.c_void_p)]),
    "bsx_peer_close": (C.c_int, [C.c_void_p, C.c_void_p]),
    "bsx_dp_adam_step": (
        C.c_int, [C.c_void_p, C.POINTER(DpExchange), C.POINTER(DpGroup), C.c_int32, C.POINTER(AdamCfg)]
    ),
    "bsx_trainer_create": (
        C.c_int, [C.c_void_p, C.c_uint32, C.c_uint32, C.POINTER(TrainConfig), C.POINTER(C.c_void_p)]
    ),
    "bsx_trainer_destroy": (C.c_int, [C.c_void_p]),
    "bsx_trainer_stats_buffers": (
        C.c_int, [C.c_void_p, C.POINTER(C.c_void_p), C.POINTER(C.c_void_p), C.POINTER(C.c_void_p)]
    ),
    "bsx_trainer_keep_gradients": (C.c_int, [C.c_void_p, C.c_int32]),
    "bsx_trainer_grad2d_accum": (C.c_int, [C.c_void_p, C.POINTER(C.c_void_p)]),
    "bsx_trainer_raster_grads": (C.c_int, [C.c_void_p, C.POINTER(C.c_void_p)]),
    "bsx_trainer_grad_buffers": (
        C.c_int,
        [C.c_void_p, C.POINTER(C.c_void_p), C.POINTER(C.c_void_p), C.POINTER(C.c_void_p), C.POINTER(C.c_void_p)],
    ),
    "bsx_train_step": (
        C.c_int,
        [C.c_void_p, C.POINTER(Camera), C.c_uint32, C.c_uint32, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
         C.c_int32, C.c_void_p, C.POINTER(TrainStats)],
    ),
    "bsx_train_step_dp": (
        C.c_int,
        [C.c_void_p, C.POINTER(Camera), C.c_uint32, C.c_uint32, C.c_void_p, C.POINTER(DpExchange),
         C.POINTER(DpSplats), C.c_int32, C.c_void_p, C.POINTER(TrainStats)],
    ),
    "bsx_trainer_refine_plan": (
        C.c_int,
        [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.POINTER(RefineConfig), C.POINTER(C.c_float),
         C.POINTER(C.c_float), C.c_uint32, C.POINTER(RefineStats)],
    ),
    "bsx_trainer_refine_apply": (
        C.c_int,
        [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_uint32,
         C.c_uint32],
    ),
    "bsx_trainer_set_median_scale": (C.c_int, [C.c_void_p, C.c_float]),
    "bsx_splat_bounds": (
        C.c_int, [C.c_void_p, C.c_void_p, C.c_uint32, C.c_uint32, C.c_float, C.POINTER(C.c_float),
                  C.POINTER(C.c_float)]
    ),
    "bsx_trainer_reserve": (C.c_int, [C.c_void_p, C.c_uint32]),
    "bsx_trainer_load_optimizer_state": (
        C.c_int, [C.c_void_p] + [C.c_void_p] * 6 + [C.c_uint32, C.c_int32, C.c_int32]
    ),
    "bsx_trainer_optimizer_state": (C.c_int, [C.c_void_p] + [C.POINTER(C.c_void_p)] * 6 + [C.POINTER(C.c_uint32)]),
    "bsx_mean_noise_step": (
        C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_uint32, C.c_float, C.c_float, C.c_uint64,
                  C.c_uint32]
    ),
    "bsx_radix_argsort_u32": (
        C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_uint32, C.c_uint32, C.c_void_p, C.c_void_p]
    ),
    "bsx_prefix_sum_u32": (C.c_int, [C.c_void_p, C.c_void_p, C.c_uint32, C.c_void_p]),
    "bsx_prefix_sum_u32_noalloc": (C.c_int, [C.c_void_p, C.c_uint32, C.c_void_p, C.c_void_p]),
    "bsx_get_tile_offsets": (C.c_int, [C.c_void_p, C.c_void_p, C.c_uint32, C.c_uint32, C.c_void_p]),
    "bsx_ply_parse": (
        C.c_int, [C.c_void_p, C.c_size_t, C.c_uint32, C.POINTER(C.c_void_p), C.POINTER(PlyInfo), C.c_char_p,
                  C.c_size_t]
    ),
    "bsx_ply_free": (None, [C.c_void_p]),
    "bsx_ply_load": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]),
    "bsx_ply_export_size": (C.c_int, [C.c_uint32, C.c_uint32, C.c_int32, C.POINTER(C.c_float),
                                      C.POINTER(C.c_uint64)]),
    "bsx_ply_export": (
        C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_uint32, C.c_uint32, C.c_int32,
                  C.POINTER(C.c_float), C.c_void_p, C.c_uint64, C.POINTER(C.c_uint64)]
    ),
}

_LIB = None


def lib() -> C.CDLL:
    """Load ``libbsx.so`` once; raise if it is absent (there is no CPU path)."""
    global _LIB
    if _LIB is None:
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"{LIB_PATH} is missing: build it with `python brush_b200/build.py` "
                "(the B200 CUDA library is required; there is no fallback)"
            )
        handle = C.CDLL(os.fspath(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _LIB = handle
    return _LIB


def check(status: int, ctx=None) -> None:
    if status != 0:
        msg = lib().bsx_last_error(ctx).decode() if ctx else lib().bsx_status_string(status).decode()
        raise BsxError(status, msg)

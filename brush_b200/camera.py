"""Camera, mirroring ``brush_render::camera::Camera`` (crates/brush-render/src/camera.rs:11-101).

The rotation is the camera-to-world quaternion stored (x, y, z, w) like glam.
Camera space is +x right, +y down, +z forward (depth); pixel (u, v) =
(fx x/z + cx, fy y/z + cy).
"""
from __future__ import annotations

import ctypes as C
import math
from dataclasses import dataclass, field

import numpy as np

from . import _lib


PINHOLE, KANNALA_BRANDT_4, RADIAL_TANGENTIAL_8, THIN_PRISM_FISHEYE = 0, 1, 2, 3


def _kb4_d(theta: float, p) -> float:
    """KB4 distortion polynomial d(theta) = theta + k1 t^3 + k2 t^5 + k3 t^7 + k4 t^9 (camera.rs:121-130)."""
    t2 = theta * theta
    t3 = t2 * theta
    t5 = t3 * t2
    t7 = t5 * t2
    t9 = t7 * t2
    return theta + float(np.float32(p[0])) * t3 + float(np.float32(p[1])) * t5 + float(np.float32(p[2])) * t7 \
        + float(np.float32(p[3])) * t9


def _kb4_dd(theta: float, p) -> float:
    t2 = theta * theta
    t4 = t2 * t2
    t6 = t4 * t2
    t8 = t6 * t2
    k = [float(np.float32(v)) for v in p[:4]]
    return 1.0 + 3.0 * k[0] * t2 + 5.0 * k[1] * t4 + 7.0 * k[2] * t6 + 9.0 * k[3] * t8


def _kb4_invert_d(target: float, p) -> float:
    """Newton solve of d(theta) = target on [0, pi] (camera.rs:145-170)."""
    if target <= 0.0:
        return 0.0
    theta = min(target, math.pi - 1e-6)
    for _ in range(50):
        f = _kb4_d(theta, p) - target
        fp = _kb4_dd(theta, p)
        if abs(fp) < 1e-12:
            break
        nxt = min(max(theta - f / fp, 0.0), math.pi)
        if abs(nxt - theta) < 1e-12:
            theta = nxt
            break
        theta = nxt
    return theta


def _rt8_radial(r: float, p) -> float:
    k = [float(np.float32(v)) for v in p[:6]]
    r2 = r * r
    r4 = r2 * r2
    r6 = r4 * r2
    return (1.0 + k[0] * r2 + k[1] * r4 + k[2] * r6) / (1.0 + k[3] * r2 + k[4] * r4 + k[5] * r6)


def _rt8_undistort_radius(r_d: float, p) -> float:
    """Fixed-point inverse of r * radial(r) = r_d (camera.rs:184-198)."""
    r = r_d
    for _ in range(30):
        factor = _rt8_radial(r, p)
        if abs(factor) < 1e-12:
            break
        r_new = r_d / factor
        if abs(r_new - r) < 1e-12:
            r = r_new
            break
        r = r_new
    return r


def fov_to_focal(fov: float, pixels: int, model: int = PINHOLE, params=(0.0,) * 8) -> float:
    """``fov_to_focal`` (camera.rs:85-101): focal f with pixels/2 = f * projection(fov/2)."""
    half = fov / 2.0
    if model == PINHOLE:
        proj = math.tan(half)
    elif model in (KANNALA_BRANDT_4, THIN_PRISM_FISHEYE):
        proj = _kb4_d(half, params)
    elif model == RADIAL_TANGENTIAL_8:
        r = math.tan(half)
        proj = r * _rt8_radial(r, params)
    else:
        raise ValueError(f"unknown camera model {model}")
    return (pixels / 2.0) / proj


def focal_to_fov(focal: float, pixels: int, model: int = PINHOLE, params=(0.0,) * 8) -> float:
    """``focal_to_fov`` (camera.rs:103-118)."""
    r_norm = (pixels / 2.0) / focal
    if model == PINHOLE:
        half = math.atan(r_norm)
    elif model in (KANNALA_BRANDT_4, THIN_PRISM_FISHEYE):
        half = _kb4_invert_d(r_norm, params)
    elif model == RADIAL_TANGENTIAL_8:
        half = math.atan(_rt8_undistort_radius(r_norm, params))
    else:
        raise ValueError(f"unknown camera model {model}")
    return 2.0 * half


def _mat_to_quat_xyzw(m: np.ndarray) -> np.ndarray:
    """Rotation matrix (columns = camera axes in world space) to an (x, y, z, w) quaternion."""
    m = np.asarray(m, dtype=np.float64)
    tr = m[0, 0] + m[1, 1] + m[2, 2]
    if tr > 0:
        s = math.sqrt(tr + 1.0) * 2
        w = 0.25 * s
        x = (m[2, 1] - m[1, 2]) / s
        y = (m[0, 2] - m[2, 0]) / s
        z = (m[1, 0] - m[0, 1]) / s
    elif m[0, 0] > m[1, 1] and m[0, 0] > m[2, 2]:
        s = math.sqrt(1.0 + m[0, 0] - m[1, 1] - m[2, 2]) * 2
        w = (m[2, 1] - m[1, 2]) / s
        x = 0.25 * s
        y = (m[0, 1] + m[1, 0]) / s
        z = (m[0, 2] + m[2, 0]) / s
    elif m[1, 1] > m[2, 2]:
        s = math.sqrt(1.0 + m[1, 1] - m[0, 0] - m[2, 2]) * 2
        w = (m[0, 2] - m[2, 0]) / s
        x = (m[0, 1] + m[1, 0]) / s
        y = 0.25 * s
        z = (m[1, 2] + m[2, 1]) / s
    else:
        s = math.sqrt(1.0 + m[2, 2] - m[0, 0] - m[1, 1]) * 2
        w = (m[1, 0] - m[0, 1]) / s
        x = (m[0, 2] + m[2, 0]) / s
        y = (m[1, 2] + m[2, 1]) / s
        z = 0.25 * s
    q = np.array([x, y, z, w])
    return q / np.linalg.norm(q)


@dataclass
class Camera:
    fov_x: float
    fov_y: float
    position: tuple = (0.0, 0.0, 0.0)
    rotation: tuple = (0.0, 0.0, 0.0, 1.0)  # (x, y, z, w), camera-to-world
    center_uv: tuple = (0.5, 0.5)
    camera_model: int = 0
    # distortion coefficients (include/bsx.h bsx_camera_model): KB4 k1..k4; RT8 k1..k6 p1 p2;
    # thin-prism fisheye k1..k4 p1 p2 sx1 sy1
    model_params: tuple = (0.0,) * 8

    @staticmethod
    def look_at(position, target=(0.0, 0.0, 0.0), fov_x: float = math.radians(60.0), img_w: int = 1,
                img_h: int = 1, up=(0.0, 1.0, 0.0)) -> "Camera":
        """Camera at ``position`` looking at ``target``; ``fov_x`` horizontal, fov_y from the aspect."""
        p = np.asarray(position, dtype=np.float64)
        t = np.asarray(target, dtype=np.float64)
        fwd = t - p
        fwd /= np.linalg.norm(fwd)
        upv = np.asarray(up, dtype=np.float64)
        if abs(float(np.dot(fwd, upv))) > 0.999:
            upv = np.array([0.0, 0.0, 1.0])
        right = np.cross(fwd, upv)
        right /= np.linalg.norm(right)
        down = np.cross(fwd, right)
        m = np.stack([right, down, fwd], axis=1)
        q = _mat_to_quat_xyzw(m)
        focal = fov_to_focal(fov_x, img_w)
        fov_y = focal_to_fov(focal, img_h)
        return Camera(fov_x=fov_x, fov_y=fov_y, position=tuple(float(v) for v in p),
                      rotation=tuple(float(v) for v in q))

    def to_c(self) -> _lib.Camera:
        c = _lib.Camera()
        c.fov_x = float(self.fov_x)
        c.fov_y = float(self.fov_y)
        c.center_uv[:] = [float(v) for v in self.center_uv]
        c.position[:] = [float(v) for v in self.position]
        c.rotation[:] = [float(v) for v in self.rotation]
        c.camera_model = int(self.camera_model)
        mp = list(self.model_params) + [0.0] * (8 - len(self.model_params))
        c.model_params[:] = [float(v) for v in mp[:8]]
        return c

    def project_uniforms(self, img_w: int, img_h: int, sh_degree: int = 0, total_splats: int = 0):
        """Host-side uniforms exactly as the library computes them (no GPU needed)."""
        u = _lib.ProjectUniforms()
        cam = self.to_c()
        _lib.check(_lib.lib().bsx_make_project_uniforms(C.byref(cam), img_w, img_h, sh_degree, total_splats,
                                                        C.byref(u)))
        return u

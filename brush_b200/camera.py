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


def fov_to_focal(fov: float, pixels: int) -> float:
    """Pinhole ``fov_to_focal`` (camera.rs:85-101)."""
    return (pixels / 2.0) / math.tan(fov / 2.0)


def focal_to_fov(focal: float, pixels: int) -> float:
    """Pinhole ``focal_to_fov`` (camera.rs:103-118)."""
    return 2.0 * math.atan((pixels / 2.0) / focal)


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
        return c

    def project_uniforms(self, img_w: int, img_h: int, sh_degree: int = 0, total_splats: int = 0):
        """Host-side uniforms exactly as the library computes them (no GPU needed)."""
        u = _lib.ProjectUniforms()
        cam = self.to_c()
        _lib.check(_lib.lib().bsx_make_project_uniforms(C.byref(cam), img_w, img_h, sh_degree, total_splats,
                                                        C.byref(u)))
        return u

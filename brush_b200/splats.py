"""Splat parameters (``Splats``, crates/brush-render/src/gaussian_splats.rs:110-127) and the
seeded synthetic scenes of the benchmark configurations.

No public dataset is used: every scene below is generated from a seed with
the shapes and value distributions the benchmark configurations name.
"""
from __future__ import annotations

import logging
import math
from dataclasses import dataclass

import numpy as np
import torch

from .camera import Camera

_log = logging.getLogger(__name__)


class SplatValidationError(ValueError):
    """A splat (or gradient) tensor holds NaN or Inf values, or has inconsistent shapes."""


def validate_tensor_val(t: torch.Tensor, name: str, min_val=None, max_val=None, strict: bool = True) -> dict:
    """NaN / Inf and out-of-range counts of a tensor (crates/brush-render/src/validation.rs:6-81).

    Range violations are logged. NaN and Inf are logged and, with ``strict`` (the
    reference promotes them to panics in its test and debug-validation builds), raise
    SplatValidationError naming the tensor and the first offending flat index."""
    v = t.detach().reshape(-1).float()
    nan = torch.isnan(v)
    inf = torch.isinf(v)
    finite = ~(nan | inf)
    counts = {"nan": int(nan.sum()), "inf": int(inf.sum()), "below_min": 0, "above_max": 0}
    if min_val is not None:
        counts["below_min"] = int((finite & (v < min_val)).sum())
    if max_val is not None:
        counts["above_max"] = int((finite & (v > max_val)).sum())
    first = {k: (int(torch.nonzero(m)[0, 0]) if c else None) for k, m, c in
             (("nan", nan, counts["nan"]), ("inf", inf, counts["inf"]))}
    if counts["nan"] or counts["inf"]:
        _log.error("tensor '%s': %d NaN (first @ %s), %d Inf (first @ %s) of %d total", name, counts["nan"],
                   first["nan"], counts["inf"], first["inf"], v.numel())
    if counts["below_min"]:
        _log.error("tensor '%s': %d values < %s of %d", name, counts["below_min"], min_val, v.numel())
    if counts["above_max"]:
        _log.error("tensor '%s': %d values > %s of %d", name, counts["above_max"], max_val, v.numel())
    if strict and (counts["nan"] or counts["inf"]):
        raise SplatValidationError(f"tensor '{name}' has {counts['nan']} NaNs (first @ {first['nan']}) and "
                                   f"{counts['inf']} Infs (first @ {first['inf']})")
    return counts


def validate_gradient(gradient: torch.Tensor, name: str, strict: bool = True) -> dict:
    """validate_gradient (validation.rs:83-85): NaN / Inf in a parameter gradient."""
    return validate_tensor_val(gradient, f"gradient_{name}", strict=strict)


@dataclass
class Splats:
    transforms: torch.Tensor     # [N,10] mean xyz, quat wxyz, log-scale xyz
    sh_coeffs: torch.Tensor      # [N,C,3]
    raw_opacities: torch.Tensor  # [N]
    render_mode: int = 0

    @property
    def num_splats(self) -> int:
        return int(self.transforms.shape[0])

    @property
    def sh_coeffs_per_splat(self) -> int:
        return int(self.sh_coeffs.shape[1])

    @property
    def sh_degree(self) -> int:
        return int(round(math.sqrt(self.sh_coeffs_per_splat))) - 1

    def means(self) -> torch.Tensor:
        return self.transforms[:, 0:3]

    def validate_values(self, strict: bool = True) -> dict:
        """Splats::validate_values (gaussian_splats.rs:323-379): every parameter free of
        NaN / Inf (raises with ``strict``), the reference's plausibility ranges logged
        (log-scales [-10, 10], scales [1e-20, 1e4] and [1e-6, 100], SH [-5, 5], raw
        opacity [-20, 20], opacity [0, 1]), and consistent shapes. The render path never
        calls it (as in the reference, where it is compiled only into test and debug
        builds): the kernels cull non-finite splats instead."""
        n = self.num_splats
        if self.transforms.dim() != 2 or self.transforms.shape[1] != 10:
            raise SplatValidationError("Transforms must be 10D (means(3) + quats(4) + log_scales(3))")
        if self.raw_opacities.shape != (n,):
            raise SplatValidationError("Inconsistent number of splats in opacity")
        if self.sh_coeffs.dim() != 3 or self.sh_coeffs.shape[2] != 3:
            raise SplatValidationError("SH coeffs must have 3 color channels")
        if self.sh_coeffs.shape[0] != n:
            raise SplatValidationError("Inconsistent number of splats in SH coeffs")
        t = self.transforms.detach().float()
        log_scales = t[:, 7:10]
        scales = torch.exp(log_scales)
        out = {
            "means": validate_tensor_val(t[:, 0:3], "means", strict=strict),
            "rotations": validate_tensor_val(t[:, 3:7], "rotations", strict=strict),
            "log_scales": validate_tensor_val(log_scales, "log_scales", -10.0, 10.0, strict),
            "scales": validate_tensor_val(scales, "scales", 1e-20, 10000.0, strict),
            "sh_coeffs": validate_tensor_val(self.sh_coeffs, "sh_coeffs", -5.0, 5.0, strict),
            "raw_opacity": validate_tensor_val(self.raw_opacities, "raw_opacity", -20.0, 20.0, strict),
            "opacities": validate_tensor_val(torch.sigmoid(self.raw_opacities.detach().float()), "opacities",
                                             0.0, 1.0, strict),
        }
        out["scales_plausible"] = validate_tensor_val(scales, "scales", 1e-6, 100.0, strict)
        return out

    def to(self, device) -> "Splats":
        return Splats(self.transforms.to(device), self.sh_coeffs.to(device), self.raw_opacities.to(device),
                      self.render_mode)

    def clone(self) -> "Splats":
        return Splats(self.transforms.clone(), self.sh_coeffs.clone(), self.raw_opacities.clone(), self.render_mode)

    @staticmethod
    def from_parts(means, quats_wxyz, log_scales, sh_coeffs, raw_opacities, render_mode: int = 0) -> "Splats":
        t = torch.cat([means, quats_wxyz, log_scales], dim=1).contiguous()
        return Splats(t, sh_coeffs.contiguous(), raw_opacities.contiguous(), render_mode)


def splat_bounds(means: torch.Tensor, percentile: float = 0.8):
    """Robust percentile AABB of the means as (center, extent), f32 as ``bounds_from_pos``
    computes it (crates/brush-train/src/splat_init.rs:130-158, bounding_box.rs:8-13).
    Device means go through the library (``bsx_splat_bounds``: order statistics by its radix
    sort under total_cmp); host means are sorted here."""
    if means.is_cuda:
        return _device_bounds(means, percentile)
    m = means.detach().float()
    p = np.float32(percentile)
    lo_v, hi_v = [], []
    for k in range(3):
        v = m[:, k]
        v = v[torch.isfinite(v)]
        if v.numel() == 0:  # an axis with no finite value: the unit box
            one = np.ones(3, np.float32)
            return np.zeros(3, np.float32), one
        n = v.numel()
        lo = int(np.float32((np.float32(1.0) - p) / np.float32(2.0)) * np.float32(n))
        hi = min(n - 1, int(np.float32((np.float32(1.0) + p) / np.float32(2.0)) * np.float32(n)))
        # order statistics by a full sort (on the tensor's device): the same values as select_nth
        vs = torch.sort(v).values
        pair = torch.stack([vs[lo], vs[hi]]).cpu().numpy()
        lo_v.append(pair[0])
        hi_v.append(pair[1])
    mn, mx = np.array(lo_v, np.float32), np.array(hi_v, np.float32)
    return (mx + mn) / np.float32(2.0), (mx - mn) / np.float32(2.0)


def _device_bounds(means: torch.Tensor, percentile: float):
    import ctypes as C

    from . import _lib
    from ._context import context

    if means.dim() != 2 or means.shape[1] != 3 or means.dtype != torch.float32 or means.stride(1) != 1:
        raise ValueError("means must be a float32 [N,3] view with unit column stride")
    ctx = context(means.device)
    center, extent = (C.c_float * 3)(), (C.c_float * 3)()
    ctx.check(_lib.lib().bsx_splat_bounds(ctx.handle, C.c_void_p(means.data_ptr()), int(means.stride(0)),
                                          int(means.shape[0]), float(np.float32(percentile)), center, extent))
    return np.array(center[:], np.float32), np.array(extent[:], np.float32)


def median_size(means: torch.Tensor, percentile: float = 0.8) -> float:
    """``BoundingBox::median_size`` of the robust percentile AABB (bounding_box.rs:23-29)."""
    _, ext = splat_bounds(means, percentile)
    return float(np.sort(ext)[1] * np.float32(2.0))


def _gen(device, seed):
    g = torch.Generator(device=device)
    g.manual_seed(int(seed))
    return g


def _normal(shape, mean, std, g, device):
    return torch.randn(shape, generator=g, device=device, dtype=torch.float32) * std + mean


def random_gt(h: int, w: int, seed: int, device="cpu") -> torch.Tensor:
    """Uniform random RGB ground truth, packed RGBA8 with alpha 255, as int32 [H,W]."""
    g = _gen(device, seed)
    rgb = torch.randint(0, 256, (h, w, 3), generator=g, device=device, dtype=torch.int32)
    packed = rgb[..., 0] | (rgb[..., 1] << 8) | (rgb[..., 2] << 16) | (255 << 24)
    return packed.to(torch.int32)


def _quats(n, g, device):
    q = torch.randn((n, 4), generator=g, device=device, dtype=torch.float32)
    return q / q.norm(dim=1, keepdim=True).clamp_min(1e-12)


def config1_scene(device="cpu", seed: int = 1, n: int = 16384):
    """16,384 splats, means U[-1,1]^3, log-scales N(-4,0.5), quats N(0,1) normalised,
    opacity logits N(0,1), SH degree 0 with DC N(0,0.3); pinhole at distance 3
    looking at the origin, fov 50 deg, 256x256; uniform random target."""
    g = _gen(device, seed)
    means = torch.rand((n, 3), generator=g, device=device) * 2.0 - 1.0
    log_scales = _normal((n, 3), -4.0, 0.5, g, device)
    quats = _quats(n, g, device)
    opac = _normal((n,), 0.0, 1.0, g, device)
    sh = _normal((n, 1, 3), 0.0, 0.3, g, device)
    splats = Splats.from_parts(means, quats, log_scales, sh, opac)
    w = h = 256
    cam = Camera.look_at((0.0, 0.0, -3.0), (0.0, 0.0, 0.0), math.radians(50.0), w, h)
    gt = random_gt(h, w, seed + 1000, device)
    return splats, cam, (w, h), gt


def clustered_scene(n: int, sh_degree: int, device="cpu", seed: int = 2, clusters: int = 64, radius: float = 5.0,
                    sigma: float = 0.3, log_scale_mean: float = -4.5, log_scale_std: float = 0.7,
                    opac_std: float = 1.5) -> Splats:
    """Means from ``clusters`` isotropic Gaussian clusters (sigma) with centres uniform
    inside a ball of ``radius``; log-scales N(mean, std); opacity logits N(0, opac_std);
    SH DC N(0,0.3) and higher bands N(0,0.1)."""
    g = _gen(device, seed)
    d = torch.randn((clusters, 3), generator=g, device=device)
    d = d / d.norm(dim=1, keepdim=True)
    r = radius * torch.rand((clusters, 1), generator=g, device=device) ** (1.0 / 3.0)
    centres = d * r
    idx = torch.randint(0, clusters, (n,), generator=g, device=device)
    means = centres[idx] + _normal((n, 3), 0.0, sigma, g, device)
    log_scales = _normal((n, 3), log_scale_mean, log_scale_std, g, device)
    quats = _quats(n, g, device)
    opac = _normal((n,), 0.0, opac_std, g, device)
    c = (sh_degree + 1) ** 2
    sh = _normal((n, c, 3), 0.0, 0.1, g, device)
    sh[:, 0, :] = _normal((n, 3), 0.0, 0.3, g, device)
    return Splats.from_parts(means, quats, log_scales, sh, opac)


def orbit_camera(i: int, count: int, radius: float, w: int, h: int, fov_deg: float = 60.0,
                 elevation: float = 0.3) -> Camera:
    th = 2.0 * math.pi * i / max(count, 1)
    pos = (radius * math.cos(th) * math.cos(elevation), radius * math.sin(elevation),
           radius * math.sin(th) * math.cos(elevation))
    return Camera.look_at(pos, (0.0, 0.0, 0.0), math.radians(fov_deg), w, h)


def hemisphere_cameras(count: int, radius: float, w: int, h: int, seed: int = 3, fov_deg: float = 60.0):
    rng = np.random.default_rng(seed)
    cams = []
    for _ in range(count):
        az = rng.uniform(0, 2 * math.pi)
        el = math.asin(rng.uniform(0.05, 0.95))
        pos = (radius * math.cos(el) * math.cos(az), radius * math.sin(el), radius * math.cos(el) * math.sin(az))
        cams.append(Camera.look_at(pos, (0.0, 0.0, 0.0), math.radians(fov_deg), w, h))
    return cams


def config2_scene(device="cuda", seed: int = 2, n: int = 1_000_000):
    """1M splats, SH degree 3, clustered means, 1920x1080, fov 60, radius-8 orbit camera."""
    splats = clustered_scene(n, 3, device, seed)
    w, h = 1920, 1080
    cam = orbit_camera(0, 1, 8.0, w, h)
    gt = random_gt(h, w, seed + 1000, device)
    return splats, cam, (w, h), gt


def config5_scene(device="cuda", seed: int = 5, n: int = 6_000_000):
    """6M splats, SH degree 3, log-scales N(-5,0.8), 3840x2160 (viewer path)."""
    splats = clustered_scene(n, 3, device, seed, log_scale_mean=-5.0, log_scale_std=0.8)
    return splats, (3840, 2160)


def perturbed(splats: Splats, seed: int, mean_std: float = 0.02, dc_std: float = 0.05) -> Splats:
    """A seed-perturbed copy: means + N(0, mean_std), SH DC + N(0, dc_std)."""
    dev = splats.transforms.device
    g = _gen(dev, seed)
    p = splats.clone()
    p.transforms[:, 0:3] += _normal((p.num_splats, 3), 0.0, mean_std, g, dev)
    p.sh_coeffs[:, 0, :] += _normal((p.num_splats, 3), 0.0, dc_std, g, dev)
    return p


def config3_scene(device="cuda", seed: int = 3, n: int = 3_000_000, views: int = 200):
    """3M splats, SH degree 3, config-2 distributions; ``views`` cameras on a radius-8
    hemisphere at 1297x840. Targets are rendered (by this library's forward pass)
    from a seed-perturbed copy of the splats, one per view."""
    from .render import render_splats

    splats = clustered_scene(n, 3, device, seed)
    w, h = 1297, 840
    cams = hemisphere_cameras(views, 8.0, w, h, seed=seed)
    src = perturbed(splats, seed + 7)
    gts = [render_splats(src, c, (w, h), packed=True)[0].clone() for c in cams]
    return splats, cams, (w, h), gts


def circle_cameras(count: int, radius: float, w: int, h: int, fov_deg: float = 60.0, elevation: float = 0.3):
    """``count`` cameras on a horizontal circle looking at the origin (viewer path)."""
    return [orbit_camera(i, count, radius, w, h, fov_deg, elevation) for i in range(count)]

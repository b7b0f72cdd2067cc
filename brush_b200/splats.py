"""Splat parameters (``Splats``, crates/brush-render/src/gaussian_splats.rs:110-127) and the
seeded synthetic scenes of the benchmark configurations.

No public dataset is used: every scene below is generated from a seed with
the shapes and value distributions the benchmark configurations name.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np
import torch

from .camera import Camera


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
    computes it (crates/brush-train/src/splat_init.rs:130-158, bounding_box.rs:8-13)."""
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

"""Forward render, mirroring ``SplatOps::render`` (crates/brush-render/src/lib.rs:69-88)
and ``RenderOutput`` / ``RenderAuxInner`` (crates/brush-render/src/render_aux.rs:16-68).

Differences of representation (same meaning):
- projected rows, ``visible``, ``max_radius`` and gradients are indexed by the
  global splat id, so ``global_from_compact_gid`` is the identity and
  ``compact_gid_from_isect`` holds global ids;
- projected rows have 12 lanes (the reference's 10 + ln(255*opacity) + pad).
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field

import torch

from . import _lib
from ._context import context, device_view, ptr
from .camera import Camera

SplatRenderMode = type("SplatRenderMode", (), {"Default": _lib.RENDER_DEFAULT, "Mip": _lib.RENDER_MIP})
RasterPass = type(
    "RasterPass",
    (),
    {
        "Forward": _lib.PASS_FORWARD,
        "Backward": _lib.PASS_BACKWARD,
        "BackwardSmoothCutoff": _lib.PASS_BACKWARD_SMOOTH_CUTOFF,
    },
)


@dataclass
class RenderAux:
    num_visible: int
    num_intersections: int
    visible: torch.Tensor       # [N] f32 (backward passes) else empty
    max_radius: torch.Tensor    # [N] f32
    tile_offsets: torch.Tensor  # [ty, tx, 2] int32 (u32 bits)
    img_size: tuple             # (w, h)


@dataclass
class RenderOutput:
    out_img: torch.Tensor                 # [H,W,4] f32, or [H,W] int32 packed RGBA8 (forward pass)
    aux: RenderAux
    projected_splats: torch.Tensor        # [N,12]
    compact_gid_from_isect: torch.Tensor  # [M] int32, global ids, tile-major front-to-back
    isect_tile: torch.Tensor              # [M] int32, sorted tile id per intersection
    depth_order: torch.Tensor             # [V] int32, visible ids sorted by depth
    tile_counts: torch.Tensor             # [N] int32
    cum_counts: torch.Tensor              # [V] int32 inclusive scan of counts in depth order
    project_uniforms: _lib.ProjectUniforms
    num_splats: int = 0
    _gid: torch.Tensor | None = field(default=None, repr=False)

    @property
    def global_from_compact_gid(self) -> torch.Tensor:
        """Identity [N] int32 (global-id indexing), built on first access so that a render
        loop does not allocate and fill N ids per frame."""
        if self._gid is None:
            self._gid = torch.arange(self.num_splats, device=self.projected_splats.device, dtype=torch.int32)
        return self._gid


def _check_splats(transforms, sh_coeffs, raw_opacities):
    if transforms.dim() != 2 or transforms.shape[1] != 10:
        raise ValueError(f"transforms must be [N,10], got {tuple(transforms.shape)}")
    n = transforms.shape[0]
    if sh_coeffs.dim() != 3 or sh_coeffs.shape[0] != n or sh_coeffs.shape[2] != 3:
        raise ValueError(f"sh_coeffs must be [N,C,3], got {tuple(sh_coeffs.shape)}")
    if raw_opacities.dim() != 1 or raw_opacities.shape[0] != n:
        raise ValueError(f"raw_opacities must be [N], got {tuple(raw_opacities.shape)}")
    for t in (transforms, sh_coeffs, raw_opacities):
        if t.dtype != torch.float32 or not t.is_cuda:
            raise ValueError("splat tensors must be float32 CUDA tensors")


def render(camera: Camera, img_size: tuple, transforms: torch.Tensor, sh_coeffs: torch.Tensor,
           raw_opacities: torch.Tensor, render_mode: int = _lib.RENDER_DEFAULT,
           background=(0.0, 0.0, 0.0), raster_pass: int = _lib.PASS_BACKWARD) -> RenderOutput:
    """Render splats to an image with the B200 pipeline. ``img_size`` is (w, h)."""
    w, h = int(img_size[0]), int(img_size[1])
    if w <= 0 or h <= 0:
        raise ValueError("Can't render images with 0 size.")
    _check_splats(transforms, sh_coeffs, raw_opacities)
    transforms = transforms.contiguous()
    sh_coeffs = sh_coeffs.contiguous()
    raw_opacities = raw_opacities.contiguous()
    dev = transforms.device.index
    ctx = context(dev)
    out = _lib.RenderOut()
    cam = camera.to_c()
    bg = (C.c_float * 3)(*[float(v) for v in background])
    n, coeffs = transforms.shape[0], sh_coeffs.shape[1]
    ctx.check(_lib.lib().bsx_render_fwd(ctx.handle, C.byref(cam), w, h, ptr(transforms), ptr(sh_coeffs),
                                        ptr(raw_opacities), n, coeffs, int(render_mode), int(raster_pass), bg,
                                        C.byref(out)))
    ctx.last_n = n
    # rasterize_bwd / project_bwd read these device buffers later (the forward
    # state of the context): keep them alive until the next render
    ctx.fwd_inputs = (transforms, sh_coeffs, raw_opacities)
    V, M = out.num_visible, out.num_intersections
    bwd = raster_pass != _lib.PASS_FORWARD
    f32, i32 = torch.float32, torch.int32
    img = (device_view(out.d_image, (h, w, 4), f32, dev) if bwd
           else device_view(out.d_image_packed, (h, w), i32, dev))
    aux = RenderAux(
        num_visible=V,
        num_intersections=M,
        visible=device_view(out.d_visible, (n,), f32, dev) if bwd else torch.empty(0, device=transforms.device),
        max_radius=device_view(out.d_max_radius, (n,), f32, dev),
        tile_offsets=device_view(out.d_tile_offsets, (out.tile_bh, out.tile_bw, 2), i32, dev),
        img_size=(w, h),
    )
    return RenderOutput(
        out_img=img,
        aux=aux,
        projected_splats=device_view(out.d_projected, (n, _lib.BSX_PROJECTED_LANES), f32, dev),
        compact_gid_from_isect=device_view(out.d_isect_gid, (M,), i32, dev),
        isect_tile=device_view(out.d_isect_tile, (M,), i32, dev),
        depth_order=device_view(out.d_depth_order, (V,), i32, dev),
        tile_counts=device_view(out.d_tile_counts, (n,), i32, dev),
        cum_counts=device_view(out.d_cum_counts, (V,), i32, dev),
        project_uniforms=out.uniforms,
        num_splats=n,
    )


def render_splats(splats, camera: Camera, img_size: tuple, background=(0.0, 0.0, 0.0), packed: bool = False):
    """``brush_render::render_splats`` (gaussian_splats.rs:418-437): image + aux."""
    out = render(camera, img_size, splats.transforms, splats.sh_coeffs, splats.raw_opacities,
                 splats.render_mode, background, _lib.PASS_FORWARD if packed else _lib.PASS_BACKWARD)
    return out.out_img, out.aux

"""Backward ops, mirroring ``SplatBwdOps`` (crates/brush-render-bwd/src/burn_glue.rs:80-172).

Both consume the state the library keeps from the last backward-pass
``render`` on the same device (the reference keeps the same state in its
autodiff node, ``GaussianBackwardState``, burn_glue.rs:264-284).
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import torch

from . import _lib
from ._context import context, ptr


@dataclass
class SplatGrads:
    v_transforms: torch.Tensor  # [N,10]
    v_coeffs: torch.Tensor      # [N,C,3]
    v_raw_opac: torch.Tensor    # [N]
    v_refine_weight: torch.Tensor  # [N]


def rasterize_bwd(v_output: torch.Tensor, compute_refine_weight: bool = True,
                  v_combined: torch.Tensor | None = None) -> torch.Tensor:
    """``v_output`` [H,W,4] -> ``v_combined`` [N, 12] (11 reference lanes + pad)."""
    dev = v_output.device.index
    ctx = context(dev)
    n = ctx.last_n
    if v_combined is None:
        v_combined = torch.empty((max(n, 1), _lib.BSX_GRAD_STRIDE), device=v_output.device, dtype=torch.float32)
    v_output = v_output.contiguous()  # held until the call returns: the kernel reads it asynchronously
    ctx.check(_lib.lib().bsx_rasterize_bwd(ctx.handle, ptr(v_output), int(compute_refine_weight),
                                           ptr(v_combined)))
    return v_combined


def project_bwd(v_combined: torch.Tensor, num_splats: int, sh_coeffs_per_splat: int,
                out: SplatGrads | None = None) -> SplatGrads:
    """``v_combined`` -> dense gradients for every splat (zeros where invisible)."""
    dev = v_combined.device.index
    ctx = context(dev)
    if out is None:
        d = v_combined.device
        out = SplatGrads(
            v_transforms=torch.empty((num_splats, 10), device=d),
            v_coeffs=torch.empty((num_splats, sh_coeffs_per_splat, 3), device=d),
            v_raw_opac=torch.empty((num_splats,), device=d),
            v_refine_weight=torch.empty((num_splats,), device=d),
        )
    ctx.check(_lib.lib().bsx_project_bwd(ctx.handle, ptr(v_combined), ptr(out.v_transforms), ptr(out.v_coeffs),
                                         ptr(out.v_raw_opac), ptr(out.v_refine_weight)))
    return out


def rasterize_bwd_ref(out_img: torch.Tensor, projected_splats: torch.Tensor, compact_gid_from_isect: torch.Tensor,
                      tile_offsets: torch.Tensor, background, img_size: tuple, v_output: torch.Tensor,
                      smooth_cutoff: bool = False, render_depth: bool = False,
                      compute_refine_weight: bool = True) -> torch.Tensor:
    """``SplatBwdOps::rasterize_bwd`` / ``rasterize_bwd_with_refine_weight`` with the reference's
    compact layouts (burn_glue.rs:84-121), stateless: ``projected_splats`` [V,10] by compact id,
    ``compact_gid_from_isect`` [M] compact ids, ``tile_offsets`` [ty,tx,2] -> ``v_combined`` [V,11]."""
    dev = out_img.device.index
    ctx = context(dev)
    v = int(projected_splats.shape[0])
    if projected_splats.dim() != 2 or projected_splats.shape[1] != 10:
        raise ValueError("projected_splats must be [V,10]")
    w, h = int(img_size[0]), int(img_size[1])
    v_combined = torch.empty((v, _lib.BSX_COMPACT_GRAD_LANES), device=out_img.device, dtype=torch.float32)
    bg = (C.c_float * 3)(*[float(x) for x in background])
    # contiguous copies are held in locals until the call returns: freed earlier, the
    # allocator could hand one's memory to the next before the kernels read it
    ids = compact_gid_from_isect.contiguous()
    img, rows, off, vout = (x.contiguous() for x in (out_img, projected_splats, tile_offsets, v_output))
    ctx.check(_lib.lib().bsx_rasterize_bwd_ref(ctx.handle, ptr(img), ptr(rows),
                                               v, ptr(ids), int(ids.numel()), ptr(off), bg, w, h,
                                               ptr(vout), int(smooth_cutoff),
                                               int(compute_refine_weight), int(render_depth), ptr(v_combined)))
    return v_combined


def project_bwd_ref(transforms: torch.Tensor, sh_coeffs: torch.Tensor, raw_opac: torch.Tensor,
                    global_from_compact_gid: torch.Tensor, project_uniforms, render_mode: int,
                    v_combined: torch.Tensor) -> SplatGrads:
    """``SplatBwdOps::project_bwd`` with the reference's compact ``v_combined`` [V,11] and
    ``global_from_compact_gid`` [V] (burn_glue.rs:127-141), stateless; dense gradients for all N splats."""
    dev = transforms.device.index
    ctx = context(dev)
    n, c = int(transforms.shape[0]), int(sh_coeffs.shape[1])
    v = int(global_from_compact_gid.numel())
    if v_combined.shape != (v, _lib.BSX_COMPACT_GRAD_LANES):
        raise ValueError("v_combined must be [V,11] with V = len(global_from_compact_gid)")
    d = transforms.device
    out = SplatGrads(torch.empty((n, 10), device=d), torch.empty((n, c, 3), device=d), torch.empty((n,), device=d),
                     torch.empty((n,), device=d))
    t, sh, op, gid, vc = (x.contiguous() for x in (transforms, sh_coeffs, raw_opac, global_from_compact_gid,
                                                   v_combined))
    ctx.check(_lib.lib().bsx_project_bwd_ref(ctx.handle, ptr(t), ptr(sh),
                                             ptr(op), n, c, ptr(gid),
                                             v, C.byref(project_uniforms), int(render_mode),
                                             ptr(vc), ptr(out.v_transforms), ptr(out.v_coeffs),
                                             ptr(out.v_raw_opac), ptr(out.v_refine_weight)))
    return out

"""Backward ops, mirroring ``SplatBwdOps`` (crates/brush-render-bwd/src/burn_glue.rs:80-172).

Both consume the state the library keeps from the last backward-pass
``render`` on the same device (the reference keeps the same state in its
autodiff node, ``GaussianBackwardState``, burn_glue.rs:264-284).
"""
from __future__ import annotations

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
    ctx.check(_lib.lib().bsx_rasterize_bwd(ctx.handle, ptr(v_output.contiguous()), int(compute_refine_weight),
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

"""Image loss, mirroring ``LossOps`` / ``image_loss`` (crates/brush-loss/src/lib.rs:935-970,1629-1679).

Per pixel and colour channel: ``l1_weight*|x - y| + ssim_weight*SSIM(x, y)``
with an 11x11 Gaussian window (sigma 1.5), y the packed RGBA8 ground truth
(optionally composited over ``bg`` and masked by its alpha). A fourth
channel, when given, is alpha matching ``|x.a - y.a|``.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import torch

from . import _lib
from ._context import context, ptr


@dataclass
class ImageLossConfig:
    l1_weight: float = 0.8
    ssim_weight: float = -0.2
    composite_bg: tuple | None = None
    mask: bool = False

    def to_c(self) -> _lib.LossCfg:
        c = _lib.LossCfg()
        c.l1_weight = float(self.l1_weight)
        c.ssim_weight = float(self.ssim_weight)
        c.composite_bg = int(self.composite_bg is not None)
        c.bg[:] = [float(v) for v in (self.composite_bg or (0.0, 0.0, 0.0))]
        c.mask = int(self.mask)
        return c


def _gt_check(gt_packed: torch.Tensor, h: int, w: int) -> torch.Tensor:
    if gt_packed.shape != (h, w) or gt_packed.dtype not in (torch.int32, torch.uint32):
        raise ValueError("gt_packed must be [H,W] packed RGBA8 (int32/uint32)")
    return gt_packed.contiguous()


def image_loss_forward(pred_chw: torch.Tensor, gt_packed: torch.Tensor, cfg: ImageLossConfig) -> torch.Tensor:
    """Loss map [C,H,W] from ``pred`` [C,H,W] (reference layout)."""
    c, h, w = pred_chw.shape
    gt = _gt_check(gt_packed, h, w)
    ctx = context(pred_chw.device.index)
    out = torch.empty_like(pred_chw)
    cfgc = cfg.to_c()
    pred = pred_chw.contiguous()  # held until the call returns
    ctx.check(_lib.lib().bsx_loss_fwd(ctx.handle, ptr(pred), ptr(gt), w, h, c, C.byref(cfgc), ptr(out)))
    return out


def image_loss_backward(pred_chw: torch.Tensor, gt_packed: torch.Tensor, dl_dmap: torch.Tensor,
                        cfg: ImageLossConfig) -> torch.Tensor:
    """d loss / d pred [C,H,W] for an arbitrary upstream ``dl_dmap`` [C,H,W]."""
    c, h, w = pred_chw.shape
    gt = _gt_check(gt_packed, h, w)
    ctx = context(pred_chw.device.index)
    out = torch.empty_like(pred_chw)
    cfgc = cfg.to_c()
    # both held until the call returns: a temporary freed early could share memory with the other
    pred, dl = pred_chw.contiguous(), dl_dmap.contiguous()
    ctx.check(_lib.lib().bsx_loss_bwd(ctx.handle, ptr(pred), ptr(gt), w, h, c, C.byref(cfgc), ptr(dl), ptr(out)))
    return out


def image_loss_fused(image_hwc4: torch.Tensor, gt_packed: torch.Tensor, cfg: ImageLossConfig,
                     loss_out: torch.Tensor | None = None, v_output: torch.Tensor | None = None):
    """Training form: mean loss over RGB (device scalar) and its gradient in [H,W,4] layout."""
    h, w, _ = image_hwc4.shape
    gt = _gt_check(gt_packed, h, w)
    ctx = context(image_hwc4.device.index)
    if loss_out is None:
        loss_out = torch.empty((1,), device=image_hwc4.device)
    if v_output is None:
        v_output = torch.empty_like(image_hwc4)
    cfgc = cfg.to_c()
    ctx.check(_lib.lib().bsx_loss_fused(ctx.handle, ptr(image_hwc4), ptr(gt), w, h, C.byref(cfgc), ptr(loss_out),
                                        ptr(v_output)))
    return loss_out, v_output

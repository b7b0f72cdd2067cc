"""AdamScaled, mirroring ``brush_train::adam_scaled`` (crates/brush-train/src/adam_scaled.rs:216-383).

One fused launch updates every parameter group. A group is a 2-D view
``[rows, cols]`` of a parameter with optional per-column learning-rate scale
and optional per-row second moment (``reduce_moment_2``, used for SH rows).
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field

import torch

from . import _lib
from ._context import context, ptr


@dataclass
class AdamGroup:
    param: torch.Tensor          # [rows, cols] view, contiguous
    grad: torch.Tensor           # same shape
    lr: float
    col_scale: list | None = None
    reduce_moment_2: bool = False
    m: torch.Tensor | None = None
    v: torch.Tensor | None = None

    def ensure_state(self) -> None:
        if self.m is None:
            self.m = torch.zeros_like(self.param)
        if self.v is None:
            shape = (self.param.shape[0],) if self.reduce_moment_2 else tuple(self.param.shape)
            self.v = torch.zeros(shape, device=self.param.device, dtype=torch.float32)


@dataclass
class AdamScaled:
    beta_1: float = 0.9
    beta_2: float = 0.999
    epsilon: float = 1e-15
    step_count: int = 0
    _scales: list = field(default_factory=list)

    def step(self, groups: list[AdamGroup], grad_scale: float = 1.0) -> None:
        if not groups:
            return
        ctx = context(groups[0].param.device.index)
        self.step_count += 1
        arr = (_lib.AdamGroup * len(groups))()
        self._scales = []
        for i, g in enumerate(groups):
            g.ensure_state()
            rows, cols = g.param.shape
            if g.grad.shape != g.param.shape:
                raise ValueError("gradient shape must match the parameter")
            arr[i].d_param = ptr(g.param).value
            arr[i].d_grad = ptr(g.grad).value
            arr[i].d_m = ptr(g.m).value
            arr[i].d_v = ptr(g.v).value
            arr[i].rows = rows
            arr[i].cols = cols
            arr[i].lr = float(g.lr)
            if g.col_scale is not None:
                sc = (C.c_float * cols)(*[float(s) for s in g.col_scale])
                self._scales.append(sc)
                arr[i].h_col_scale = C.cast(sc, C.POINTER(C.c_float))
            else:
                arr[i].h_col_scale = None
            arr[i].reduce_moment_2 = int(g.reduce_moment_2)
        cfg = _lib.AdamCfg(beta_1=self.beta_1, beta_2=self.beta_2, epsilon=self.epsilon, step=self.step_count,
                           grad_scale=float(grad_scale))
        ctx.check(_lib.lib().bsx_adam_step(ctx.handle, arr, len(groups), C.byref(cfg)))

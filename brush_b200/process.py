"""The training-loop driver: ``train_stream`` restates the iteration loop of
crates/brush-process/src/train_stream.rs:355-590 (LOD phase 0; the LOD
decimation, DiG features, appearance models and rerun logging are outside this
library) over the native trainer, with ``eval_stats`` (crates/brush-train/src/
eval.rs:22-75) and PLY checkpoints named as ``export_checkpoint``
(train_stream.rs:931-951). It yields the reference's ``TrainMessage`` kinds.

Views are (Camera, (w, h), packed ground truth [H, W] int32) triples; the ground
truth may live on the host (it is uploaded per step) or on the device.
"""
from __future__ import annotations

import math
import os
import time
from dataclasses import dataclass, field
from typing import Iterator, Optional, Sequence

import numpy as np
import torch

from .loss import ImageLossConfig, image_loss_forward
from .ply import splat_to_ply
from .render import render
from .splats import Splats
from .train import RefineConfig, SplatTrainer, TrainConfig


@dataclass
class ProcessConfig:
    """ProcessConfig subset (crates/brush-process/src/config.rs:10-56)."""
    seed: int = 42
    start_iter: int = 0
    eval_every: int = 1000
    export_every: int = 5000
    export_path: Optional[str] = None  # None: no files are written
    export_name: str = "export_{iter}.ply"


@dataclass
class TrainStep:
    iter: int
    total_elapsed: float  # seconds of training (steps and refines)
    loss: float


@dataclass
class RefineStep:
    cur_splat_count: int
    iter: int


@dataclass
class EvalResult:
    iter: int
    avg_psnr: float
    avg_ssim: float


@dataclass
class Exported:
    iter: int
    path: str


@dataclass
class DoneTraining:
    splats: Splats


class SceneLoader:
    """Seeded epoch shuffles of the training views (the role of brush-dataset's loader)."""

    def __init__(self, n: int, seed: int):
        self.n = n
        self.rng = np.random.default_rng(seed)
        self.order: list[int] = []

    def next_index(self) -> int:
        if not self.order:
            self.order = list(self.rng.permutation(self.n))
        return int(self.order.pop())


def eval_stats(splats: Splats, camera, img_size, gt_packed: torch.Tensor) -> tuple[float, float]:
    """(PSNR, SSIM) of one view as eval.rs:22-75: render on black, 8-bit round trip,
    MSE = mean of the squared L1 map, PSNR = 10 ln(1/MSE) / ln 10, SSIM = mean SSIM map."""
    out = render(camera, img_size, splats.transforms, splats.sh_coeffs, splats.raw_opacities)
    rgb = out.out_img[..., :3]
    rgb = torch.round(rgb * 255.0) / 255.0
    chw = rgb.permute(2, 0, 1).contiguous()
    gt = gt_packed.to(chw.device)
    l1 = image_loss_forward(chw, gt, ImageLossConfig(l1_weight=1.0, ssim_weight=0.0))
    mse = (l1 * l1).mean()
    psnr = torch.log(1.0 / mse) * 10.0 / math.log(10.0)
    ssim = image_loss_forward(chw, gt, ImageLossConfig(l1_weight=0.0, ssim_weight=1.0)).mean()
    return float(psnr), float(ssim)


def _export_name(name: str, it: int, total: int) -> str:
    digits = int(math.floor(math.log10(max(total, 1)))) + 1
    return name.replace("{iter}", f"{it:0{digits}d}")


def train_stream(splats: Splats, views: Sequence, config: TrainConfig, refine: Optional[RefineConfig] = None,
                 process: Optional[ProcessConfig] = None, eval_views: Sequence = (),
                 up_axis=None) -> Iterator[object]:
    """Runs ``config.total_train_iters`` steps; yields TrainStep after every step,
    RefineStep after every densification, EvalResult / Exported on their cadence and
    DoneTraining last. ``splats`` is trained in place (its tensors are rebound on refine)."""
    process = process or ProcessConfig()
    trainer = SplatTrainer(config, splats)
    loader = SceneLoader(len(views), process.seed)
    total = config.total_train_iters
    dev = splats.transforms.device
    elapsed = 0.0
    try:
        for it in range(process.start_iter, total):
            t0 = time.perf_counter()
            cam, size, gt = views[loader.next_index()]
            # the refine weight only feeds high-gradient growth, which stops at
            # growth_stop_iter (refinement_weight_needed, train.rs:428-430; train_stream.rs:458)
            need_weight = refine is not None and it < refine.growth_stop_iter
            st = trainer.step(cam, size, gt.to(dev, non_blocking=True), splats, compute_refine_weight=need_weight)
            # refine gate on the phase iteration just completed (train_stream.rs:475-498)
            if refine is not None and refine.due(it, total):
                rs = trainer.refine(splats, it, it, total, refine)
                yield RefineStep(cur_splat_count=rs.total_splats, iter=it)
            it1 = it + 1
            loss = float(st.loss)
            elapsed += time.perf_counter() - t0
            yield TrainStep(iter=it1, total_elapsed=elapsed, loss=loss)
            if eval_views and (it1 % process.eval_every == 0 or it1 == total):
                scores = [eval_stats(splats, c, s, g) for c, s, g in eval_views]
                yield EvalResult(iter=it1, avg_psnr=float(np.mean([p for p, _ in scores])),
                                 avg_ssim=float(np.mean([q for _, q in scores])))
            if process.export_path is not None and (it1 % process.export_every == 0 or it1 == total):
                os.makedirs(process.export_path, exist_ok=True)
                path = os.path.join(process.export_path, _export_name(process.export_name, it1, total))
                with open(path, "wb") as fh:
                    fh.write(splat_to_ply(splats, up_axis))
                yield Exported(iter=it1, path=path)
    finally:
        trainer.close()
    yield DoneTraining(splats=splats)

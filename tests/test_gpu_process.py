"""The training-loop driver (brush_b200.process.train_stream, after
crates/brush-process/src/train_stream.rs:355-590): message sequence, refine cadence,
eval statistics (crates/brush-train/src/eval.rs:22-75) and PLY checkpoints."""
import math
import os

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _views(src, n, w, h):
    from brush_b200.render import render_splats
    from brush_b200.splats import orbit_camera

    views = []
    for i in range(n):
        cam = orbit_camera(i, n, 8.0, w, h)
        gt = render_splats(src, cam, (w, h), packed=True)[0].clone().cpu()
        views.append((cam, (w, h), gt))
    return views


def test_train_stream_messages_eval_and_export(cuda, tmp_path):
    import brush_b200 as bsx
    from brush_b200.ply import load_splat_from_ply
    from brush_b200.process import (DoneTraining, EvalResult, Exported, ProcessConfig, RefineStep, TrainStep,
                                    eval_stats, train_stream)
    from brush_b200.splats import clustered_scene, perturbed

    splats = clustered_scene(20000, 1, "cuda", seed=31, log_scale_mean=-3.5)
    views = _views(perturbed(splats, 5, mean_std=0.05, dc_std=0.2), 6, 192, 128)
    total = 300
    proc = ProcessConfig(eval_every=100, export_every=150, export_path=str(tmp_path), seed=3)
    msgs = list(train_stream(splats, views, bsx.TrainConfig(total_train_iters=total),
                             bsx.RefineConfig(refine_every=100, growth_grad_threshold=1e-5), proc,
                             eval_views=views[:2]))
    steps = [m for m in msgs if isinstance(m, TrainStep)]
    assert [m.iter for m in steps] == list(range(1, total + 1))
    assert all(math.isfinite(m.loss) for m in steps)
    refines = [m for m in msgs if isinstance(m, RefineStep)]
    assert [m.iter for m in refines] == [100, 200]  # phase progress <= 0.95 gates 300
    evals = [m for m in msgs if isinstance(m, EvalResult)]
    assert [m.iter for m in evals] == [100, 200, 300]
    exports = [m for m in msgs if isinstance(m, Exported)]
    assert [os.path.basename(m.path) for m in exports] == ["export_150.ply", "export_300.ply"]
    assert isinstance(msgs[-1], DoneTraining)
    # training on these targets improves the fit
    assert evals[-1].avg_psnr > evals[0].avg_psnr
    # the checkpoint is the trained splats
    back = load_splat_from_ply(exports[-1].path).splats
    assert back.num_splats == splats.num_splats == refines[-1].cur_splat_count
    assert torch.equal(back.sh_coeffs, splats.sh_coeffs)
    p, s = eval_stats(back, *views[0])
    assert abs(p - eval_stats(splats, *views[0])[0]) < 1e-3 and 0.0 < s <= 1.0


def test_eval_stats_identical_render_is_perfect(cuda):
    """A target rendered from the same splats (8-bit) scores SSIM ~ 1 and a high PSNR."""
    from brush_b200.process import eval_stats
    from brush_b200.splats import config1_scene
    from brush_b200.render import render_splats

    splats, cam, size, _ = config1_scene("cuda", seed=4)
    gt = render_splats(splats, cam, size, packed=True)[0].clone()
    psnr, ssim = eval_stats(splats, cam, size, gt)
    assert ssim > 0.99 and psnr > 40.0

"""Host logic of the training-loop driver on CPU, with a stand-in trainer (no GPU).

``train_stream`` restates crates/brush-process/src/train_stream.rs:355-590: the
refine gate on the phase iteration just completed (phase_iter > 0, a multiple of
refine_every, f32 progress <= 0.95; :466-482), the message order (refine, then
the step's TrainStep with the post-increment iteration; :499-513), and the
checkpoint name padded to the digits of the step count (export_checkpoint,
:931-951). The GPU test of the same driver runs the real trainer.
"""
import math
from types import SimpleNamespace

import numpy as np
import pytest
import torch

from brush_b200 import process as proc
from brush_b200.train import RefineConfig, TrainConfig


class _FakeTrainer:
    instances = []

    def __init__(self, config, splats):
        self.steps, self.refines, self.closed = [], [], False
        self.weight_flags = []
        self.n = 1000
        _FakeTrainer.instances.append(self)

    def step(self, cam, size, gt, splats, compute_refine_weight=True):
        self.steps.append(cam)
        self.weight_flags.append(compute_refine_weight)
        return SimpleNamespace(loss=torch.tensor(1.0 / (len(self.steps) + 1)), num_visible=0, num_intersections=0)

    def refine(self, splats, it, phase_iter, phase_total, cfg):
        self.refines.append((it, phase_iter, phase_total))
        self.n += 10
        return SimpleNamespace(total_splats=self.n)

    def close(self):
        self.closed = True


@pytest.fixture
def fake_trainer(monkeypatch):
    _FakeTrainer.instances.clear()
    monkeypatch.setattr(proc, "SplatTrainer", _FakeTrainer)
    return _FakeTrainer


def _views(n):
    return [(i, (8, 8), torch.zeros((8, 8), dtype=torch.int32)) for i in range(n)]


def _splats():
    return SimpleNamespace(transforms=torch.zeros((4, 10)))


def test_message_order_and_refine_cadence(fake_trainer):
    total = 1000
    cfg = TrainConfig(total_train_iters=total)
    rcfg = RefineConfig(refine_every=100)
    msgs = list(proc.train_stream(_splats(), _views(7), cfg, rcfg))
    tr = fake_trainer.instances[0]
    assert tr.closed
    assert isinstance(msgs[-1], proc.DoneTraining)
    steps = [m for m in msgs if isinstance(m, proc.TrainStep)]
    assert [m.iter for m in steps] == list(range(1, total + 1))
    # refines after phase iterations 100..900: the multiples of 100 whose progress is at most 0.95
    expect = [it for it in range(1, total) if it % 100 == 0 and np.float32(it) / np.float32(total) <= 0.95]
    assert [r[0] for r in tr.refines] == expect == list(range(100, 1000, 100))
    assert all(r == (it, it, total) for r, it in zip(tr.refines, expect))
    # each RefineStep comes right before the TrainStep of the same step (post-increment iter)
    for i, m in enumerate(msgs):
        if isinstance(m, proc.RefineStep):
            assert isinstance(msgs[i + 1], proc.TrainStep) and msgs[i + 1].iter == m.iter + 1
    counts = [m.cur_splat_count for m in msgs if isinstance(m, proc.RefineStep)]
    assert counts == [1000 + 10 * (k + 1) for k in range(len(expect))]


def test_refine_gate_progress_limit():
    """progress = phase_iter / phase_total in f32, clamped to [0, 1], refines only while <= 0.95."""
    r = RefineConfig(refine_every=50)
    assert not r.due(0, 1000)
    assert r.due(50, 1000) and r.due(950, 1000)
    assert not r.due(1000, 1000) and not r.due(975, 1000)
    assert not r.due(49, 1000)
    assert r.due(50, 0) is False  # phase_total 0: progress clamps to 1


def test_scene_loader_epochs_cover_every_view():
    ld = proc.SceneLoader(13, seed=5)
    seen = [ld.next_index() for _ in range(13 * 3)]
    for e in range(3):
        assert sorted(seen[13 * e: 13 * (e + 1)]) == list(range(13))
    ld2 = proc.SceneLoader(13, seed=5)
    assert [ld2.next_index() for _ in range(13 * 3)] == seen


def test_every_view_is_trained_once_per_epoch(fake_trainer):
    views = _views(5)
    list(proc.train_stream(_splats(), views, TrainConfig(total_train_iters=15)))
    cams = fake_trainer.instances[0].steps
    for e in range(3):
        assert sorted(cams[5 * e: 5 * (e + 1)]) == list(range(5))


@pytest.mark.parametrize("total,it,name", [(1000, 100, "export_0100.ply"), (999, 7, "export_007.ply"),
                                           (30000, 5000, "export_05000.ply"), (1, 1, "export_1.ply"),
                                           (10, 10, "export_10.ply")])
def test_export_name_digits(total, it, name):
    assert proc._export_name("export_{iter}.ply", it, total) == name
    assert int(math.floor(math.log10(total))) + 1 == len(name) - len("export_.ply")


def test_trainer_closed_when_the_stream_is_abandoned(fake_trainer):
    gen = proc.train_stream(_splats(), _views(3), TrainConfig(total_train_iters=100))
    for _ in range(5):
        next(gen)
    gen.close()
    assert fake_trainer.instances[0].closed


def test_start_iter_resumes_the_count(fake_trainer):
    msgs = list(proc.train_stream(_splats(), _views(3), TrainConfig(total_train_iters=20),
                                  process=proc.ProcessConfig(start_iter=15)))
    assert [m.iter for m in msgs if isinstance(m, proc.TrainStep)] == [16, 17, 18, 19, 20]


def test_refine_weight_only_until_growth_stops(fake_trainer):
    """compute_refine_weight = iter < growth_stop_iter (refinement_weight_needed, train.rs:428-430),
    and never without densification."""
    cfg = TrainConfig(total_train_iters=40)
    list(proc.train_stream(_splats(), _views(3), cfg, RefineConfig(refine_every=10, growth_stop_iter=25)))
    flags = fake_trainer.instances[0].weight_flags
    assert flags == [it < 25 for it in range(40)]
    list(proc.train_stream(_splats(), _views(3), cfg))
    assert fake_trainer.instances[1].weight_flags == [False] * 40

#!/usr/bin/env python3
"""Benchmark: Brush's differentiable Gaussian-splat training step on B200.

Default workload (the headline metric): 1,000,000 splats,
SH degree 3, 1920x1080, seeded synthetic scene (64 isotropic clusters, sigma
0.3, inside a radius-5 ball; log-scales N(-4.5,0.7); opacity logits
N(0,1.5)), 16 cameras on a radius-8 orbit, uniform random targets. One step =
render forward (backward-pass bookkeeping) -> 0.8 L1 + 0.2 (1-SSIM) loss and
gradient -> raster backward -> projection backward -> [N>1: the peer-memory
gradient exchange fused with Adam] -> fused Adam with the reference's
learning-rate table -> refine statistics, one bsx_train_step call.
``--workload`` selects the other BASELINE configurations (cfg1, cfg3 and the
render-only cfg5) as additional measurements.

With N GPUs (one process per GPU, torchrun) every rank trains on its own view
against replicated splats each step (weak scaling); value = views/s over all
ranks. Splat parameters (236 MB) plus per-step buffers exceed the 126 MB L2,
so no explicit flush is done between steps.

``--impl reference`` times the CPU restatement of the reference's algorithm
(the reference itself is Rust/wgpu and cannot be built or run on this box).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "train steps/s @1M splats SH3 1080p; fwd+bwd ms; % HBM roofline"
WORKLOAD = "cfg2: 1M splats SH3 1920x1080 full train step (fwd+SSIM/L1+bwd+Adam)"


def _peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d.get("hbm_gbs", 6650.0)), "measured"
    return 6650.0, "fallback"


class ClockSampler:
    """Samples nvidia-smi clocks / throttle reasons every 20 ms; keeps the samples that fall
    inside the timed region (host monotonic clock, bracketed by device synchronisation)."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []
        self.region = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "20"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except (FileNotFoundError, OSError):
            self.proc = None
            return
        deadline = time.monotonic() + 5.0  # nvidia-smi is sampling before the timed region starts
        while not self.lines and time.monotonic() < deadline and self.proc.poll() is None:
            time.sleep(0.01)

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append((time.monotonic(), line.strip()))

    def mark(self, t0: float, t1: float) -> None:
        self.region = (t0, t1)

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.05)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        t0, t1 = self.region if self.region else (float("-inf"), float("inf"))
        inside = [ln for ts, ln in self.lines if t0 <= ts <= t1]
        chosen = inside
        if not chosen and self.lines:  # region shorter than one sample: the nearest sample
            chosen = [min(self.lines, key=lambda x: abs(x[0] - 0.5 * (t0 + t1)))[1]]
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in chosen:
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
            except ValueError:
                continue
            for nm, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm), "samples_in_region": len(inside)}


# Algorithmic bytes moved by each kernel per launch (fp32 = 4 B). N splats,
# V visible, M intersections, Mp intersections surviving the forward early-out,
# P pixels, T tiles, C SH coefficients per splat.
def kernel_bytes(name, N, V, M, Mp, P, T, C, W=1, fused_adam=False):
    row = 4 * (11 + 3 * C)  # bytes of one splat's parameters (or gradients)
    if name == "project_bwd_kernel" and fused_adam:
        # single-GPU step: projection backward + AdamScaled in one kernel. Per splat:
        # v_combined 48 + refine 4 + parameters read and written 2 (44 + 12C) +
        # first moment read and written 2 (44 + 12C) + second moments 2 * 48
        return (324 + 48 * C) * N
    table = {
        "project_fwd_kernel": 44 * N + 8 * N + N // 8 + V * (12 * C + 48 + 4),
        "compact_visible_kernel": 4 * N + N // 8 + 12 * V,
        "sort_hist_kernel": 4 * V,  # depth sort; the tile sort adds 4 M (below)
        "sort_pass_kernel": 16 * V,
        "scan_kernel": 12 * V,
        "emit_kernel": V * (4 + 48 + 8) + 8 * M,
        "tile_offsets_kernel": 8 * M + 8 * T,
        "tile_order_kernel": 16 * T + 4 * T,  # ranges read twice, order written
        # + Mp: the training pass stores each staged intersection's band mask (1 B),
        # which the backward reads
        "raster_fwd_kernel": 52 * Mp + 16 * P + 8 * T + 4 * V + Mp,
        # SSIM pass: image + ground truth in, nine partial planes out; gradient pass:
        # the planes, image and ground truth in, the gradient image out
        "loss_ssim_kernel": 20 * P + 36 * P,
        "loss_grad_kernel": 36 * P + 20 * P + 16 * P,
        "loss_l1_fused_kernel": 36 * P,
        "loss_mean_kernel": 0,
        "raster_bwd_kernel": 32 * P + 52 * Mp + 48 * V + Mp,
        "project_bwd_kernel": 48 * N + V * (44 + 12 * C) + N * (48 + 12 * C),
        "adam_kernel": (316 + 60 * C) * N,
        "gather_stats_kernel": 36 * N,
        # NVLink bytes per rank: peer gradient rows in + parameter rows out
        "dp_adam_kernel": 2 * (W - 1) * (N // W) * row if W > 1 else 0,
    }
    return table.get(name, 0)


# ---- workloads (synthetic, seeded) -------------------------
WORKLOADS = {
    "cfg1": "cfg1: 16,384 splats SH0 256x256 full train step (fwd+SSIM/L1+bwd+Adam lr 1e-3)",
    "cfg2": WORKLOAD,
    "cfg3": "cfg3: 3M splats SH3 1297x840, 200 hemisphere views, full train step (fwd+SSIM/L1+bwd+Adam)",
    "cfg4": ("cfg4: densification run from 100k splats SH3 1280x720, 100 hemisphere views, refine every 100 "
             "steps with the 3DGS rule (average view-space gradient >= 2e-4: clone small / split large, prune "
             "opacity < 0.005, cap 1.5M)"),
    "cfg5": "cfg5: 6M splats SH3 3840x2160 render-only forward (viewer path, packed RGBA8), 120-frame circle",
    "ply": "ply: 1M splats SH3 (cfg2 scene) as a binary little-endian 3DGS PLY in pinned host memory -> device "
           "splats (import), and back (export)",
}


def build_workload(name, dev, world):
    """(splats, cameras, (w, h), host targets, TrainConfig or None for render-only)."""
    import torch

    import brush_b200 as bsx
    from brush_b200 import splats as S

    if name == "cfg1":
        splats, cam, size, gt = S.config1_scene(dev, seed=1)
        # the configuration's step is render, loss, backward and one Adam step: no mean noise
        return splats, [cam], size, [gt.cpu()], bsx.TrainConfig(uniform_lr=1e-3, mean_noise=False)
    if name == "cfg2":
        splats, _, size, _ = S.config2_scene(dev, seed=2)
        w, h = size
        cams = [S.orbit_camera(i, 16, 8.0, w, h) for i in range(16)]
        return splats, cams, size, [S.random_gt(h, w, 1000 + i, "cpu") for i in range(16)], bsx.TrainConfig()
    if name == "cfg3":
        splats, cams, size, gts = S.config3_scene(dev, seed=3)
        return splats, cams, size, [g.cpu() for g in gts], bsx.TrainConfig()
    if name == "cfg4":
        splats = S.clustered_scene(100_000, 3, dev, seed=4)
        w, h = 1280, 720
        cams = S.hemisphere_cameras(100, 8.0, w, h, seed=4)
        return splats, cams, (w, h), [S.random_gt(h, w, 4000 + i, "cpu") for i in range(100)], \
            bsx.TrainConfig(total_train_iters=3000, accumulate_grad2d=True)
    if name == "cfg5":
        splats, size = S.config5_scene(dev, seed=5)
        cams = S.circle_cameras(120, 8.0, size[0], size[1])
        return splats, cams, size, None, None
    raise ValueError(name)


def _exchange_label(args, world, train, trainer):
    if world == 1 or not train:
        return None
    if args.exchange == "nccl":
        return "NCCL reduce-scatter + sharded Adam + all-gather"
    if trainer is not None and trainer.peer is not None and trainer.peer.mc_base:
        return "NVLink multicast fused kernel: in-switch gradient sum + Adam + multicast parameter store"
    return "peer-memory fused reduce+Adam+broadcast kernel (gradient rows pushed by the projection backward)"


def _time_region(args, world, body):
    """Barrier + sync, CUDA events around body(), sync + barrier; returns the max over ranks (ms)."""
    import torch

    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    body()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    if world > 1:
        torch.distributed.barrier()
        t = torch.tensor([ms], device="cuda")
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms = float(t.item())
    return ms


def run_ours(args, rank, world, local_rank):
    import torch

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    import brush_b200 as bsx
    from brush_b200._context import context
    from brush_b200.render import render

    pg = torch.distributed.group.WORLD if world > 1 else None
    splats, cams, size, gts_cpu, tcfg = build_workload(args.workload, dev, world)
    w, h = size
    ncam = len(cams)
    train = tcfg is not None
    ctx = context(dev)
    refine_cfg = None
    if args.workload == "cfg4":
        if world > 1:
            raise SystemExit("cfg4 (densification) runs on one GPU")
        # BASELINE configuration 4's rule: the original 3DGS gradient-threshold densification
        refine_cfg = bsx.RefineConfig(refine_every=100, growth_grad_threshold=2e-4, min_opacity=0.005,
                                      max_splats=1_500_000, rule=bsx.REFINE_GRAD_THRESHOLD, percent_dense=0.01)
    refines = []

    def view(step):
        return (step * world + rank) % ncam

    # Training changes the splats and with them the work per step (scales and
    # opacities grow, and so do the intersections), so every measured region
    # below restarts from the same snapshot with a fresh trainer and the same
    # warm-up: the timed region, the per-kernel pass and the end-to-end run
    # all measure the same steps.
    snapshot = splats.clone()
    live = {"splats": splats, "trainer": None}

    def restart():
        # every region starts from an empty workspace, so buffer growth (a
        # densification run grows it repeatedly) costs every region the same
        refines.clear()
        torch.cuda.synchronize()
        ctx.trim()
        if not train:
            for i in range(args.warmup):
                step(i)
            return
        if live["trainer"] is not None:
            live["trainer"].close()
        live["splats"] = snapshot.clone()
        live["trainer"] = bsx.SplatTrainer(tcfg, live["splats"], process_group=pg, exchange=args.exchange)
        if refine_cfg is not None:  # the run's splat budget is allocated once, before timing
            live["trainer"].reserve(refine_cfg.max_splats, live["splats"])
        for i in range(args.warmup):
            step(i)

    if train:
        gts_host = [g.pin_memory() for g in gts_cpu]
        gts_dev = [g.to(dev) for g in gts_host]

        def step(i, gt=None):
            k = view(i)
            st = live["trainer"].step(cams[k], size, gts_dev[k] if gt is None else gt, live["splats"])
            it = i + 1
            if refine_cfg is not None and refine_cfg.due(it, tcfg.total_train_iters):
                rs = live["trainer"].refine(live["splats"], it, it, tcfg.total_train_iters, refine_cfg)
                refines.append((it, rs.total_splats, rs.num_added, rs.num_pruned))
            return st
    else:
        def step(i, gt=None):
            k = view(i)
            return render(cams[k], size, splats.transforms, splats.sh_coeffs, splats.raw_opacities,
                          raster_pass=bsx._lib.PASS_FORWARD)

    restart()

    # ---- timed region: device-resident inputs, no instrumentation ------------
    sampler = ClockSampler(local_rank)
    sampler.start()
    l0 = ctx.launches()
    stats = []

    def timed():
        for i in range(args.steps):
            stats.append(step(args.warmup + i))

    refines.clear()
    h0 = time.monotonic()
    ms = _time_region(args, world, timed)
    sampler.mark(h0, time.monotonic())
    timed_refines = list(refines)
    timed_n = live["splats"].num_splats
    launches = ctx.launches() - l0
    clocks = sampler.stop()

    # ---- per-kernel table: a separate pass over the same steps with CUDA
    # events around every launch (kept out of the timed region above) --------
    restart()
    ctx.profile_reset()
    ctx.profile(True)
    _time_region(args, world, lambda: [step(args.warmup + i) for i in range(args.steps)])
    ctx.profile(False)
    prof = ctx.profile_read()

    # ---- per-step distribution: an event after every step on the launching
    # stream (no host synchronisation added), the max over ranks per step -----
    restart()
    marks = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps + 1)]

    def per_step():
        marks[0].record()
        for i in range(args.steps):
            step(args.warmup + i)
            marks[i + 1].record()

    _time_region(args, world, per_step)
    step_times = torch.tensor([marks[i].elapsed_time(marks[i + 1]) for i in range(args.steps)], device=dev)
    if world > 1:
        torch.distributed.all_reduce(step_times, op=torch.distributed.ReduceOp.MAX)
    q = torch.quantile(step_times.double().cpu(), torch.tensor([0.1, 0.5, 0.9], dtype=torch.float64)).tolist()
    step_ms = {"p10": round(q[0], 4), "median": round(q[1], 4), "p90": round(q[2], 4),
               "note": "per-step CUDA-event times of a separate pass over the same steps (max over ranks)"}

    # ---- e2e: public API with host buffers ----------------------------------
    # Training: every step uploads its ground truth from pinned host memory and
    # reads its loss back into pinned host memory, inside the timed region; the
    # upload of step i+1 runs on a copy stream while step i computes (double
    # buffer), as a data loader would. It is issued once step i has been
    # enqueued, i.e. after step i's mid-step count read-back: an 8 MB upload
    # still in flight delays that 8-byte read-back (measured: 2.5 % of the
    # step when the upload was issued before the step). Render-only: every frame's packed image
    # is copied back to pinned host memory (no tensor input per frame: the
    # camera travels in the launch parameters).
    restart()
    compute = torch.cuda.current_stream()
    copy = torch.cuda.Stream()
    base = args.warmup
    if train:
        gt_buf = [torch.empty_like(gts_dev[0]) for _ in range(2)]
        loaded = [torch.cuda.Event() for _ in range(2)]
        consumed = [torch.cuda.Event() for _ in range(2)]
        loss_host = torch.empty(args.steps, dtype=torch.float32).pin_memory()

        def upload(i):
            b = i % 2
            with torch.cuda.stream(copy):
                if i >= 2:
                    copy.wait_event(consumed[b])
                gt_buf[b].copy_(gts_host[view(base + i)], non_blocking=True)
                loaded[b].record(copy)

        def e2e():
            upload(0)
            for i in range(args.steps):
                b = i % 2
                compute.wait_event(loaded[b])
                st = step(base + i, gt_buf[b])
                consumed[b].record(compute)
                loss_host[i:i + 1].copy_(st.loss, non_blocking=True)
                if i + 1 < args.steps:
                    upload(i + 1)

        e2e_sampler = ClockSampler(local_rank)
        e2e_sampler.start()
        h1 = time.monotonic()
        e2e_ms = _time_region(args, world, e2e)
        e2e_sampler.mark(h1, time.monotonic())
        clocks_e2e = e2e_sampler.stop()
        assert torch.isfinite(loss_host).all(), "non-finite loss in the end-to-end run"
        h2d, d2h = int(w * h * 4), 4
    else:
        frames_host = [torch.empty((h, w), dtype=torch.int32).pin_memory() for _ in range(2)]

        def e2e():
            for i in range(args.steps):
                out = step(base + i)
                frames_host[i % 2].copy_(out.out_img, non_blocking=True)

        e2e_sampler = ClockSampler(local_rank)
        e2e_sampler.start()
        h1 = time.monotonic()
        e2e_ms = _time_region(args, world, e2e)
        e2e_sampler.mark(h1, time.monotonic())
        clocks_e2e = e2e_sampler.stop()
        h2d, d2h = 0, int(w * h * 4)

    V = int(statistics.mean(s.num_visible if train else s.aux.num_visible for s in stats))
    M = int(statistics.mean(s.num_intersections if train else s.aux.num_intersections for s in stats))
    # surviving intersections after the forward early-out (backward-pass render of one view)
    sp = live["splats"]
    r = render(cams[view(args.warmup)], size, sp.transforms, sp.sh_coeffs, sp.raw_opacities)
    off = r.aux.tile_offsets.reshape(-1, 2).to(torch.int64)
    Mp = int((off[:, 1] - off[:, 0]).clamp_min(0).sum()) if train else M
    N, C = splats.num_splats, splats.sh_coeffs_per_splat
    P, T = w * h, ((w + 15) // 16) * ((h + 15) // 16)
    tile_passes = (max(1, T.bit_length()) + 7) // 8
    peak, peak_kind = _peaks()
    kernels = {}
    total_prof = max(sum(v[0] for v in prof.values()), 1e-9)
    for name, (tot, cnt) in prof.items():
        avg_ms = tot / max(cnt, 1)
        b = kernel_bytes(name, N, V, M, Mp, P, T, C, world, fused_adam=train and world == 1)
        if name in ("sort_pass_kernel", "sort_hist_kernel"):
            # two sorts per step: V depth keys (4 passes) and M tile keys
            per_step = (4 * 16 * V + tile_passes * 16 * M) if name == "sort_pass_kernel" else 4 * V + 4 * M
            b = per_step / max(cnt / args.steps, 1)
        if name == "raster_fwd_kernel" and not train:
            b = 52 * M + 4 * P + 8 * T
        kernels[name] = {"launches": cnt, "avg_ms": round(avg_ms, 4), "share": round(tot / total_prof, 4),
                         "alg_bytes": int(b), "gbs": round(b / (avg_ms * 1e-3) / 1e9, 1) if avg_ms > 0 else None}
    dom = max(prof.items(), key=lambda kv: kv[1][0])[0] if prof else None
    traffic = None
    tfile = ROOT / "profiles" / "dram_traffic_cfg2.txt"
    if args.workload == "cfg2" and tfile.exists() and dom:
        for ln in tfile.read_text().splitlines():
            parts = ln.split()
            if len(parts) == 2 and not ln.startswith("#") and parts[0] == dom:
                traffic = int(parts[1])
    roof = None
    if dom:
        kd = kernels[dom]
        ach = kd["gbs"] or 0.0
        roof = {"bound": "hbm", "kernel": dom, "achieved": ach, "peak": peak, "unit": "GB/s",
                "frac": round(ach / peak, 4), "traffic": traffic, "peak_source": f"{peak_kind} hbm_gbs",
                "note": "raster kernels are FP32/MUFU issue-bound; HBM fraction is reported as the spec asks"}
    value = args.steps * world / (ms * 1e-3)
    e2e_value = args.steps * world / (e2e_ms * 1e-3)
    unit = "train steps/s" if train else "frames/s"
    line = {
        "metric": METRIC if train else "render frames/s @6M splats SH3 2160p; ms per stage",
        "value": round(value, 3), "unit": unit, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded; no dataset)",
        "config": {"workload": WORKLOADS[args.workload], "splats": N, "sh_degree": int(round(C ** 0.5)) - 1,
                   "width": w, "height": h, "views": ncam,
                   "views_per_step_per_gpu": 1, "parallelism": f"dp{world}",
                   "l2": "inputs larger than L2" if N * (44 + 12 * C) > 126e6 else "inputs smaller than L2",
                   "exchange": _exchange_label(args, world, train, live["trainer"]),
                   "num_visible": V, "num_intersections": M, "intersections_after_early_out": Mp},
        "e2e": {"value": round(e2e_value, 3), "unit": unit, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
        # one view per GPU per step: views/s is the whole-job value; an optimizer step
        # consumes one view per GPU
        "throughput": {"views_per_s": round(value, 3),
                       "optimizer_steps_per_s": round(args.steps / (ms * 1e-3), 3)} if train else None,
        "gpu_launches": int(launches),
        "step_ms": step_ms,
        "roofline": roof,
        "kernels": kernels,
        "clocks": clocks,
        "clocks_e2e": clocks_e2e,
    }
    not_fwdbwd = ("adam_kernel", "dp_adam_kernel", "gather_stats_kernel")
    if refine_cfg is not None:
        line["refine"] = {"every": refine_cfg.refine_every, "refines_in_timed_region": len(timed_refines),
                          "start_splats": N, "end_splats": timed_n,
                          "log": [{"iter": r[0], "splats": r[1], "added": r[2], "pruned": r[3]}
                                  for r in timed_refines]}
    if train:
        line["fwd_bwd_ms"] = round(sum(v[0] for n, v in prof.items() if n not in not_fwdbwd) / args.steps, 4)
        if world == 1:
            line["fwd_bwd_note"] = "includes the Adam update fused into project_bwd_kernel"
        live["trainer"].close()
    else:
        stage = {"project": ("project_fwd_kernel", "compact_visible_kernel"), "scan": ("scan_kernel",),
                 "sort": ("sort_hist_kernel", "sort_pass_kernel"), "emit": ("emit_kernel", "tile_offsets_kernel"),
                 "rasterize": ("raster_fwd_kernel",)}
        line["stages_ms"] = {k: round(sum(prof[n][0] for n in v if n in prof) / args.steps, 4) for k, v in stage.items()}
    return line


def run_ply(args, rank, world, local_rank):
    """PLY import / export throughput (splats/s) through the public API's C entry points:
    each import step parses the header and uploads + decodes every row; each export
    step encodes and reads the file back into pinned host memory."""
    import ctypes as C

    import torch

    from brush_b200 import _lib
    from brush_b200 import splats as S
    from brush_b200._context import context, ptr
    from brush_b200.ply import export_into, export_size, load_splat_from_ply

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    splats, _, _, _ = S.config2_scene(dev, seed=2)
    size = export_size(splats)
    host = torch.empty(size, dtype=torch.uint8).pin_memory()
    n_file = export_into(splats, host)
    L = _lib.lib()
    ctx = context(dev)
    ctx.bind_stream()
    n, c = splats.num_splats, splats.sh_coeffs_per_splat
    t = torch.empty((n, 10), device=dev)
    sh = torch.empty((n, c, 3), device=dev)
    op = torch.empty((n,), device=dev)
    err = C.create_string_buffer(256)

    def import_step():
        h = C.c_void_p()
        info = _lib.PlyInfo()
        if L.bsx_ply_parse(host.data_ptr(), n_file, 1, C.byref(h), C.byref(info), err, 256):
            raise RuntimeError(err.value.decode())
        try:
            ctx.check(L.bsx_ply_load(ctx.handle, h, ptr(t), ptr(sh), ptr(op)))
        finally:
            L.bsx_ply_free(h)

    out = torch.empty(size, dtype=torch.uint8).pin_memory()

    def export_step():
        export_into(splats, out)

    for _ in range(args.warmup):
        import_step()
        export_step()
    torch.cuda.synchronize()
    assert torch.equal(sh, splats.sh_coeffs) and torch.equal(out[:n_file], host[:n_file])
    sampler = ClockSampler(local_rank)
    sampler.start()
    h0 = time.monotonic()
    l0 = ctx.launches()
    ms_imp = _time_region(args, world, lambda: [import_step() for _ in range(args.steps)])
    launches = ctx.launches() - l0
    ms_exp = _time_region(args, world, lambda: [export_step() for _ in range(args.steps)])
    sampler.mark(h0, time.monotonic())
    clocks = sampler.stop()
    ctx.profile_reset()
    ctx.profile(True)
    for _ in range(args.steps):
        import_step()
        export_step()
    torch.cuda.synchronize()
    ctx.profile(False)
    prof = ctx.profile_read()
    peak, peak_kind = _peaks()
    row_bytes = (14 + 3 * (c - 1)) * 4
    splat_bytes = 4 * (10 + 3 * c + 1)
    kernels = {}
    for name, (tot, cnt) in prof.items():
        alg = n * (row_bytes + splat_bytes)
        kernels[name] = {"launches": cnt, "avg_ms": round(tot / cnt, 4), "alg_bytes": alg,
                         "gbs": round(alg / (tot / cnt * 1e-3) / 1e9, 1)}
    dec = kernels.get("ply_decode_kernel", {"gbs": 0.0, "avg_ms": 0.0})
    value = world * n * args.steps / (ms_imp * 1e-3)
    line = {
        "metric": "PLY import splats/s (1M splats SH3, pinned host file bytes -> device splats)",
        "value": round(value, 1), "unit": "splats/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms_imp / args.steps, 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded cfg2 scene written as PLY)",
        "config": {"workload": WORKLOADS["ply"], "splats": n, "sh_degree": splats.sh_degree,
                   "file_bytes": n_file, "l2": "inputs larger than L2"},
        "e2e": {"value": round(value, 1), "unit": "splats/s", "h2d_bytes_per_step": n_file,
                "d2h_bytes_per_step": 0},
        "export": {"value": round(world * n * args.steps / (ms_exp * 1e-3), 1), "unit": "splats/s",
                   "ms_per_step": round(ms_exp / args.steps, 4), "d2h_bytes_per_step": n_file},
        "gpu_launches": launches,
        "roofline": {"bound": "hbm", "kernel": "ply_decode_kernel", "achieved": dec["gbs"], "peak": peak,
                     "unit": "GB/s", "frac": round(dec["gbs"] / peak, 4), "traffic": None, "peak_source": peak_kind,
                     "note": "the import is bound by the host-to-device copy of the file; the decode kernel "
                             "is the device part"},
        "h2d_gbs": round(n_file / (ms_imp / args.steps * 1e-3) / 1e9, 1),
        "kernels": kernels, "clocks": clocks,
    }
    return line


NATIVE_BUILD = "g++ -O3 -march=native -fopenmp -ffp-contract=off (built on the host that runs it)"


def cpu_baseline_sample(workload="cfg2"):
    """One oracle step (all host threads) on the same workload: a full training step, or a
    forward render for the render-only workload. Returns (seconds, threads)."""
    import numpy as np

    from brush_b200 import splats as S
    from oracle import oracle as orc

    if workload == "cfg1":
        splats, cam, size, gt = S.config1_scene("cpu", seed=1)
    elif workload == "cfg3":
        raise ValueError("cfg3 has no CPU sample (its targets are rendered by the GPU library)")
    elif workload == "ply":
        # the CPU restatement's decode of a 20 000-row sample of the same file, scaled per splat
        import torch

        sp, _, _, _ = S.config2_scene("cpu", seed=2, n=20000)
        data = _ply_host_bytes(sp)
        t0 = time.perf_counter()
        orc.ply_decode(data)
        return (time.perf_counter() - t0) * (1_000_000 / 20000), 1
    elif workload == "cfg5":
        splats, size = S.config5_scene("cpu", seed=5)
        cam = S.circle_cameras(120, 8.0, size[0], size[1])[0]
        t0 = time.perf_counter()
        orc.RenderResult(cam, size, splats.transforms.numpy(), splats.sh_coeffs.numpy(),
                         splats.raw_opacities.numpy())
        return time.perf_counter() - t0, orc.threads()
    else:
        splats, cam, size, gt = S.config2_scene("cpu", seed=2)
    t = splats.transforms.numpy()
    sh = splats.sh_coeffs.numpy()
    op = splats.raw_opacities.numpy()
    w, h = size
    t0 = time.perf_counter()
    r = orc.RenderResult(cam, size, t, sh, op)
    chw = np.ascontiguousarray(r.image[..., :3].transpose(2, 0, 1))
    oc = orc.loss_cfg(0.8, -0.2)
    orc.loss_fwd(chw, gt.numpy(), oc)
    dl = np.full((3, h, w), np.float32(1.0 / (3 * h * w)), np.float32)
    g = orc.loss_bwd(chw, gt.numpy(), oc, dl)
    vo = np.zeros((h, w, 4), np.float32)
    vo[..., :3] = g.transpose(1, 2, 0)
    vc = r.rasterize_bwd(vo)
    vt, vs, vop, _ = r.project_bwd(vc)
    n = t.shape[0]
    new = []
    for p, gr, red in [(t.copy(), vt, False), (sh.reshape(n, -1).copy(), vs.reshape(n, -1), True),
                       (op.reshape(n, 1).copy(), vop.reshape(n, 1), False)]:
        orc.adam(p, gr, np.zeros_like(p), np.zeros(n, np.float32) if red else np.zeros_like(p), 1e-3, None, red)
        new.append(p)
    # the mean-noise step after the optimizer (train.rs:1095-1169), gated on this step's visibility
    orc.mean_noise_step(new[0], new[2], r.visible, 5e-3, 1.0, 42, 1)
    return time.perf_counter() - t0, orc.threads()


def _ply_host_bytes(sp) -> bytes:
    """The 3DGS binary PLY of CPU splats, written with numpy (same layout as splat_to_ply)."""
    import numpy as np

    t = sp.transforms.numpy()
    sh = sp.sh_coeffs.numpy()
    op = sp.raw_opacities.numpy()
    n, c = t.shape[0], sh.shape[1]
    q = t[:, 3:7]
    rn = np.maximum(np.sqrt(((q[:, 0] * q[:, 0] + q[:, 1] * q[:, 1]) + q[:, 2] * q[:, 2]) + q[:, 3] * q[:, 3]),
                    np.float32(1e-12))
    cols = [t[:, 0], t[:, 1], t[:, 2], t[:, 7], t[:, 8], t[:, 9], op] + [q[:, k] / rn for k in range(4)]
    cols += [sh[:, 0, k] for k in range(3)] + [sh[:, k, ch] for ch in range(3) for k in range(1, c)]
    rows = np.stack(cols, 1).astype("<f4")
    names = ["x", "y", "z", "scale_0", "scale_1", "scale_2", "opacity", "rot_0", "rot_1", "rot_2", "rot_3",
             "f_dc_0", "f_dc_1", "f_dc_2"] + [f"f_rest_{k}" for k in range(3 * (c - 1))]
    head = "ply\nformat binary_little_endian 1.0\nelement vertex %d\n" % n
    head += "".join(f"property float {nm}\n" for nm in names) + "end_header\n"
    return head.encode() + rows.tobytes()


def run_reference(args, rank, world):
    if rank != 0:
        return None
    from oracle import build as obuild

    from oracle import oracle as orc

    orc.use_library(obuild.build_native())
    orc.set_threads(os.cpu_count() or 1)
    if args.workload == "cfg3":
        return {"impl": "reference", "unavailable": "cfg3 targets are rendered by the GPU library; no CPU sample"}
    if args.workload == "ply":
        times = []
        for i in range(args.warmup + args.steps):
            dt, cores = cpu_baseline_sample("ply")
            if i >= args.warmup:
                times.append(dt)
        value = 1_000_000 * args.steps / sum(times)
        return {"impl": "reference", "metric": "PLY import splats/s (1M splats SH3, pinned host file bytes -> "
                "device splats)", "value": round(value, 1), "unit": "splats/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(1000 * sum(times) / args.steps, 2),
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
                "data": "synthetic (seeded cfg2 scene written as PLY)", "config": {"workload": WORKLOADS["ply"]},
                "cpu_baseline": {"value": round(value, 1), "unit": "splats/s", "cores": 1, "kind": "port",
                                 "sample": "the CPU restatement's decode of a 20 000-row sample of the same file, "
                                           "scaled to 1M splats"},
                "e2e": {"value": round(value, 1), "unit": "splats/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}}
    times = []
    for i in range(args.warmup + args.steps):
        dt, cores = cpu_baseline_sample(args.workload)
        if i >= args.warmup:
            times.append(dt)
    total = sum(times)
    value = args.steps / total
    unit = "frames/s" if args.workload == "cfg5" else "train steps/s"
    what = "forward render" if args.workload == "cfg5" else "train step"
    return {
        "impl": "reference", "metric": METRIC if args.workload != "cfg5" else "render frames/s @6M splats SH3 2160p",
        "value": round(value, 5), "unit": unit, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(1000 * total / args.steps, 2),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded; no dataset)",
        "config": {"workload": WORKLOADS[args.workload]},
        "cpu_baseline": {"value": round(value, 5), "unit": unit, "cores": cores, "kind": "port",
                         "build": NATIVE_BUILD,
                         "sample": f"one full {args.workload} {what} per timed step (CPU restatement of the "
                                   "reference algorithm; the Rust/wgpu reference cannot be built or run on this box)"},
        "e2e": {"value": round(value, 5), "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--exchange", default="auto", choices=["auto", "peer", "nvls", "nccl"],
                    help="data-parallel gradient exchange with --gpus > 1")
    ap.add_argument("--workload", default="cfg2", choices=sorted(WORKLOADS),
                    help="BASELINE configuration (cfg2 is the headline metric)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        line = run_reference(args, rank, world)
        if line is not None:
            print(json.dumps(line), flush=True)
        return
    import torch

    if world > 1:
        import datetime

        torch.cuda.set_device(local_rank)
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                             device_id=torch.device("cuda", local_rank))
    from brush_b200 import build as bbuild

    if rank == 0:
        bbuild.build()
    if world > 1:
        torch.distributed.barrier()
    if args.workload == "ply":
        line = run_ply(args, rank, world, local_rank)
    else:
        line = run_ours(args, rank, world, local_rank)
    if rank == 0 and world == 1 and not args.no_cpu_baseline and args.workload != "cfg3":
        from oracle import build as obuild

        from oracle import oracle as orc

        orc.use_library(obuild.build_native())
        orc.set_threads(os.cpu_count() or 1)
        dt, cores = cpu_baseline_sample(args.workload)
        if args.workload == "ply":
            line["cpu_baseline"] = {"value": round(1_000_000 / dt, 1), "unit": "splats/s", "cores": cores,
                                    "kind": "port", "build": NATIVE_BUILD,
                                    "sample": "the CPU restatement's decode of a 20 000-row sample "
                                              "of the same file, scaled to 1M splats"}
        else:
            what = "forward render" if args.workload == "cfg5" else "train step"
            # the same sample on one host thread (the restatement's loops are OpenMP-parallel)
            orc.set_threads(1)
            dt1, _ = cpu_baseline_sample(args.workload)
            orc.set_threads(os.cpu_count() or 1)
            line["cpu_baseline"] = {"value": round(1.0 / dt, 5), "unit": line["unit"], "cores": cores,
                                    "kind": "port", "build": NATIVE_BUILD,
                                    "value_1core": round(1.0 / dt1, 5),
                                    "sample": f"one full {args.workload} {what} on the CPU restatement, all host "
                                              f"threads ({cores}); value_1core: the same on one thread"}
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()

#!/usr/bin/env python3
"""Benchmark: Brush's differentiable Gaussian-splat training step on B200.

Workload: 1,000,000 splats, SH degree 3, 1920x1080,
seeded synthetic scene (64 isotropic clusters, sigma 0.3, inside a radius-5
ball; log-scales N(-4.5,0.7); opacity logits N(0,1.5)), cameras on a radius-8
orbit, uniform random targets. One step = render forward (backward-pass
bookkeeping) -> 0.8 L1 + 0.2 (1-SSIM) loss and gradient -> raster backward ->
projection backward -> [N>1: NCCL all-reduce of the flat gradient] -> fused
Adam with the reference's learning-rate table -> refine statistics.

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
    """Samples nvidia-smi clocks / throttle reasons while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except (FileNotFoundError, OSError):
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
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
                "reasons": sorted(reasons), "samples": len(sm)}


# Algorithmic bytes moved by each kernel per launch (fp32 = 4 B). N splats,
# V visible, M intersections, Mp intersections surviving the forward early-out,
# P pixels, T tiles, C SH coefficients per splat.
def kernel_bytes(name, N, V, M, Mp, P, T, C, W=1):
    row = 4 * (11 + 3 * C)  # bytes of one splat's parameters (or gradients)
    table = {
        "project_fwd_kernel": 44 * N + 8 * N + N // 8 + V * (12 * C + 48 + 4),
        "compact_visible_kernel": 4 * N + N // 8 + 12 * V,
        "sort_hist_kernel": 4 * V,  # depth sort; the tile sort adds 4 M (below)
        "sort_pass_kernel": 16 * V,
        "scan_kernel": 12 * V,
        "emit_kernel": V * (4 + 48 + 8) + 8 * M,
        "tile_offsets_kernel": 8 * M + 8 * T,
        "raster_fwd_kernel": 52 * Mp + 16 * P + 8 * T + 4 * V,
        "loss_fused_kernel": 36 * P,
        "loss_mean_kernel": 0,
        "raster_bwd_kernel": 32 * P + 52 * Mp + 48 * V,
        "project_bwd_kernel": 48 * N + V * (44 + 12 * C) + N * (48 + 12 * C),
        "adam_kernel": (316 + 60 * C) * N,
        "gather_stats_kernel": 36 * N,
        # NVLink bytes per rank: peer gradient rows in + parameter rows out
        "dp_adam_kernel": 2 * (W - 1) * (N // W) * row if W > 1 else 0,
    }
    return table.get(name, 0)


def run_ours(args, rank, world, local_rank):
    import torch

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    import brush_b200 as bsx
    from brush_b200._context import context
    from brush_b200.splats import config2_scene, orbit_camera, random_gt

    pg = None
    if world > 1:
        pg = torch.distributed.group.WORLD
    splats, _, size, _ = config2_scene(dev, seed=2)
    w, h = size
    ncam = 16
    cams = [orbit_camera(i, ncam, 8.0, w, h) for i in range(ncam)]
    gts_host = [random_gt(h, w, 1000 + i, "cpu").pin_memory() for i in range(ncam)]
    gts_dev = [g.to(dev) for g in gts_host]
    trainer = bsx.SplatTrainer(bsx.TrainConfig(), splats, process_group=pg, exchange=args.exchange)
    ctx = context(dev)

    def view(step):
        return (step * world + rank) % ncam

    def step(i, gt=None):
        k = view(i)
        return trainer.step(cams[k], size, gts_dev[k] if gt is None else gt, splats)

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()

    # ---- timed region: device-resident inputs -------------------------------
    sampler = ClockSampler(local_rank)
    sampler.start()
    ctx.profile_reset()
    ctx.profile(True)
    l0 = ctx.launches()
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    stats = []
    e0.record()
    for i in range(args.steps):
        stats.append(step(args.warmup + i))
    e1.record()
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    ms = e0.elapsed_time(e1)
    launches = ctx.launches() - l0
    ctx.profile(False)
    prof = ctx.profile_read()
    clocks = sampler.stop()
    t = torch.tensor([ms], device=dev)
    if world > 1:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    ms = float(t.item())

    # ---- e2e: public API with host buffers (GT upload + loss readback) -------
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    x0, x1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    x0.record()
    for i in range(args.steps):
        k = view(args.warmup + args.steps + i)
        gt = gts_host[k].to(dev, non_blocking=True)
        st = step(args.warmup + args.steps + i, gt)
        float(st.loss.item())
    x1.record()
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    e2e_ms = x0.elapsed_time(x1)
    t = torch.tensor([e2e_ms], device=dev)
    if world > 1:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    e2e_ms = float(t.item())

    # fwd+bwd time (render + loss + raster bwd + project bwd) from the profile
    fwdbwd_names = [n for n in prof if n not in ("adam_kernel",)]
    fwdbwd_ms = sum(prof[n][0] for n in fwdbwd_names) / args.steps

    V = int(statistics.mean(s.num_visible for s in stats))
    M = int(statistics.mean(s.num_intersections for s in stats))
    out = trainer  # noqa: F841
    # surviving intersections after the forward early-out
    Mp = M
    try:
        from brush_b200.render import render

        r = render(cams[view(0)], size, splats.transforms, splats.sh_coeffs, splats.raw_opacities)
        off = r.aux.tile_offsets.reshape(-1, 2).to(torch.int64)
        Mp = int((off[:, 1] - off[:, 0]).clamp_min(0).sum())
    except Exception:  # noqa: BLE001
        pass
    N, C = splats.num_splats, splats.sh_coeffs_per_splat
    P, T = w * h, ((w + 15) // 16) * ((h + 15) // 16)
    peak, peak_kind = _peaks()
    kernels = {}
    for name, (tot, cnt) in prof.items():
        avg_ms = tot / max(cnt, 1)
        b = kernel_bytes(name, N, V, M, Mp, P, T, C, world)
        if name in ("sort_pass_kernel", "sort_hist_kernel"):
            # two sorts per step: V depth keys (4 passes) and M tile keys (2 passes at 1080p)
            per_step = 4 * 16 * V + 2 * 16 * M if name == "sort_pass_kernel" else 4 * V + 4 * M
            b = per_step / max(cnt / args.steps, 1)
        kernels[name] = {"launches": cnt, "avg_ms": round(avg_ms, 4), "share": round(tot / max(sum(v[0] for v in prof.values()), 1e-9), 4),
                         "alg_bytes": int(b), "gbs": round(b / (avg_ms * 1e-3) / 1e9, 1) if avg_ms > 0 else None}
    dom = max(prof.items(), key=lambda kv: kv[1][0])[0] if prof else None
    traffic = None
    tfile = ROOT / "profiles" / "dram_traffic_cfg2.txt"
    if tfile.exists() and dom:
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
    line = {
        "metric": METRIC, "value": round(value, 3), "unit": "train steps/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded; no dataset)",
        "config": {"workload": WORKLOAD, "splats": N, "sh_degree": 3, "width": w, "height": h,
                   "views_per_step_per_gpu": 1, "parallelism": f"dp{world}", "l2": "inputs larger than L2",
                   "exchange": (None if world == 1 else
                                "peer-memory fused reduce+Adam+broadcast kernel" if args.exchange == "peer" else
                                "NCCL reduce-scatter + sharded Adam + all-gather"),
                   "num_visible": V, "num_intersections": M, "intersections_after_early_out": Mp},
        "fwd_bwd_ms": round(fwdbwd_ms, 4),
        "e2e": {"value": round(e2e_value, 3), "unit": "train steps/s",
                "h2d_bytes_per_step": int(w * h * 4), "d2h_bytes_per_step": 4},
        "gpu_launches": int(launches),
        "roofline": roof,
        "kernels": kernels,
        "clocks": clocks,
    }
    trainer.close()
    return line


def cpu_baseline_sample(dev_scene=None):
    """One oracle training step (all host threads) on the same config-2 workload."""
    import numpy as np

    from brush_b200.splats import config2_scene
    from oracle import oracle as orc

    splats, cam, size, gt = config2_scene("cpu", seed=2)
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
    for p, gr, red in [(t.copy(), vt, False), (sh.reshape(n, -1).copy(), vs.reshape(n, -1), True),
                       (op.reshape(n, 1).copy(), vop.reshape(n, 1), False)]:
        orc.adam(p, gr, np.zeros_like(p), np.zeros(n, np.float32) if red else np.zeros_like(p), 1e-3, None, red)
    return time.perf_counter() - t0, orc.threads()


def run_reference(args, rank, world):
    if rank != 0:
        return None
    from oracle import build as obuild

    obuild.build()
    from oracle import oracle as orc

    orc.set_threads(os.cpu_count() or 1)
    times = []
    for i in range(args.warmup + args.steps):
        dt, cores = cpu_baseline_sample()
        if i >= args.warmup:
            times.append(dt)
    total = sum(times)
    value = args.steps / total
    return {
        "impl": "reference", "metric": METRIC, "value": round(value, 5), "unit": "train steps/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(1000 * total / args.steps, 2),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded; no dataset)",
        "config": {"workload": WORKLOAD, "splats": 1_000_000, "sh_degree": 3, "width": 1920, "height": 1080},
        "cpu_baseline": {"value": round(value, 5), "unit": "train steps/s", "cores": cores, "kind": "port",
                         "sample": "full config-2 train step per timed step (CPU restatement of the reference "
                                   "algorithm; the Rust/wgpu reference cannot be built or run on this box)"},
        "e2e": {"value": round(value, 5), "unit": "train steps/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--exchange", default="peer", choices=["peer", "nccl"],
                    help="data-parallel gradient exchange with --gpus > 1")
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
    line = run_ours(args, rank, world, local_rank)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        from oracle import build as obuild

        obuild.build()
        from oracle import oracle as orc

        orc.set_threads(os.cpu_count() or 1)
        dt, cores = cpu_baseline_sample()
        line["cpu_baseline"] = {"value": round(1.0 / dt, 5), "unit": "train steps/s", "cores": cores, "kind": "port",
                                "sample": "one full config-2 train step on the CPU restatement, all host threads"}
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()

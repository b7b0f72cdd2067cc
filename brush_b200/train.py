"""Training step, mirroring ``SplatTrainer::step_with_refine_weight``
(crates/brush-train/src/train.rs:619-1182).

One step: backward-pass render -> fused SSIM+L1 loss and its gradient ->
raster backward -> projection backward -> fused AdamScaled over transforms /
SH / opacity with the reference's learning-rate table (train.rs:964-1051) ->
refine statistics (stats.rs:111-121).

On one GPU, and with several ranks using the peer-memory exchange, the whole
step is one call into the library (``bsx_train_step`` / ``bsx_train_step_dp``,
a native trainer owning gradients, moments, schedules and statistics). The
NCCL alternative (``exchange="nccl"``) orchestrates the same kernels from
here around reduce-scatter / all-gather (brush_b200.dist).

The reference's mean-noise injection after Adam (train.rs:1095-1169) is
applied (TrainConfig.mean_noise, on by default) with normals from a
counter-based generator, so it is reproducible; the parity tests switch it off.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np
import torch

from . import _lib
from ._context import context, device_view, ptr
from .adam import AdamGroup, AdamScaled
from .camera import Camera
from .dist import all_gather_rows, reduce_gradients, reduce_scatter_rows, row_shard
from .loss import ImageLossConfig, image_loss_fused
from .render import render
from .render_bwd import SplatGrads, project_bwd, rasterize_bwd
from .splats import Splats, splat_bounds


@dataclass
class TrainConfig:
    """Hot-path subset of ``TrainConfig`` (crates/brush-train/src/config.rs:9-498) with its defaults."""
    total_train_iters: int = 30000
    lr_mean: float = 2e-5
    lr_mean_end: float = 2e-7
    lr_coeffs_dc: float = 2e-3
    lr_coeffs_sh_scale: float = 10.0
    lr_opac: float = 0.012
    lr_scale: float = 7e-3
    lr_scale_end: float = 5e-3
    lr_rotation: float = 2e-3
    ssim_weight: float = 0.2
    background_color: tuple = (0.0, 0.0, 0.0)
    bounds_percentile: float = 0.8
    # A single learning rate for every parameter (benchmark configuration 1:
    # "one Adam step, lr 1e-3"); None selects the reference table above.
    uniform_lr: float | None = None
    # Mean-noise injection after the optimizer step (train.rs:1095-1169), on by default
    # like the reference: low-opacity splats' means move by N(0,1) * (1-opacity)^150 *
    # lr_mean * mean_noise_weight (clamped to the median bounds size). With
    # mrnf_noise_injection (default) only splats visible since the last refine move,
    # otherwise only those visible in this step. Drawn from a counter-based generator
    # seeded by noise_seed, so runs are reproducible and data-parallel replicas agree.
    mean_noise: bool = True
    mean_noise_weight: float = 50.0
    mrnf_noise_injection: bool = True
    noise_seed: int = 42
    # keep the view-space gradient-norm sum the gradient-threshold densification rule reads
    accumulate_grad2d: bool = False

    def to_c(self, median_scale: float, render_mode: int, gather_stats: bool) -> _lib.TrainConfig:
        c = _lib.TrainConfig()
        c.total_train_iters = int(self.total_train_iters)
        c.lr_mean, c.lr_mean_end = float(self.lr_mean), float(self.lr_mean_end)
        c.lr_coeffs_dc, c.lr_coeffs_sh_scale = float(self.lr_coeffs_dc), float(self.lr_coeffs_sh_scale)
        c.lr_opac = float(self.lr_opac)
        c.lr_scale, c.lr_scale_end = float(self.lr_scale), float(self.lr_scale_end)
        c.lr_rotation = float(self.lr_rotation)
        c.ssim_weight = float(self.ssim_weight)
        c.background[:] = [float(v) for v in self.background_color]
        c.median_scale = float(median_scale)
        c.uniform_lr = float(self.uniform_lr) if self.uniform_lr is not None else 0.0
        c.render_mode = int(render_mode)
        c.gather_stats = int(gather_stats)
        c.mean_noise = int(self.mean_noise)
        c.noise_vis_gate = int(self.mrnf_noise_injection)
        c.mean_noise_weight = float(self.mean_noise_weight)
        c.noise_seed = int(self.noise_seed)
        c.accumulate_grad2d = int(self.accumulate_grad2d)
        return c


@dataclass
class RefineConfig:
    """Refine options of ``TrainConfig`` (crates/brush-train/src/config.rs:100-330) with their defaults."""
    refine_every: int = 200
    max_splats: int = 10_000_000
    growth_grad_threshold: float = 0.0025
    growth_select_fraction: float = 0.07
    growth_stop_iter: int = 15000
    split_at_screen_size: float = 0.5
    opac_decay: float = 0.004
    scale_decay: float = 0.002
    min_scale_prune: bool = True
    min_scale_prune_threshold: float = 1e-10
    near_zero_rotation_prune: bool = True
    radial_bounds_prune: bool = False
    min_opacity: float = 1.0 / 255.0
    prune_extent_factor: float = 100.0
    split_long_axis_scale: float = 0.5
    split_other_axis_scale: float = 0.85
    split_opacity_scale: float = 0.6
    seed: int = 42
    # _lib.REFINE_REFERENCE: the reference's refine_for_phase; _lib.REFINE_GRAD_THRESHOLD: the
    # original 3DGS rule (average view-space gradient norm >= growth_grad_threshold: clone
    # splats whose largest scale is <= percent_dense x the bounds extent, split the others
    # into two), which needs TrainConfig.accumulate_grad2d
    rule: int = _lib.REFINE_REFERENCE
    percent_dense: float = 0.01

    def to_c(self) -> _lib.RefineConfig:
        c = _lib.RefineConfig()
        for name, _ in _lib.RefineConfig._fields_:
            setattr(c, name, type(getattr(c, name))(getattr(self, name)))
        return c

    def due(self, phase_iter: int, phase_total: int) -> bool:
        """The training loop's gate (crates/brush-process/src/train_stream.rs:481-483)."""
        progress = min(max(np.float32(phase_iter) / np.float32(max(phase_total, 1)), 0.0), 1.0)
        return phase_iter > 0 and phase_iter % self.refine_every == 0 and progress <= 0.95


def _world_of(process_group) -> int:
    return 1 if process_group is None else torch.distributed.get_world_size(process_group)


@dataclass
class TrainStepStats:
    num_visible: int
    num_intersections: int
    loss: torch.Tensor  # device scalar
    lr_mean: float


@dataclass
class RefineRecord:
    """``RefineRecord`` statistics (crates/brush-train/src/stats.rs:11-127), plus the
    view-space gradient-norm sum of the gradient-threshold rule (native trainer)."""
    refine_weight_norm: torch.Tensor
    vis_weight: torch.Tensor
    max_screen_size: torch.Tensor
    grad2d_accum: torch.Tensor | None = None

    @staticmethod
    def new(n: int, device) -> "RefineRecord":
        z = lambda: torch.zeros(n, device=device)
        return RefineRecord(z(), z(), z())

    def gather_stats(self, refine_weight, visible, screen_radius) -> None:
        """gather_stats (stats.rs:111-121); without a refine weight gather_aux_stats (:123-127)."""
        if refine_weight is not None:
            torch.maximum(self.refine_weight_norm, refine_weight, out=self.refine_weight_norm)
        self.vis_weight.add_(visible)
        torch.maximum(self.max_screen_size, screen_radius, out=self.max_screen_size)


class _NativeTrainer:
    """Owner of one ``bsx_trainer`` (gradients, moments, schedules, statistics)."""

    def __init__(self, device: int, n: int, c: int, cfg: _lib.TrainConfig):
        self.ctx = context(device)
        self.device = device
        self.n, self.c = n, c
        h = C.c_void_p()
        self.ctx.check(_lib.lib().bsx_trainer_create(self.ctx.handle, n, c, C.byref(cfg), C.byref(h)))
        self.handle = h
        self.gather = bool(cfg.gather_stats)

    def grads(self) -> SplatGrads:
        p = [C.c_void_p() for _ in range(4)]
        self.ctx.check(_lib.lib().bsx_trainer_grad_buffers(self.handle, *[C.byref(x) for x in p]))
        n, c, d = self.n, self.c, self.device
        return SplatGrads(device_view(p[0].value, (n, 10), torch.float32, d),
                          device_view(p[1].value, (n, c, 3), torch.float32, d),
                          device_view(p[2].value, (n,), torch.float32, d),
                          device_view(p[3].value, (n,), torch.float32, d))

    def raster_grads(self) -> torch.Tensor:
        """The last step's raster-backward rows [N, 12] (the projection backward's input)."""
        p = C.c_void_p()
        self.ctx.check(_lib.lib().bsx_trainer_raster_grads(self.handle, C.byref(p)))
        return device_view(p.value, (self.n, _lib.BSX_GRAD_STRIDE), torch.float32, self.device)

    def record(self) -> RefineRecord | None:
        if not self.gather:
            return None
        p = [C.c_void_p() for _ in range(4)]
        self.ctx.check(_lib.lib().bsx_trainer_stats_buffers(self.handle, *[C.byref(x) for x in p[:3]]))
        self.ctx.check(_lib.lib().bsx_trainer_grad2d_accum(self.handle, C.byref(p[3])))
        return RefineRecord(*[device_view(x.value, (self.n,), torch.float32, self.device) for x in p])

    def optimizer_state(self):
        """((m_transforms, m_sh, m_opac), (v_transforms, v_sh, v_opac)) views, or None before the first step."""
        p = [C.c_void_p() for _ in range(6)]
        rows = C.c_uint32()
        self.ctx.check(_lib.lib().bsx_trainer_optimizer_state(self.handle, *[C.byref(x) for x in p], C.byref(rows)))
        r, d = rows.value, self.device
        if r == 0 or not p[0].value:
            return None
        shapes = [(r, 10), (r, self.c, 3), (r,), (r, 10), (r,), (r,)]
        views = [device_view(x.value, sh, torch.float32, d) for x, sh in zip(p, shapes)]
        return tuple(views[:3]), tuple(views[3:])

    def load_optimizer_state(self, m, v, rows: int, world: int = 1, rank: int = 0) -> None:
        """Replace the moments with device tensors laid out as optimizer_state() returns them."""
        arrs = [t.contiguous() for t in (*m, *v)]
        self.ctx.check(_lib.lib().bsx_trainer_load_optimizer_state(self.handle, *[t.data_ptr() for t in arrs],
                                                                    int(rows), int(world), int(rank)))
        torch.cuda.current_stream(self.device).synchronize()

    def close(self) -> None:
        if self.handle:
            self.ctx.check(_lib.lib().bsx_trainer_destroy(self.handle))
            self.handle = None


class SplatTrainer:
    def __init__(self, config: TrainConfig, splats: Splats, process_group=None, gather_stats: bool = True,
                 shard_optimizer: bool = True, exchange: str = "auto", keep_gradients: bool = False):
        self.config = config
        # The single-GPU step applies AdamScaled inside the projection backward;
        # keep_gradients also writes the dense gradients to ``grads``.
        self.keep_gradients = keep_gradients
        # Data-parallel exchange with several ranks:
        #   "peer": one fused kernel over peer memory (brush_b200.peer); the
        #           splat parameters then live in the exchange region and the
        #           tensors of ``splats`` are rebound to it.
        #   "nccl": with shard_optimizer and N divisible by the world size,
        #           reduce-scatter gradients -> fused Adam on this rank's row
        #           shard -> all-gather; otherwise all-reduce -> full Adam.
        #   "nvls": the peer exchange over PyTorch symmetric memory with an
        #           NVLink multicast mapping: the gradient rows are summed in the
        #           NVSwitch and the updated rows multicast to every rank
        #           (falls back to "peer" where the devices offer no multicast).
        #   "auto": "nvls" from 8 ranks on, "peer" below. Per GPU and link
        #           direction the multicast form moves about (1 + 1/W) S bytes
        #           per step (S: the parameter bytes; the switch also returns
        #           each rank its own copy) against 2 (W - 1) / W S for the
        #           peer form, whose gradient push overlaps the projection
        #           backward. Measured on 8 B200s at config 2: 2691 vs 2662
        #           views/s at 8 ranks, 1351 vs 1387 at 4.
        if exchange not in ("auto", "peer", "nvls", "nccl"):
            raise ValueError("exchange must be 'auto', 'peer', 'nvls' or 'nccl'")
        if exchange == "auto":
            exchange = "nvls" if _world_of(process_group) >= 8 else "peer"
        self.exchange = exchange
        self.peer = None
        self.native = None
        self.shard_optimizer = shard_optimizer
        self.adam = AdamScaled(epsilon=1e-15)
        self.step_count = 0
        self.pg = process_group
        self.world = 1 if process_group is None else torch.distributed.get_world_size(process_group)
        self.gather_stats = gather_stats
        # trainer bounds (percentile AABB of the means); the rate uses their median size
        # as f32 (lr * median_scale as f64, train.rs:656,991); refine updates both
        self.bounds = splat_bounds(splats.means(), config.bounds_percentile)
        self.median_scale = float(np.float32(np.sort(self.bounds[1])[1] * np.float32(2.0)))
        t = max(config.total_train_iters, 1)
        self.mean_decay = (config.lr_mean_end / config.lr_mean) ** (1.0 / t)
        self.scale_decay = ((config.lr_scale_end / config.lr_scale) ** (1.0 / t)
                            if config.lr_scale > 0 and config.lr_scale_end > 0 else 1.0)
        # burn ExponentialLrScheduler state: starts at initial / gamma (first step uses the initial rate)
        self._mean_prev = config.lr_mean / self.mean_decay
        self._scale_prev = config.lr_scale / self.scale_decay
        self._alloc(splats)

    def _alloc(self, splats: Splats) -> None:
        n, c = splats.num_splats, splats.sh_coeffs_per_splat
        dev = splats.transforms.device
        self.n, self.c = n, c
        self.loss = torch.empty(1, device=dev)
        self.v_output = None
        self.groups = None
        old_peer, self.peer = self.peer, None
        old_native, self.native = self.native, None
        if self.world == 1 or self.exchange in ("peer", "nvls"):
            self.native = _NativeTrainer(dev.index, n, c, self.config.to_c(self.median_scale, splats.render_mode,
                                                                          self.gather_stats))
            self.native.ctx.check(_lib.lib().bsx_trainer_keep_gradients(self.native.handle,
                                                                        int(self.keep_gradients)))
            self.record = self.native.record()
            if self.world > 1:
                from .peer import PeerExchange

                self.peer = PeerExchange(n, c, dev.index, self.pg, multicast=self.exchange == "nvls")
                self.peer.load(splats.transforms, splats.sh_coeffs, splats.raw_opacities)
                splats.transforms, splats.sh_coeffs, splats.raw_opacities = self.peer.params
                # dense gradients of this rank's view only with keep_gradients; otherwise
                # these buffers hold the exchange slots the ranks push their rows into
                self.grads = SplatGrads(*self.peer.grads, v_refine_weight=self.peer.refine)
                self._dp = self.peer.train_structs()
            else:
                self.grads = self.native.grads()
            self.flat_grad = None
            self.sharded = False
        else:
            # One flat gradient buffer so data-parallel ranks all-reduce once per step.
            self.flat_grad = torch.empty(n * (10 + 3 * c + 1), device=dev)
            g = self.flat_grad
            self.grads = SplatGrads(
                v_transforms=g[: n * 10].view(n, 10),
                v_coeffs=g[n * 10: n * (10 + 3 * c)].view(n, c, 3),
                v_raw_opac=g[n * (10 + 3 * c):].view(n),
                v_refine_weight=torch.empty(n, device=dev),
            )
            self.v_combined = torch.empty((max(n, 1), _lib.BSX_GRAD_STRIDE), device=dev)
            self.record = RefineRecord.new(n, dev) if self.gather_stats else None
            self.sharded = self.shard_optimizer and n % self.world == 0
            if self.sharded:
                self.rank = torch.distributed.get_rank(self.pg)
                self.row0, self.row1 = row_shard(n, self.world, self.rank)
                r = self.row1 - self.row0
                self.shard_grads = (torch.empty((r, 10), device=dev), torch.empty((r, 3 * c), device=dev),
                                    torch.empty((r, 1), device=dev))
        if old_peer is not None:
            old_peer.close()
        if old_native is not None:
            old_native.close()

    def _lr_table(self):
        """Rates of this step: burn ExponentialLrScheduler, stepped once per optimizer step."""
        cfg = self.config
        if cfg.uniform_lr is not None:
            return cfg.uniform_lr, None, cfg.uniform_lr, None, cfg.uniform_lr, cfg.uniform_lr
        self._mean_prev *= self.mean_decay
        self._scale_prev *= self.scale_decay
        lr_mean = self._mean_prev * self.median_scale
        lr_scale = self._scale_prev
        tscale = [lr_mean] * 3 + [cfg.lr_rotation] * 4 + [lr_scale] * 3
        sh_scale = [1.0] + [1.0 / cfg.lr_coeffs_sh_scale] * (self.c - 1)
        sh_cols = [s for s in sh_scale for _ in range(3)]
        return 1.0, tscale, cfg.lr_coeffs_dc, sh_cols, cfg.lr_opac, lr_mean

    def step(self, camera: Camera, img_size: tuple, gt_packed: torch.Tensor, splats: Splats,
             compute_refine_weight: bool = True) -> TrainStepStats:
        """One optimisation step in place on ``splats`` (device tensors)."""
        if splats.num_splats != self.n or splats.sh_coeffs_per_splat != self.c:
            self._alloc(splats)
        if self.native is not None:
            return self._native_step(camera, img_size, gt_packed, splats, compute_refine_weight)
        return self._nccl_step(camera, img_size, gt_packed, splats, compute_refine_weight)

    def _native_step(self, camera, img_size, gt_packed, splats, compute_refine_weight) -> TrainStepStats:
        L = _lib.lib()
        ctx = context(splats.transforms.device)
        w, h = img_size
        cam = camera.to_c()
        st = _lib.TrainStats()
        if gt_packed.shape != (h, w) or gt_packed.dtype not in (torch.int32, torch.uint32):
            raise ValueError("gt_packed must be [H,W] packed RGBA8 (int32/uint32)")
        if self.peer is None:
            ctx.check(L.bsx_train_step(self.native.handle, C.byref(cam), w, h, ptr(gt_packed), ptr(splats.transforms),
                                       ptr(splats.sh_coeffs), ptr(splats.raw_opacities), int(compute_refine_weight),
                                       ptr(self.loss), C.byref(st)))
        else:
            ex, sp = self._dp
            ctx.check(L.bsx_train_step_dp(self.native.handle, C.byref(cam), w, h, ptr(gt_packed), C.byref(ex),
                                          C.byref(sp), int(compute_refine_weight), ptr(self.loss), C.byref(st)))
        self.step_count = int(st.step)
        return TrainStepStats(int(st.num_visible), int(st.num_intersections), self.loss, float(st.lr_mean))

    def _nccl_step(self, camera, img_size, gt_packed, splats, compute_refine_weight) -> TrainStepStats:
        self.step_count += 1
        cfg = self.config
        out = render(camera, img_size, splats.transforms, splats.sh_coeffs, splats.raw_opacities,
                     splats.render_mode, cfg.background_color, _lib.PASS_BACKWARD)
        ssim_w = cfg.ssim_weight
        lcfg = ImageLossConfig(l1_weight=1.0 - ssim_w, ssim_weight=-ssim_w) if ssim_w > 0 else ImageLossConfig(1.0, 0.0)
        if self.v_output is None or self.v_output.shape != out.out_img.shape:
            self.v_output = torch.empty_like(out.out_img)
        image_loss_fused(out.out_img, gt_packed, lcfg, self.loss, self.v_output)
        rasterize_bwd(self.v_output, compute_refine_weight, self.v_combined)
        project_bwd(self.v_combined, self.n, self.c, self.grads)
        n, c = self.n, self.c
        full_params = (splats.transforms, splats.sh_coeffs.view(n, 3 * c), splats.raw_opacities.view(n, 1))
        full_grads = (self.grads.v_transforms, self.grads.v_coeffs.view(n, 3 * c), self.grads.v_raw_opac.view(n, 1))
        if self.sharded:
            reduce_scatter_rows(full_grads, self.shard_grads, self.pg)
            if self.record is not None:
                torch.distributed.all_reduce(self.grads.v_refine_weight, op=torch.distributed.ReduceOp.MAX,
                                             group=self.pg)
            grad_scale = 1.0 / self.world
            params = tuple(p[self.row0:self.row1] for p in full_params)
            grads = self.shard_grads
        else:
            grad_scale = reduce_gradients(self.flat_grad,
                                          self.grads.v_refine_weight if self.record is not None else None, self.pg)
            params, grads = full_params, full_grads
        lr_t, tscale, lr_sh, sh_cols, lr_op, lr_mean = self._lr_table()
        if self.groups is None:
            self.groups = [AdamGroup(params[0], grads[0], lr_t),
                           AdamGroup(params[1], grads[1], lr_sh, reduce_moment_2=True),
                           AdamGroup(params[2], grads[2], lr_op)]
        g0, g1, g2 = self.groups
        g0.param, g1.param, g2.param = params
        g0.grad, g1.grad, g2.grad = grads
        g0.lr, g0.col_scale = lr_t, tscale
        g1.lr, g1.col_scale = lr_sh, sh_cols
        g2.lr = lr_op
        self.adam.step(self.groups, grad_scale=grad_scale)
        if self.sharded:
            all_gather_rows(full_params, self.pg, self.rank, self.world)
        if self.record is not None:
            self.record.gather_stats(self.grads.v_refine_weight if compute_refine_weight else None, out.aux.visible,
                                     out.aux.max_radius)
        self._mean_noise(splats, out.aux.visible, lr_mean)
        return TrainStepStats(out.aux.num_visible, out.aux.num_intersections, self.loss, lr_mean)

    def _mean_noise(self, splats: Splats, visible: torch.Tensor, lr_mean: float) -> None:
        """The mean-noise step after the optimizer (train.rs:1095-1169) through the operator
        bsx_mean_noise_step; every rank gates on the MAX of the ranks' gates, so replicas agree."""
        cfg = self.config
        ms = np.float32(self.median_scale)
        if not cfg.mean_noise or not (np.isfinite(ms) and ms > 0):
            return
        if cfg.mrnf_noise_injection and self.record is not None:
            gate = (self.record.vis_weight > 0).float()
        else:
            gate = visible.clone()
        if self.world > 1:
            torch.distributed.all_reduce(gate, op=torch.distributed.ReduceOp.MAX, group=self.pg)
        scale = np.float32(np.float32(lr_mean) * np.float32(cfg.mean_noise_weight))
        ctx = context(splats.transforms.device)
        ctx.check(_lib.lib().bsx_mean_noise_step(ctx.handle, ptr(splats.transforms), ptr(splats.raw_opacities),
                                                 ptr(gate), self.n, float(scale), float(ms), int(cfg.noise_seed),
                                                 int(self.step_count)))

    def reserve(self, max_splats: int, splats: Splats) -> None:
        """Allocate up front for a run that grows to ``max_splats`` (single-GPU native trainer):
        the trainer's and context's per-splat buffers and the refine output storages."""
        if self.native is None or self.world > 1:
            raise NotImplementedError("reserve applies to the single-GPU native trainer")
        ctx = context(splats.transforms.device)
        ctx.check(_lib.lib().bsx_trainer_reserve(self.native.handle, int(max_splats)))
        dev = splats.transforms.device
        self._store = [tuple(torch.empty(shape, device=dev) for shape in
                             ((max_splats, 10), (max_splats, self.c, 3), (max_splats,))) for _ in range(2)]
        self._store_next = 0

    def _refine_storage(self, n2: int, splats: Splats):
        """Output splat tensors for a refine: views of one of two storages used in turn (the
        other holds the splats being refined), each grown with headroom, so a growing run
        does not allocate at every refine. The splat tensors from before a refine are
        overwritten by the refine after next."""
        dev = splats.transforms.device
        if not hasattr(self, "_store"):
            self._store, self._store_next = [None, None], 0
        k = self._store_next
        if self._store[k] is not None and splats.transforms.data_ptr() == self._store[k][0].data_ptr():
            k ^= 1  # never write into the storage being read
        buf = self._store[k]
        if buf is None or buf[0].shape[0] < n2:
            cap = max(n2, int(n2 * 1.5))
            buf = (torch.empty((cap, 10), device=dev), torch.empty((cap, self.c, 3), device=dev),
                   torch.empty((cap,), device=dev))
            self._store[k] = buf
        self._store_next = k ^ 1
        return buf[0][:n2], buf[1][:n2], buf[2][:n2]

    def refine(self, splats: Splats, global_iter: int, phase_iter: int | None = None, phase_total: int | None = None,
               refine_config: RefineConfig | None = None) -> _lib.RefineStats:
        """``SplatTrainer::refine_for_phase`` (crates/brush-train/src/train.rs:1191-1534) in place on
        ``splats``: prune, replace, split oversized, grow by gradient; the splat tensors are
        replaced by tensors of the new count and the optimizer state follows the rows."""
        if self.native is None:
            raise NotImplementedError("refine runs on the native trainer (one GPU, or the peer exchange)")
        cfg = refine_config or RefineConfig()
        if self.world > 1:
            self._gather_for_refine()
        phase_iter = global_iter if phase_iter is None else phase_iter
        phase_total = self.config.total_train_iters if phase_total is None else phase_total
        L = _lib.lib()
        ctx = context(splats.transforms.device)
        center = (C.c_float * 3)(*[float(v) for v in self.bounds[0]])
        extent = (C.c_float * 3)(*[float(v) for v in self.bounds[1]])
        st = _lib.RefineStats()
        c = cfg.to_c()
        ctx.check(L.bsx_trainer_refine_plan(self.native.handle, ptr(splats.transforms), ptr(splats.sh_coeffs),
                                            ptr(splats.raw_opacities), C.byref(c), center, extent, int(global_iter),
                                            C.byref(st)))
        n2 = int(st.total_splats)
        nt, nsh, nop = self._refine_storage(n2, splats)
        ctx.check(L.bsx_trainer_refine_apply(self.native.handle, ptr(splats.transforms), ptr(splats.sh_coeffs),
                                             ptr(splats.raw_opacities), ptr(nt), ptr(nsh), ptr(nop),
                                             int(phase_iter), int(phase_total)))
        splats.transforms, splats.sh_coeffs, splats.raw_opacities = nt, nsh, nop
        self.n = n2
        self.native.n = n2
        self.record = self.native.record()
        if self.world > 1:
            self._reshard_after_refine(splats)
        else:
            self.grads = self.native.grads()
        # new bounds and rate scale (train.rs:1506, :656)
        self.bounds = splat_bounds(splats.means(), self.config.bounds_percentile)
        self.median_scale = float(np.float32(np.sort(self.bounds[1])[1] * np.float32(2.0)))
        ctx.check(L.bsx_trainer_set_median_scale(self.native.handle, self.median_scale))
        return st

    def _gather_for_refine(self) -> None:
        """Every rank refines the same model identically: combine the ranks' statistics
        (visibility SUM, screen size MAX; the refine weights are already MAX-combined by the
        exchange) and give every rank the full optimizer state (all-gather of the row shards)."""
        rec = self.record
        torch.distributed.all_reduce(rec.vis_weight, op=torch.distributed.ReduceOp.SUM, group=self.pg)
        if self.config.accumulate_grad2d:
            torch.distributed.all_reduce(rec.grad2d_accum, op=torch.distributed.ReduceOp.SUM, group=self.pg)
        torch.distributed.all_reduce(rec.max_screen_size, op=torch.distributed.ReduceOp.MAX, group=self.pg)
        state = self.native.optimizer_state()
        n, w = self.n, self.world
        if state is None:
            return
        bounds = [n * r // w for r in range(w + 1)]
        pad = max(bounds[r + 1] - bounds[r] for r in range(w))
        full = []
        for t in (*state[0], *state[1]):
            flat = t.reshape(t.shape[0], -1)
            mine = torch.zeros((pad, flat.shape[1]), device=flat.device)
            mine[:flat.shape[0]] = flat
            gathered = torch.empty((w * pad, flat.shape[1]), device=flat.device)
            torch.distributed.all_gather_into_tensor(gathered, mine, group=self.pg)
            rows = [gathered[r * pad: r * pad + bounds[r + 1] - bounds[r]] for r in range(w)]
            full.append(torch.cat(rows, 0).reshape((n,) + tuple(t.shape[1:])))
        self.native.load_optimizer_state(full[:3], full[3:], n, 1, 0)

    def _reshard_after_refine(self, splats: Splats) -> None:
        """After a data-parallel refine: a new exchange region for the new count, the splats
        copied into it, and this rank's row shard of the (full, refined) optimizer state."""
        from .peer import PeerExchange

        old = self.peer
        self.peer = PeerExchange(self.n, self.c, splats.transforms.device.index, self.pg,
                                 multicast=self.exchange == "nvls")
        self.peer.load(splats.transforms, splats.sh_coeffs, splats.raw_opacities)
        splats.transforms, splats.sh_coeffs, splats.raw_opacities = self.peer.params
        self.grads = SplatGrads(*self.peer.grads, v_refine_weight=self.peer.refine)
        self._dp = self.peer.train_structs()
        old.close()
        state = self.native.optimizer_state()
        if state is not None:
            rank = torch.distributed.get_rank(self.pg)
            r0, r1 = self.n * rank // self.world, self.n * (rank + 1) // self.world
            shard = [t[r0:r1].clone() for t in (*state[0], *state[1])]
            self.native.load_optimizer_state(shard[:3], shard[3:], r1 - r0, self.world, rank)

    def close(self) -> None:
        """Release the exchange region (collective over the process group) and the native trainer."""
        if self.peer is not None:
            self.peer.close()
            self.peer = None
        if self.native is not None:
            self.native.close()
            self.native = None

"""Training step, mirroring ``SplatTrainer::step_with_refine_weight``
(crates/brush-train/src/train.rs:619-1182).

One step: backward-pass render -> fused SSIM+L1 loss and its gradient ->
raster backward -> projection backward -> fused AdamScaled over transforms /
SH / opacity with the reference's learning-rate table (train.rs:964-1051) ->
refine statistics (stats.rs:111-121). With several ranks (one view each) the
gradient exchange and Adam are one peer-memory kernel (brush_b200.peer), or
NCCL collectives around the fused Adam (brush_b200.dist).

Not applied: the reference's random mean-noise injection after Adam
(train.rs:1095-1169); it draws from a non-reproducible RNG stream and is
outside the parity contract.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import torch

from . import _lib
from .adam import AdamGroup, AdamScaled
from .camera import Camera
from .dist import all_gather_rows, reduce_gradients, reduce_scatter_rows, row_shard
from .loss import ImageLossConfig, image_loss_fused
from .render import render
from .render_bwd import SplatGrads, project_bwd, rasterize_bwd
from .splats import Splats, median_size


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


@dataclass
class TrainStepStats:
    num_visible: int
    num_intersections: int
    loss: torch.Tensor  # device scalar
    lr_mean: float


@dataclass
class RefineRecord:
    """``RefineRecord`` statistics (crates/brush-train/src/stats.rs:11-127)."""
    refine_weight_norm: torch.Tensor
    vis_weight: torch.Tensor
    max_screen_size: torch.Tensor

    @staticmethod
    def new(n: int, device) -> "RefineRecord":
        z = lambda: torch.zeros(n, device=device)
        return RefineRecord(z(), z(), z())

    def gather_stats(self, refine_weight, visible, screen_radius) -> None:
        torch.maximum(self.refine_weight_norm, refine_weight, out=self.refine_weight_norm)
        self.vis_weight.add_(visible)
        torch.maximum(self.max_screen_size, screen_radius, out=self.max_screen_size)


class SplatTrainer:
    def __init__(self, config: TrainConfig, splats: Splats, process_group=None, gather_stats: bool = True,
                 shard_optimizer: bool = True, exchange: str = "peer"):
        self.config = config
        # Data-parallel exchange with several ranks:
        #   "peer": one fused kernel over peer memory (brush_b200.peer); the
        #           splat parameters then live in the exchange region and the
        #           tensors of ``splats`` are rebound to it.
        #   "nccl": with shard_optimizer and N divisible by the world size,
        #           reduce-scatter gradients -> fused Adam on this rank's row
        #           shard -> all-gather; otherwise all-reduce -> full Adam.
        if exchange not in ("peer", "nccl"):
            raise ValueError("exchange must be 'peer' or 'nccl'")
        self.exchange = exchange
        self.peer = None
        self.shard_optimizer = shard_optimizer
        self.adam = AdamScaled(epsilon=1e-15)
        self.step_count = 0
        self.pg = process_group
        self.world = 1 if process_group is None else torch.distributed.get_world_size(process_group)
        self.gather_stats = gather_stats
        self.median_scale = median_size(splats.means(), config.bounds_percentile)
        t = max(config.total_train_iters, 1)
        self.mean_decay = (config.lr_mean_end / config.lr_mean) ** (1.0 / t)
        self.scale_decay = ((config.lr_scale_end / config.lr_scale) ** (1.0 / t)
                            if config.lr_scale > 0 and config.lr_scale_end > 0 else 1.0)
        self._alloc(splats)

    def _alloc(self, splats: Splats) -> None:
        n, c = splats.num_splats, splats.sh_coeffs_per_splat
        dev = splats.transforms.device
        self.n, self.c = n, c
        use_peer = self.world > 1 and self.exchange == "peer"
        if not use_peer:
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
        self.loss = torch.empty(1, device=dev)
        self.v_output = None
        self.record = RefineRecord.new(n, dev) if self.gather_stats else None
        self.groups = None
        old, self.peer = self.peer, None
        if use_peer:
            from .peer import PeerExchange

            self.peer = PeerExchange(n, c, dev.index, self.pg)
            self.peer.load(splats.transforms, splats.sh_coeffs, splats.raw_opacities)
            splats.transforms, splats.sh_coeffs, splats.raw_opacities = self.peer.params
            self.grads = SplatGrads(*self.peer.grads, v_refine_weight=self.peer.refine)
            self.flat_grad = None
        if old is not None:
            old.close()
        self.sharded = (self.peer is None and self.shard_optimizer and self.world > 1 and n % self.world == 0)
        if self.sharded:
            self.rank = torch.distributed.get_rank(self.pg)
            self.row0, self.row1 = row_shard(n, self.world, self.rank)
            r = self.row1 - self.row0
            self.shard_grads = (torch.empty((r, 10), device=dev), torch.empty((r, 3 * c), device=dev),
                                torch.empty((r, 1), device=dev))

    def _lr_table(self):
        cfg = self.config
        k = self.step_count
        if cfg.uniform_lr is not None:
            return cfg.uniform_lr, None, cfg.uniform_lr, None, cfg.uniform_lr, cfg.uniform_lr
        lr_mean = cfg.lr_mean * self.mean_decay ** k * self.median_scale
        lr_scale = cfg.lr_scale * self.scale_decay ** k
        tscale = [lr_mean] * 3 + [cfg.lr_rotation] * 4 + [lr_scale] * 3
        sh_scale = [1.0] + [1.0 / cfg.lr_coeffs_sh_scale] * (self.c - 1)
        sh_cols = [s for s in sh_scale for _ in range(3)]
        return 1.0, tscale, cfg.lr_coeffs_dc, sh_cols, cfg.lr_opac, lr_mean

    def step(self, camera: Camera, img_size: tuple, gt_packed: torch.Tensor, splats: Splats,
             compute_refine_weight: bool = True) -> TrainStepStats:
        """One optimisation step in place on ``splats`` (device tensors)."""
        if splats.num_splats != self.n or splats.sh_coeffs_per_splat != self.c:
            self._alloc(splats)
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
        if self.peer is not None:
            lr_t, tscale, lr_sh, sh_cols, lr_op, lr_mean = self._lr_table()
            with_refine = self.record is not None and compute_refine_weight
            self.peer.adam_step(self.adam, [(lr_t, tscale, False), (lr_sh, sh_cols, True), (lr_op, None, False)],
                                1.0 / self.world, with_refine)
            if with_refine:
                self.record.gather_stats(self.grads.v_refine_weight, out.aux.visible, out.aux.max_radius)
            return TrainStepStats(out.aux.num_visible, out.aux.num_intersections, self.loss, lr_mean)
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
            if compute_refine_weight:
                self.record.gather_stats(self.grads.v_refine_weight, out.aux.visible, out.aux.max_radius)
        return TrainStepStats(out.aux.num_visible, out.aux.num_intersections, self.loss, lr_mean)

    def close(self) -> None:
        """Release the data-parallel exchange region (collective over the process group)."""
        if self.peer is not None:
            self.peer.close()
            self.peer = None

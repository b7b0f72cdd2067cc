"""Data-parallel exchange for the training step (one process per GPU).

Views are sharded across ranks, splats are replicated. Each rank computes the
gradient of its own view into one flat buffer; one all-reduce (SUM) per step
combines them and the optimizer applies ``1/world`` so the update uses the
mean-of-views gradient. Refine weights are combined with MAX so densification
decisions are identical on every rank. The reference trains one view per step
on one device (crates/brush-process/src/train_stream.rs:449-465); with one
rank this module is a no-op.
"""
from __future__ import annotations

import torch


def view_for(step: int, rank: int, world: int, num_views: int) -> int:
    """View trained by ``rank`` at ``step``: ranks take consecutive views, round-robin."""
    return (step * world + rank) % num_views


def reduce_gradients(flat_grad: torch.Tensor, refine_weight: torch.Tensor | None, group=None) -> float:
    """SUM-all-reduce the flat gradient (MAX for refine weights); return the Adam grad scale."""
    if group is None or not torch.distributed.is_initialized():
        return 1.0
    world = torch.distributed.get_world_size(group)
    if world == 1:
        return 1.0
    torch.distributed.all_reduce(flat_grad, op=torch.distributed.ReduceOp.SUM, group=group)
    if refine_weight is not None:
        torch.distributed.all_reduce(refine_weight, op=torch.distributed.ReduceOp.MAX, group=group)
    return 1.0 / world


def splat_checksum(*tensors: torch.Tensor) -> torch.Tensor:
    """Order-independent float64 checksum of the replicated splats (consistency probe)."""
    acc = torch.zeros((), dtype=torch.float64, device=tensors[0].device)
    for t in tensors:
        acc = acc + t.double().sum() + (t.double() * torch.arange(t.numel(), device=t.device,
                                                                  dtype=torch.float64).view(t.shape) % 7).sum()
    return acc


def replicas_agree(group, *tensors: torch.Tensor, tol: float = 0.0) -> bool:
    """True when every rank holds the same splats (max - min of the checksum <= tol)."""
    c = splat_checksum(*tensors).reshape(1)
    lo, hi = c.clone(), c.clone()
    torch.distributed.all_reduce(lo, op=torch.distributed.ReduceOp.MIN, group=group)
    torch.distributed.all_reduce(hi, op=torch.distributed.ReduceOp.MAX, group=group)
    return float(hi - lo) <= tol


def row_shard(n: int, world: int, rank: int) -> tuple[int, int]:
    """Rows [start, end) of every parameter owned by ``rank`` (requires n % world == 0)."""
    rows = n // world
    return rank * rows, (rank + 1) * rows


def _coalesced(group, fn):
    """Issue the collectives ``fn`` enqueues as one NCCL group where supported."""
    backend = torch.distributed.get_backend(group)
    if backend == "nccl":
        with torch.distributed._coalescing_manager(group=group):
            fn()
    else:
        fn()


def reduce_scatter_rows(fulls, shards, group) -> None:
    """SUM-reduce row-sharded tensors: shards[i] <- rows of this rank of sum over ranks of fulls[i]."""
    def run():
        for f, s in zip(fulls, shards):
            torch.distributed.reduce_scatter_tensor(s, f, op=torch.distributed.ReduceOp.SUM, group=group)
    _coalesced(group, run)


def all_gather_rows(fulls, group, rank: int, world: int) -> None:
    """In-place all-gather: every rank's row shard of each tensor is copied to all ranks."""
    def run():
        for f in fulls:
            rows = f.shape[0] // world
            torch.distributed.all_gather_into_tensor(f, f[rank * rows:(rank + 1) * rows], group=group)
    _coalesced(group, run)

"""GPU primitives, mirroring brush-sort (``radix_argsort``, crates/brush-sort/src/lib.rs:16-129),
brush-prefix-sum (``prefix_sum``, crates/brush-prefix-sum/src/lib.rs:11-87) and
``get_tile_offsets`` (crates/brush-render/src/get_tile_offset.rs:10-62).
u32 data travel as int32 tensors (same bits)."""
from __future__ import annotations

import torch

from . import _lib
from ._context import context, ptr


def _u32(t: torch.Tensor) -> torch.Tensor:
    if t.dtype not in (torch.int32, torch.uint32):
        raise ValueError("expected int32/uint32 tensor")
    return t.contiguous()


def radix_argsort(keys: torch.Tensor, values: torch.Tensor, sorting_bits: int):
    """Stable sort of (keys, values) by keys & mask(ceil4(bits)); inputs untouched."""
    keys, values = _u32(keys), _u32(values)
    if keys.shape != values.shape or keys.dim() != 1:
        raise ValueError("keys and values must be 1-D and equal length")
    ctx = context(keys.device.index)
    ko, vo = torch.empty_like(keys), torch.empty_like(values)
    ctx.check(_lib.lib().bsx_radix_argsort_u32(ctx.handle, ptr(keys), ptr(values), keys.numel(), int(sorting_bits),
                                               ptr(ko), ptr(vo)))
    return ko, vo


def prefix_sum(values: torch.Tensor) -> torch.Tensor:
    """Inclusive u32 prefix sum (wrapping)."""
    values = _u32(values)
    ctx = context(values.device.index)
    out = torch.empty_like(values)
    ctx.check(_lib.lib().bsx_prefix_sum_u32(ctx.handle, ptr(values), values.numel(), ptr(out)))
    return out


def get_tile_offsets(tile_ids: torch.Tensor, num_tiles: int) -> torch.Tensor:
    """[num_tiles, 2] start/end of each tile's run in sorted ``tile_ids``."""
    tile_ids = _u32(tile_ids)
    ctx = context(tile_ids.device.index)
    out = torch.empty((num_tiles, 2), dtype=torch.int32, device=tile_ids.device)
    ctx.check(_lib.lib().bsx_get_tile_offsets(ctx.handle, ptr(tile_ids), tile_ids.numel(), num_tiles, ptr(out)))
    return out

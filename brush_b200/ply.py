"""Splat PLY import and export, mirroring crates/brush-serde: ``load_splat_from_ply``
(src/import.rs:167-178) and ``splat_to_ply`` (src/export.rs:170-191).

The header is parsed on the host; the rows are decoded on the GPU straight into
the splat tensors (``bsx_ply_parse`` / ``bsx_ply_load``), and export encodes the
rows on the GPU (``bsx_ply_export``). Errors in the file raise ``BsxError`` with
status ``BSX_ERR_FORMAT`` and the reference's message.
"""
from __future__ import annotations

import ctypes as C
import os
from dataclasses import dataclass
from typing import BinaryIO, Optional, Sequence, Union

import torch

from . import _lib
from ._context import context, ptr
from .splats import Splats


@dataclass
class ParseMetadata:
    """ParseMetadata (import.rs:18-24)."""
    up_axis: Optional[tuple]       # from a "Vertical axis:" comment
    render_mode: Optional[int]     # RENDER_DEFAULT / RENDER_MIP from "SplatRenderMode:", else None
    total_splats: int              # rows kept after subsampling
    progress: float = 1.0


@dataclass
class SplatMessage:
    """SplatMessage (import.rs:97-100) with the data already on the device as Splats."""
    meta: ParseMetadata
    splats: Splats
    compressed: bool = False


def _read_bytes(source) -> bytes:
    if isinstance(source, (bytes, bytearray, memoryview)):
        return bytes(source)
    if isinstance(source, (str, os.PathLike)):
        with open(source, "rb") as fh:
            return fh.read()
    return source.read()


def load_splat_from_ply(source: Union[bytes, str, os.PathLike, BinaryIO], subsample_points: Optional[int] = None,
                        device: Union[str, torch.device] = "cuda") -> SplatMessage:
    """Decode a PLY (standard 3DGS properties, RGB colours, or the SuperSplat compressed
    layout) into device-resident Splats. ``subsample_points`` keeps every k-th row."""
    data = _read_bytes(source)
    sub = 1 if subsample_points is None else int(subsample_points)
    buf = (C.c_uint8 * max(len(data), 1)).from_buffer_copy(data if data else b"\0")
    info = _lib.PlyInfo()
    handle = C.c_void_p()
    err = C.create_string_buffer(512)
    L = _lib.lib()
    status = L.bsx_ply_parse(buf, len(data), sub, C.byref(handle), C.byref(info), err, len(err))
    if status != 0:
        msg = err.value.decode() or L.bsx_status_string(status).decode()
        raise _lib.BsxError(status, msg)
    try:
        dev = torch.device(device)
        if dev.type != "cuda":
            raise ValueError("PLY decoding runs on the GPU: pass a CUDA device")
        n, c = int(info.num_splats), int(info.sh_coeffs)
        t = torch.empty((n, 10), dtype=torch.float32, device=dev)
        sh = torch.empty((n, c, 3), dtype=torch.float32, device=dev)
        op = torch.empty((n,), dtype=torch.float32, device=dev)
        ctx = context(dev)
        ctx.bind_stream()
        ctx.check(L.bsx_ply_load(ctx.handle, handle, ptr(t), ptr(sh), ptr(op)))
        ctx.sync()  # the upload reads `buf`
    finally:
        L.bsx_ply_free(handle)
    up = tuple(float(v) for v in info.up_axis) if info.has_up_axis else None
    mode = None if info.render_mode < 0 else int(info.render_mode)
    meta = ParseMetadata(up_axis=up, render_mode=mode, total_splats=n)
    return SplatMessage(meta, Splats(t, sh, op, mode or 0), bool(info.compressed))


def splat_to_ply(splats: Splats, up_axis: Optional[Sequence[float]] = None, mip: Optional[bool] = None) -> bytes:
    """The binary little-endian PLY of ``splats`` (quaternions normalised, SH rest in the
    3DGS channel-major order), with the reference's header comments."""
    t = splats.transforms.detach().float().contiguous()
    sh = splats.sh_coeffs.detach().float().contiguous()
    op = splats.raw_opacities.detach().float().contiguous()
    if t.device.type != "cuda":
        raise ValueError("PLY export runs on the GPU: move the splats to a CUDA device")
    n, c = int(t.shape[0]), int(sh.shape[1])
    render_mip = bool(splats.render_mode == _lib.RENDER_MIP) if mip is None else bool(mip)
    up = (C.c_float * 3)(*[float(v) for v in up_axis]) if up_axis is not None else None
    L = _lib.lib()
    size = C.c_uint64()
    status = L.bsx_ply_export_size(n, c, int(render_mip), up, C.byref(size))
    if status != 0:
        raise _lib.BsxError(status, f"cannot export {c} SH coefficients per channel (degrees 0-3)")
    out = (C.c_uint8 * int(size.value))()
    written = C.c_uint64()
    ctx = context(t.device)
    ctx.bind_stream()
    ctx.check(L.bsx_ply_export(ctx.handle, ptr(t), ptr(sh), ptr(op), n, c, int(render_mip), up, out,
                               size.value, C.byref(written)))
    return bytes(out)[: int(written.value)]

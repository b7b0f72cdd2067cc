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

import numpy as np
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


def _host_view(source):
    """(keep-alive object, address, length) of the file bytes without copying them
    where possible: bytes, bytearray, a uint8 numpy array or a CPU uint8 tensor (pinned
    memory makes the upload asynchronous); paths and readers are read once."""
    if isinstance(source, (str, os.PathLike)):
        with open(source, "rb") as fh:
            source = fh.read()
    elif hasattr(source, "read"):
        source = source.read()
    if isinstance(source, memoryview):
        source = source.tobytes()
    if isinstance(source, bytes):
        return source, C.cast(C.c_char_p(source), C.c_void_p).value, len(source)
    if isinstance(source, bytearray):
        buf = (C.c_uint8 * max(len(source), 1)).from_buffer(source) if source else None
        return (source, buf), (C.addressof(buf) if buf is not None else None), len(source)
    if isinstance(source, torch.Tensor):
        if source.device.type != "cpu" or source.dtype != torch.uint8 or not source.is_contiguous():
            raise ValueError("expected a contiguous CPU uint8 tensor of file bytes")
        return source, source.data_ptr(), source.numel()
    arr = np.ascontiguousarray(np.asarray(source, dtype=np.uint8))
    return arr, arr.ctypes.data, arr.size


def load_splat_from_ply(source: Union[bytes, str, os.PathLike, BinaryIO], subsample_points: Optional[int] = None,
                        device: Union[str, torch.device] = "cuda") -> SplatMessage:
    """Decode a PLY (standard 3DGS properties, RGB colours, or the SuperSplat compressed
    layout) into device-resident Splats. ``subsample_points`` keeps every k-th row."""
    keep, addr, size = _host_view(source)
    sub = 1 if subsample_points is None else int(subsample_points)
    info = _lib.PlyInfo()
    handle = C.c_void_p()
    err = C.create_string_buffer(512)
    L = _lib.lib()
    status = L.bsx_ply_parse(addr, size, sub, C.byref(handle), C.byref(info), err, len(err))
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
        ctx.sync()  # the upload reads the caller's bytes
    finally:
        L.bsx_ply_free(handle)
    up = tuple(float(v) for v in info.up_axis) if info.has_up_axis else None
    mode = None if info.render_mode < 0 else int(info.render_mode)
    meta = ParseMetadata(up_axis=up, render_mode=mode, total_splats=n)
    return SplatMessage(meta, Splats(t, sh, op, mode or 0), bool(info.compressed))


def splat_to_ply(splats: Splats, up_axis: Optional[Sequence[float]] = None, mip: Optional[bool] = None) -> bytes:
    """The binary little-endian PLY of ``splats`` (quaternions normalised, SH rest in the
    3DGS channel-major order), with the reference's header comments."""
    size = export_size(splats, up_axis, mip)
    out = bytearray(size)
    n = export_into(splats, out, up_axis, mip)
    return bytes(memoryview(out)[:n])


def export_size(splats: Splats, up_axis: Optional[Sequence[float]] = None, mip: Optional[bool] = None) -> int:
    """Bytes of ``splat_to_ply(splats, ...)``."""
    c = int(splats.sh_coeffs.shape[1])
    render_mip = bool(splats.render_mode == _lib.RENDER_MIP) if mip is None else bool(mip)
    up = (C.c_float * 3)(*[float(v) for v in up_axis]) if up_axis is not None else None
    size = C.c_uint64()
    status = _lib.lib().bsx_ply_export_size(splats.num_splats, c, int(render_mip), up, C.byref(size))
    if status != 0:
        raise _lib.BsxError(status, f"cannot export {c} SH coefficients per channel (degrees 0-3)")
    return int(size.value)


def export_into(splats: Splats, out, up_axis: Optional[Sequence[float]] = None, mip: Optional[bool] = None) -> int:
    """Writes the PLY into ``out`` (a bytearray, uint8 numpy array or CPU uint8 tensor,
    pinned memory for an asynchronous read-back) and returns its length."""
    t = splats.transforms.detach().float().contiguous()
    sh = splats.sh_coeffs.detach().float().contiguous()
    op = splats.raw_opacities.detach().float().contiguous()
    if t.device.type != "cuda":
        raise ValueError("PLY export runs on the GPU: move the splats to a CUDA device")
    n, c = int(t.shape[0]), int(sh.shape[1])
    render_mip = bool(splats.render_mode == _lib.RENDER_MIP) if mip is None else bool(mip)
    up = (C.c_float * 3)(*[float(v) for v in up_axis]) if up_axis is not None else None
    keep, addr, cap = _host_view(out)
    written = C.c_uint64()
    ctx = context(t.device)
    ctx.bind_stream()
    ctx.check(_lib.lib().bsx_ply_export(ctx.handle, ptr(t), ptr(sh), ptr(op), n, c, int(render_mip), up, addr,
                                        cap, C.byref(written)))
    return int(written.value)

"""Per-device bsx context and zero-copy views of library-owned device memory."""
from __future__ import annotations

import ctypes as C
import threading

import torch

from . import _lib

_CTX: dict[int, "Context"] = {}
_LOCK = threading.Lock()


class Context:
    """Owns one ``bsx_ctx`` (workspace + last-forward state) on one CUDA device."""

    def __init__(self, device: int):
        self.device = device
        h = C.c_void_p()
        with torch.cuda.device(device):
            _lib.check(_lib.lib().bsx_create(device, C.byref(h)))
        self.handle = h
        self.last_n = 0  # splat count of the last forward render
        self.fwd_inputs = ()  # splat tensors of the last forward render (read by the backward)

    def bind_stream(self) -> None:
        """Enqueue subsequent library work on torch's current stream of this device."""
        s = torch.cuda.current_stream(self.device).cuda_stream
        _lib.check(_lib.lib().bsx_set_stream(self.handle, C.c_void_p(s)), self.handle)

    def check(self, status: int) -> None:
        _lib.check(status, self.handle)

    def launches(self) -> int:
        return int(_lib.lib().bsx_launch_count(self.handle))

    def profile(self, on: bool) -> None:
        """Bracket every kernel launch with CUDA events on the bound stream."""
        self.check(_lib.lib().bsx_profile_enable(self.handle, int(on)))

    def profile_reset(self) -> None:
        self.check(_lib.lib().bsx_profile_reset(self.handle))

    def profile_read(self) -> dict:
        """{kernel name: (total ms, launches)} accumulated since the last reset."""
        L = _lib.lib()
        self.check(L.bsx_profile_collect(self.handle))
        out = {}
        for i in range(L.bsx_profile_count(self.handle)):
            name, ms, cnt = C.c_char_p(), C.c_double(), C.c_uint64()
            self.check(L.bsx_profile_entry(self.handle, i, C.byref(name), C.byref(ms), C.byref(cnt)))
            out[name.value.decode()] = (ms.value, int(cnt.value))
        return out

    def trim(self) -> None:
        """Release the grow-only workspace (reallocated on demand)."""
        self.check(_lib.lib().bsx_trim(self.handle))

    def sync(self) -> None:
        self.check(_lib.lib().bsx_sync(self.handle))


def context(device: torch.device | int | None = None) -> Context:
    if device is None:
        idx = torch.cuda.current_device()
    elif isinstance(device, torch.device):
        idx = device.index if device.index is not None else torch.cuda.current_device()
    else:
        idx = int(device)
    with _LOCK:
        ctx = _CTX.get(idx)
        if ctx is None:
            ctx = Context(idx)
            _CTX[idx] = ctx
    ctx.bind_stream()
    return ctx


class _DeviceArray:
    """Minimal ``__cuda_array_interface__`` exporter for a raw device pointer."""

    def __init__(self, ptr: int, shape: tuple, typestr: str):
        self.__cuda_array_interface__ = {
            "shape": tuple(int(s) for s in shape),
            "typestr": typestr,
            "data": (int(ptr), False),
            "version": 3,
            "strides": None,
            "stream": None,
        }


_TYPESTR = {torch.float32: "<f4", torch.int32: "<i4"}


def device_view(ptr: int | None, shape: tuple, dtype: torch.dtype, device: int) -> torch.Tensor:
    """A tensor aliasing library-owned memory (valid until the next call that reuses it)."""
    n = 1
    for s in shape:
        n *= int(s)
    if not ptr or n == 0:
        return torch.empty(shape, dtype=dtype, device=f"cuda:{device}")
    return torch.as_tensor(_DeviceArray(ptr, shape, _TYPESTR[dtype]), device=f"cuda:{device}")


def ptr(t: torch.Tensor | None) -> C.c_void_p:
    if t is None:
        return C.c_void_p(0)
    if not t.is_cuda:
        raise ValueError("bsx entry points take CUDA tensors")
    if not t.is_contiguous():
        raise ValueError("bsx entry points take contiguous tensors")
    return C.c_void_p(t.data_ptr())

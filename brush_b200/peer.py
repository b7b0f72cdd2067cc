"""Data-parallel exchange over peer memory: one fused kernel per step.

Each rank owns one exchange region (library-allocated device memory exported
with CUDA IPC and mapped by every other rank of the node) holding the splat
parameters, their gradients, the refine weights, the mean-noise gate and the
exchange flag words.
``bsx_dp_adam_step`` then replaces "all-reduce gradients, Adam, keep replicas
in sync": rank ``r`` sums the gradient rows of its shard over every rank in
rank order, applies AdamScaled with its shard's moments, and stores the new
rows into every rank's parameters. No NCCL call is on the step path; the
process group is used only to swap IPC handles at setup and for barriers at
teardown.

The reference trains on one device (crates/brush-process/src/train_stream.rs:449-465);
the exchange is this library's addition.
"""
from __future__ import annotations

import ctypes as C

import torch

from . import _lib
from ._context import context, device_view

_ALIGN = 64  # floats (256 bytes) between sub-buffers


def _up(x: int) -> int:
    return (x + _ALIGN - 1) // _ALIGN * _ALIGN


def shard_rows(rows: int, rank: int, world: int) -> tuple[int, int]:
    """Rows [begin, end) that ``rank`` owns (the kernel's split: rows*r // world)."""
    return rows * rank // world, rows * (rank + 1) // world


class ExchangeLayout:
    """Float offsets of the sub-buffers of one rank's exchange region.

    The gradient sub-buffers hold ``world`` slots of ``slot_rows`` rows (the
    largest shard, rounded up to 4 rows so that every slot starts 16-byte
    aligned): the training step's projection backward stores the rows of the
    shard that rank q owns into slot ``rank`` of rank q's region. Their first
    ``n`` rows double as a dense [n, cols] gradient for the paths that write one."""

    def __init__(self, n: int, c: int, world: int = 1):
        self.n, self.c = n, c
        widths = {"transforms": 10, "sh": 3 * c, "opac": 1}
        self.slot_rows = (-(-n // world) + 3) // 4 * 4
        grad_rows = max(n, world * self.slot_rows)
        off = 0
        self.offsets = {}
        for kind in ("param", "grad"):
            for name, w in widths.items():
                self.offsets[(kind, name)] = off
                off = _up(off + (n if kind == "param" else grad_rows) * w)
        self.offsets["refine"] = off
        off = _up(off + n)
        self.offsets["gate"] = off  # the mean-noise gate (MAX-combined like the refine weights)
        off = _up(off + n)
        self.offsets["flags"] = off
        off = _up(off + _lib.BSX_DP_FLAG_WORDS)
        self.floats = off
        self.widths = widths

    @property
    def nbytes(self) -> int:
        return 4 * self.floats


class PeerExchange:
    """This rank's exchange region, every rank's mapping of it, and the shard's Adam moments."""

    def __init__(self, n: int, c: int, device: int, group, timeout_s: float = 5.0, multicast: bool = False):
        self.group = group
        self.world = torch.distributed.get_world_size(group)
        self.rank = torch.distributed.get_rank(group)
        if self.world > _lib.BSX_MAX_RANKS:
            raise ValueError(f"the peer exchange supports at most {_lib.BSX_MAX_RANKS} ranks")
        self.device = device
        self.ctx = context(device)
        self.layout = ExchangeLayout(n, c, self.world)
        self.timeout_ns = int(timeout_s * 1e9)
        self.epoch = 0
        self.mc_base = 0
        self._symm = None
        self._opened = []
        if not (multicast and self.world > 1 and self._alloc_multicast()):
            self._alloc_ipc()
        self.params = (self._view(("param", "transforms"), (n, 10)), self._view(("param", "sh"), (n, c, 3)),
                       self._view(("param", "opac"), (n,)))
        self.grads = (self._view(("grad", "transforms"), (n, 10)), self._view(("grad", "sh"), (n, c, 3)),
                      self._view(("grad", "opac"), (n,)))
        self.refine = self._view("refine", (n,))
        self.row0, self.row1 = shard_rows(n, self.rank, self.world)
        self.m = self.v = None  # shard moments of adam_step (the native trainer keeps its own)
        self._closed = False

    def _alloc_ipc(self) -> None:
        """The region from bsx_peer_alloc, mapped by the other ranks through CUDA IPC handles."""
        L = _lib.lib()
        own = C.c_void_p()
        handle = C.create_string_buffer(_lib.BSX_PEER_HANDLE_BYTES)
        self.ctx.check(L.bsx_peer_alloc(self.ctx.handle, self.layout.nbytes, C.byref(own), handle))
        self._own = own.value
        handles = [None] * self.world
        torch.distributed.all_gather_object(handles, handle.raw, group=self.group)
        self.bases = []
        for q, h in enumerate(handles):
            if q == self.rank:
                self.bases.append(self._own)
                continue
            p = C.c_void_p()
            self.ctx.check(L.bsx_peer_open(self.ctx.handle, C.create_string_buffer(h, len(h)), C.byref(p)))
            self.bases.append(p.value)
            self._opened.append(p.value)

    def _alloc_multicast(self) -> bool:
        """The region as PyTorch symmetric memory: every rank's copy mapped on every rank, and
        one NVLink multicast mapping over all copies (NVSwitch). False, with nothing kept,
        when some rank's device offers no multicast (every rank then takes the IPC path)."""
        import torch.distributed._symmetric_memory as symm_mem

        dev = torch.device("cuda", self.device)
        t = symm_mem.empty(self.layout.floats, dtype=torch.float32, device=dev)
        hdl = symm_mem.rendezvous(t, self.group)

        def attr(name):
            v = getattr(hdl, name)
            return v() if callable(v) else v

        mc = int(attr("multicast_ptr") or 0)
        ok = torch.tensor([1 if mc else 0], dtype=torch.int32, device=dev)
        torch.distributed.all_reduce(ok, op=torch.distributed.ReduceOp.MIN, group=self.group)
        if int(ok.item()) == 0:
            torch.distributed.barrier(group=self.group)
            del hdl, t
            return False
        t.zero_()  # flag words start at zero
        torch.cuda.synchronize(self.device)
        torch.distributed.barrier(group=self.group)
        self._symm = (t, hdl)
        self._own = t.data_ptr()
        self.bases = [int(p) for p in attr("buffer_ptrs")]
        if self.bases[self.rank] != self._own:
            raise RuntimeError("symmetric memory: own buffer pointer mismatch")
        self.mc_base = mc
        return True

    def _mc(self, key) -> int:
        return self.mc_base + 4 * self.layout.offsets[key]

    def _view(self, key, shape) -> torch.Tensor:
        return device_view(self._own + 4 * self.layout.offsets[key], shape, torch.float32, self.device)

    def _ptr(self, q: int, key) -> int:
        return self.bases[q] + 4 * self.layout.offsets[key]

    def load(self, transforms: torch.Tensor, sh_coeffs: torch.Tensor, raw_opacities: torch.Tensor) -> None:
        """Copy the splats into this rank's region (every rank loads the same splats)."""
        for dst, src in zip(self.params, (transforms, sh_coeffs, raw_opacities)):
            dst.copy_(src.reshape(dst.shape))

    def adam_step(self, adam, specs, grad_scale: float, with_refine: bool) -> None:
        """One fused exchange + AdamScaled step. ``specs``: (lr, col_scale, reduce_moment_2) for
        transforms, SH rows and opacities."""
        L = _lib.lib()
        if self.m is None:
            rows, dev = self.row1 - self.row0, torch.device("cuda", self.device)
            self.m = [torch.zeros((rows, w), device=dev) for w in self.layout.widths.values()]
            self.v = [torch.zeros((rows, 10), device=dev), torch.zeros((rows,), device=dev),
                      torch.zeros((rows, 1), device=dev)]
        adam.step_count += 1
        self.epoch += 1
        ex = _lib.DpExchange()
        ex.rank, ex.world = self.rank, self.world
        for q in range(self.world):
            ex.d_flags[q] = self._ptr(q, "flags")
            ex.d_refine[q] = self._ptr(q, "refine")
        ex.refine_rows = self.layout.n if with_refine else 0
        ex.epoch = self.epoch
        ex.timeout_ns = self.timeout_ns
        arr = (_lib.DpGroup * 3)()
        keep = []
        for i, (name, (lr, col_scale, reduce)) in enumerate(zip(("transforms", "sh", "opac"), specs)):
            g = arr[i]
            for q in range(self.world):
                g.d_param[q] = self._ptr(q, ("param", name))
                g.d_grad[q] = self._ptr(q, ("grad", name))
            g.d_m = self.m[i].data_ptr()
            g.d_v = self.v[i].data_ptr()
            g.rows = self.layout.n
            g.cols = self.layout.widths[name]
            g.lr = float(lr)
            if col_scale is not None:
                sc = (C.c_float * g.cols)(*[float(s) for s in col_scale])
                keep.append(sc)
                g.h_col_scale = C.cast(sc, C.POINTER(C.c_float))
            else:
                g.h_col_scale = None
            g.reduce_moment_2 = int(reduce)
        if not specs[1][2]:
            raise ValueError("the SH group keeps a per-row second moment (reduce_moment_2)")
        cfg = _lib.AdamCfg(beta_1=adam.beta_1, beta_2=adam.beta_2, epsilon=adam.epsilon, step=adam.step_count,
                           grad_scale=float(grad_scale))
        self.ctx.check(L.bsx_dp_adam_step(self.ctx.handle, C.byref(ex), arr, 3, C.byref(cfg)))

    def train_structs(self):
        """(bsx_dp_exchange, bsx_dp_splats) describing every rank's region, for bsx_train_step_dp."""
        ex = _lib.DpExchange()
        ex.rank, ex.world = self.rank, self.world
        sp = _lib.DpSplats()
        for q in range(self.world):
            ex.d_flags[q] = self._ptr(q, "flags")
            ex.d_refine[q] = self._ptr(q, "refine")
            ex.d_gate[q] = self._ptr(q, "gate")
            sp.d_transforms[q] = self._ptr(q, ("param", "transforms"))
            sp.d_sh_coeffs[q] = self._ptr(q, ("param", "sh"))
            sp.d_raw_opac[q] = self._ptr(q, ("param", "opac"))
            sp.d_v_transforms[q] = self._ptr(q, ("grad", "transforms"))
            sp.d_v_sh_coeffs[q] = self._ptr(q, ("grad", "sh"))
            sp.d_v_raw_opac[q] = self._ptr(q, ("grad", "opac"))
        ex.refine_rows = self.layout.n
        ex.timeout_ns = self.timeout_ns
        ex.grad_slot_rows = self.layout.slot_rows
        if self.mc_base:
            # multicast form: dense gradients, reduced in the switch
            ex.grad_slot_rows = 0
            ex.d_refine_mc = self._mc("refine")
            ex.d_gate_mc = self._mc("gate")
            for kind, prefix in (("param", "mc_"), ("grad", "mc_v_")):
                for name, field in (("transforms", "transforms"), ("sh", "sh_coeffs"), ("opac", "raw_opac")):
                    setattr(sp, prefix + field, self._mc((kind, name)))
        return ex, sp

    def close(self) -> None:
        """Unmap the other ranks' regions, then free this rank's (collective)."""
        if self._closed:
            return
        self._closed = True
        torch.cuda.synchronize(self.device)
        torch.distributed.barrier(group=self.group)
        if self._symm is not None:
            # every rank has finished with every copy before any is released
            self._symm = None
            torch.cuda.synchronize(self.device)
            torch.distributed.barrier(group=self.group)
            return
        L = _lib.lib()
        for p in self._opened:
            self.ctx.check(L.bsx_peer_close(self.ctx.handle, C.c_void_p(p)))
        torch.distributed.barrier(group=self.group)
        self.ctx.check(L.bsx_peer_free(self.ctx.handle, C.c_void_p(self._own)))

"""Data-parallel training step on 2 and 4 GPUs (skipped with fewer GPUs), and the
peer-exchange kernel's single-GPU forms.

Each rank trains its own view; after one step (the fused peer-memory exchange
with the gradient rows pushed into their owners' slots, the same exchange
pulling dense gradients (keep_gradients), NCCL reduce-scatter -> sharded fused
Adam -> all-gather, or NCCL all-reduce -> fused Adam) every rank holds
identical splats, equal to the CPU oracle's step on the mean of the ranks'
views' gradients (render, loss, backward and AdamScaled restated on the CPU). The peer modes use an odd
splat count, so the shards differ in size and projection blocks straddle owner
boundaries; on 4 GPUs the gradient push is checked the same way.
"""
import datetime
import multiprocessing as mp
import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parent.parent


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _scene(dev, n=40000):
    from brush_b200.splats import clustered_scene, orbit_camera, random_gt

    splats = clustered_scene(n, 3, "cpu", seed=77).to(dev)
    w, h = 320, 256
    cams = [orbit_camera(i, 4, 8.0, w, h) for i in range(4)]
    gts = [random_gt(h, w, 90 + i, "cpu").to(dev) for i in range(4)]
    return splats, cams, (w, h), gts


def _worker(rank, world, port, q, mode):
    sys.path.insert(0, str(ROOT))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import brush_b200 as bsx
    from brush_b200.dist import view_for

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    torch.distributed.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                                         timeout=datetime.timedelta(seconds=60))
    try:
        splats, cams, size, gts = _scene(dev, _n_of(mode))
        tr = bsx.SplatTrainer(bsx.TrainConfig(uniform_lr=1e-3, mean_noise=False), splats, process_group=torch.distributed.group.WORLD,
                              gather_stats=False, shard_optimizer=mode == "sharded_adam",
                              exchange="nvls" if mode == "nvls" else "peer" if mode.startswith("peer") else "nccl",
                              keep_gradients=mode == "peer_keep")
        v = view_for(0, rank, world, len(cams))
        tr.step(cams[v], size, gts[v], splats)
        torch.cuda.synchronize()
        tr.peer and tr.peer.ctx.sync()
        q.put((rank, "ok", splats.transforms.cpu().numpy(), splats.sh_coeffs.cpu().numpy(),
               splats.raw_opacities.cpu().numpy(), (tr.peer is not None, tr.sharded),
               bool(tr.peer is not None and tr.peer.mc_base)))
        tr.close()
    except Exception as e:  # noqa: BLE001
        q.put((rank, "error", repr(e)))
    finally:
        torch.distributed.destroy_process_group()


def _n_of(mode):
    # odd counts: uneven shards, and (40003) shard starts off the 16-byte grid for the
    # multicast form's single-float path
    return 40003 if mode == "nvls" else 40001 if mode.startswith("peer") else 40000


def _oracle_mean_of_views(orc, n, world=2):
    """The CPU oracle's data-parallel step: the gradients of the ranks' views (render, 0.8 L1 +
    0.2 (1 - SSIM), raster and projection backward) summed, then AdamScaled (lr 1e-3) with the
    gradient scaled by 1/world. Returns (transforms, sh, opacities) and the summed gradients."""
    from brush_b200.dist import view_for

    splats, cams, size, gts = _scene("cpu", n)
    w, h = size
    t, sh, op = splats.transforms.numpy(), splats.sh_coeffs.numpy(), splats.raw_opacities.numpy()
    n, c = t.shape[0], sh.shape[1]
    acc = None
    oc = orc.loss_cfg(0.8, -0.2)
    for r in range(world):
        v = view_for(0, r, world, len(cams))
        rr = orc.RenderResult(cams[v], size, t, sh, op)
        chw = np.ascontiguousarray(rr.image[..., :3].transpose(2, 0, 1))
        dl = np.full((3, h, w), np.float32(1.0 / (3 * h * w)), np.float32)
        vo = np.zeros((h, w, 4), np.float32)
        vo[..., :3] = orc.loss_bwd(chw, gts[v].numpy(), oc, dl).transpose(1, 2, 0)
        vt, vs, vop, _ = rr.project_bwd(rr.rasterize_bwd(vo, False))
        parts = [vt, vs.reshape(n, 3 * c), vop.reshape(n, 1)]
        acc = parts if acc is None else [a + b for a, b in zip(acc, parts)]
    out = []
    for p, g, red in zip((t.copy(), sh.reshape(n, 3 * c).copy(), op.reshape(n, 1).copy()), acc, (False, True, False)):
        orc.adam(p, g, np.zeros_like(p), np.zeros(n, np.float32) if red else np.zeros_like(p), 1e-3, None, red,
                 grad_scale=1.0 / world)
        out.append(p)
    return (out[0], out[1].reshape(n, c, 3), out[2].reshape(n)), acc


def _assert_close_to_oracle_step(got, ref, grads, lr=1e-3):
    """Every element: within 1e-4 of the oracle's step, except where the oracle's summed
    gradient is within the 1e-3 gradient tolerance of zero, where Adam's first update
    (lr * g / (|g| + eps), or g / rms(row) for the SH rows) may point the other way."""
    n = ref[0].shape[0]
    for k, (a, b, g) in enumerate(zip(got, ref, grads)):
        a = a.reshape(n, -1).astype(np.float64)
        b = b.reshape(n, -1).astype(np.float64)
        g = np.abs(g.reshape(n, -1).astype(np.float64))
        if k == 1:
            rms = np.sqrt((g * g).mean(axis=1, keepdims=True))
            small = np.broadcast_to(rms <= 1e-3 * rms.max(), a.shape)
            allow = np.where(small, 2.0 * lr * np.sqrt(a.shape[1]) * 1.001, 1e-4)
        else:
            small = g <= 1e-3 * g.max(axis=0, keepdims=True)
            allow = np.where(small, 2.0 * lr * 1.001, 1e-4)
        assert (np.abs(a - b) <= allow).all(), k
        assert small.mean() < 0.5, k  # most elements meet the tight bound


@pytest.mark.parametrize("world", [2, 4])
@pytest.mark.parametrize("mode", ["peer", "peer_keep", "sharded_adam", "allreduce", "nvls"])
def test_multi_gpu_step_matches_mean_of_views(cuda, orc, mode, world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    if world > 2 and mode not in ("peer", "nvls"):
        pytest.skip("the other exchanges are checked on 2 GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, mode)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted([q.get(timeout=300) for _ in range(world)], key=lambda r: r[0])
    for p in procs:
        p.join(timeout=60)
    assert all(r[1] == "ok" for r in res), res
    if mode == "nvls" and not res[0][6]:
        pytest.skip("the devices offer no NVLink multicast")
    assert res[0][5] == (mode.startswith("peer") or mode == "nvls", mode == "sharded_adam")
    for r in res[1:]:
        for k in (2, 3, 4):
            np.testing.assert_array_equal(res[0][k], r[k])
    ref, grads = _oracle_mean_of_views(orc, _n_of(mode), world)
    _assert_close_to_oracle_step([res[0][k] for k in (2, 3, 4)], ref, grads)


def _dp_call(lib, ctx, groups, world, rank, flags, epoch, timeout_ns, step=1, grad_scale=1.0):
    import ctypes as C

    from brush_b200 import _lib

    ex = _lib.DpExchange()
    ex.rank, ex.world = rank, world
    for q in range(world):
        ex.d_flags[q] = flags[q].data_ptr()
    ex.refine_rows = 0
    ex.epoch = epoch
    ex.timeout_ns = timeout_ns
    arr = (_lib.DpGroup * len(groups))()
    for i, g in enumerate(groups):
        for q in range(world):
            arr[i].d_param[q] = g["param"][q].data_ptr()
            arr[i].d_grad[q] = g["grad"][q].data_ptr()
        arr[i].d_m = g["m"].data_ptr()
        arr[i].d_v = g["v"].data_ptr()
        arr[i].rows, arr[i].cols = g["param"][0].shape
        arr[i].lr = g["lr"]
        arr[i].h_col_scale = None
        arr[i].reduce_moment_2 = int(g["reduce"])
    cfg = _lib.AdamCfg(beta_1=0.9, beta_2=0.999, epsilon=1e-15, step=step, grad_scale=grad_scale)
    return lib.bsx_dp_adam_step(ctx.handle, C.byref(ex), arr, len(groups), C.byref(cfg))


def test_dp_kernel_world_one_equals_adam(cuda):
    """With one rank the exchange kernel is the fused Adam: bit-equal parameters and moments."""
    from brush_b200 import _lib
    from brush_b200._context import context
    from brush_b200.adam import AdamGroup, AdamScaled

    rng = np.random.default_rng(5)
    n = 30011
    shapes = [(n, 10, False), (n, 48, True), (n, 1, False)]
    ctx = context(0)
    lib = _lib.lib()
    flags = [torch.zeros(_lib.BSX_DP_FLAG_WORDS, dtype=torch.int32, device="cuda")]
    p0 = [rng.normal(0, 1, (r, c)).astype(np.float32) for r, c, _ in shapes]
    ref = [AdamGroup(torch.from_numpy(p.copy()).cuda(), None, 1e-3, reduce_moment_2=red)
           for p, (_, _, red) in zip(p0, shapes)]
    dp = [dict(param=[torch.from_numpy(p.copy()).cuda()], grad=[None], m=torch.zeros(r, c, device="cuda"),
               v=torch.zeros((r,) if red else (r, c), device="cuda"), lr=1e-3, reduce=red)
          for p, (r, c, red) in zip(p0, shapes)]
    opt = AdamScaled()
    for step in (1, 2, 3):
        grads = [torch.from_numpy(rng.normal(0, 1, p.shape).astype(np.float32)).cuda() for p in p0]
        for g, gr in zip(ref, grads):
            g.grad = gr
        opt.step(ref, grad_scale=0.5)
        for d, gr in zip(dp, grads):
            d["grad"] = [gr]
        ctx.check(_dp_call(lib, ctx, dp, 1, 0, flags, step, int(1e9), step=step, grad_scale=0.5))
    ctx.sync()
    for g, d in zip(ref, dp):
        np.testing.assert_array_equal(g.param.cpu().numpy(), d["param"][0].cpu().numpy())
        np.testing.assert_array_equal(g.m.cpu().numpy(), d["m"].cpu().numpy())
        np.testing.assert_array_equal(g.v.cpu().numpy(), d["v"].cpu().numpy())


def test_dp_kernel_times_out_when_a_rank_never_arrives(cuda):
    """Rank 0 of a 2-rank exchange whose partner never launches: the bounded wait
    expires, the launch ends, and the host reads BSX_ERR_DEVICE_TIMEOUT."""
    import time

    from brush_b200 import _lib
    from brush_b200._context import context

    ctx = context(0)
    lib = _lib.lib()
    n, c = 4096, 10
    # the absent rank's buffers are ordinary local memory that nothing signals
    flags = [torch.zeros(_lib.BSX_DP_FLAG_WORDS, dtype=torch.int32, device="cuda") for _ in range(2)]
    g = dict(param=[torch.zeros(n, c, device="cuda") for _ in range(2)],
             grad=[torch.ones(n, c, device="cuda") for _ in range(2)],
             m=torch.zeros(n // 2, c, device="cuda"), v=torch.zeros(n // 2, c, device="cuda"), lr=1e-3, reduce=False)
    t0 = time.perf_counter()
    ctx.check(_dp_call(lib, ctx, [g], 2, 0, flags, 1, int(2e8)))
    with pytest.raises(_lib.BsxError) as ei:
        ctx.sync()
    dt = time.perf_counter() - t0
    assert ei.value.status == 4  # BSX_ERR_DEVICE_TIMEOUT
    assert dt < 30.0
    # the context stays usable: the error word was cleared and a world-1 call succeeds
    g1 = dict(param=[g["param"][0]], grad=[g["grad"][0]], m=torch.zeros(n, c, device="cuda"),
              v=torch.zeros(n, c, device="cuda"), lr=1e-3, reduce=False)
    ctx.check(_dp_call(lib, ctx, [g1], 1, 0, [torch.zeros(64, dtype=torch.int32, device="cuda")], 1, int(1e9)))
    ctx.sync()
    assert torch.isfinite(g["param"][0]).all()


def _refine_worker(rank, world, port, q, exchange="peer"):
    sys.path.insert(0, str(ROOT))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import brush_b200 as bsx
    from brush_b200.dist import view_for

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    torch.distributed.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                                         timeout=datetime.timedelta(seconds=60))
    try:
        splats, cams, size, gts = _scene(dev)
        tr = bsx.SplatTrainer(bsx.TrainConfig(), splats, process_group=torch.distributed.group.WORLD,
                              exchange=exchange)
        for k in range(4):
            v = view_for(k, rank, world, len(cams))
            tr.step(cams[v], size, gts[v], splats)
        torch.cuda.synchronize()
        n = splats.num_splats
        rec = [x.cpu().numpy().copy() for x in (tr.record.refine_weight_norm, tr.record.vis_weight,
                                                tr.record.max_screen_size)]
        (m_t, m_s, m_o), (v_t, v_s, v_o) = tr.native.optimizer_state()
        shard = [x.reshape(x.shape[0], -1).cpu().numpy().copy() for x in (m_t, m_s, m_o, v_t, v_s, v_o)]
        pre = [x.cpu().numpy().copy() for x in (splats.transforms, splats.sh_coeffs, splats.raw_opacities)]
        bounds = (tr.bounds[0].copy(), tr.bounds[1].copy())
        cfg = bsx.RefineConfig(growth_grad_threshold=2e-5, growth_select_fraction=0.3, split_at_screen_size=0.05,
                               seed=99)
        st = tr.refine(splats, 200, 200, 3000, cfg)
        torch.cuda.synchronize()
        post = [x.cpu().numpy().copy() for x in (splats.transforms, splats.sh_coeffs, splats.raw_opacities)]
        for k in range(4, 7):
            v = view_for(k, rank, world, len(cams))
            tr.step(cams[v], size, gts[v], splats)
        torch.cuda.synchronize()
        tr.peer.ctx.sync()
        later = [x.cpu().numpy().copy() for x in (splats.transforms, splats.sh_coeffs, splats.raw_opacities)]
        q.put((rank, "ok", dict(rec=rec, shard=shard, pre=pre, bounds=bounds, post=post, later=later,
                                total=st.total_splats, added=st.num_added, mc=bool(tr.peer.mc_base))))
        tr.close()
    except Exception as e:  # noqa: BLE001
        import traceback

        q.put((rank, "error", traceback.format_exc()))
    finally:
        torch.distributed.destroy_process_group()


@pytest.mark.parametrize("exchange", ["peer", "nvls"])
def test_two_gpu_refine_identical_on_both_ranks_and_matches_oracle(cuda, orc, exchange):
    """Four steps (mean noise on, gated on the combined visibility), a refine, three more steps:
    both replicas stay bit-identical, and the refine equals the oracle's on the combined state."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_refine_worker, args=(r, 2, port, q, exchange)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted([q.get(timeout=300) for _ in range(2)], key=lambda r: r[0])
    for p in procs:
        p.join(timeout=60)
    assert all(r[1] == "ok" for r in res), res
    a, b = res[0][2], res[1][2]
    if exchange == "nvls" and not a["mc"]:
        pytest.skip("the devices offer no NVLink multicast")
    assert a["total"] == b["total"] and a["added"] > 0
    for x, y in zip(a["post"] + a["later"], b["post"] + b["later"]):
        np.testing.assert_array_equal(x, y)
    # the oracle refines the combined state: statistics combined over ranks, full moments
    rec = (np.maximum(a["rec"][0], b["rec"][0]), a["rec"][1] + b["rec"][1], np.maximum(a["rec"][2], b["rec"][2]))
    full = [np.concatenate([sa, sb], 0) for sa, sb in zip(a["shard"], b["shard"])]
    n = a["pre"][0].shape[0]
    moments = ((full[0], full[1], full[2].reshape(n)), (full[3], full[4].reshape(n), full[5].reshape(n)))
    ref = orc.refine(*a["pre"], rec, moments, orc.refine_cfg(growth_grad_threshold=2e-5, growth_select_fraction=0.3,
                                                              split_at_screen_size=0.05, seed=99),
                     a["bounds"][0], a["bounds"][1], 200, 0, 200, 3000)
    assert ref["stats"].total_splats == a["total"]
    np.testing.assert_array_equal(a["post"][0], ref["transforms"])
    np.testing.assert_array_equal(a["post"][1], ref["sh"])
    np.testing.assert_array_equal(a["post"][2], ref["opac"])

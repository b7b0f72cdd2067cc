"""Data-parallel host logic on CPU (gloo, world sizes 2 and 4), with the oracle as the compute.

- every rank trains its own view; after the exchange all ranks hold identical
  splats equal to a single-process Adam step on the mean-of-views gradient;
- a rank that dies before the collective makes the survivor fail fast with an
  error instead of hanging.
"""
import datetime
import multiprocessing as mp
import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _scene():
    from brush_b200.splats import config1_scene, orbit_camera

    splats, _, size, _ = config1_scene("cpu", seed=11, n=3000)
    w, h = 96, 80
    cams = [orbit_camera(i, 4, 3.0, w, h, fov_deg=50.0) for i in range(4)]
    from brush_b200.splats import random_gt

    gts = [random_gt(h, w, 50 + i, "cpu").numpy() for i in range(4)]
    return splats, cams, (w, h), gts


def _view_grad(orc, splats, cam, size, gt):
    w, h = size
    r = orc.RenderResult(cam, size, splats.transforms.numpy(), splats.sh_coeffs.numpy(), splats.raw_opacities.numpy())
    chw = np.ascontiguousarray(r.image[..., :3].transpose(2, 0, 1))
    oc = orc.loss_cfg(0.8, -0.2)
    dl = np.full((3, h, w), np.float32(1.0 / (3 * h * w)), np.float32)
    vo = np.zeros((h, w, 4), np.float32)
    vo[..., :3] = orc.loss_bwd(chw, gt, oc, dl).transpose(1, 2, 0)
    vc = r.rasterize_bwd(vo)
    vt, vs, vop, vr = r.project_bwd(vc)
    return np.concatenate([vt.ravel(), vs.ravel(), vop.ravel()]).astype(np.float32), vr


def _apply(orc, splats, flat, scale):
    n, c = splats.num_splats, splats.sh_coeffs_per_splat
    t = splats.transforms.numpy().copy()
    sh = splats.sh_coeffs.numpy().reshape(n, 3 * c).copy()
    op = splats.raw_opacities.numpy().reshape(n, 1).copy()
    gt_, gs, go = flat[: n * 10].reshape(n, 10), flat[n * 10: n * (10 + 3 * c)].reshape(n, 3 * c), flat[n * (10 + 3 * c):]
    orc.adam(t, gt_, np.zeros_like(t), np.zeros_like(t), 1e-3, None, False, grad_scale=scale)
    orc.adam(sh, gs, np.zeros_like(sh), np.zeros(n, np.float32), 1e-3, None, True, grad_scale=scale)
    orc.adam(op, go.reshape(n, 1), np.zeros_like(op), np.zeros_like(op), 1e-3, None, False, grad_scale=scale)
    return t, sh, op


def _apply_sharded(orc, splats, flat, rank, world, group):
    """reduce-scatter rows -> Adam on this rank's rows -> in-place all-gather."""
    import torch

    from brush_b200.dist import all_gather_rows, reduce_scatter_rows, row_shard

    n, c = splats.num_splats, splats.sh_coeffs_per_splat
    ft = torch.from_numpy(flat)
    fulls_g = (ft[: n * 10].view(n, 10), ft[n * 10: n * (10 + 3 * c)].view(n, 3 * c), ft[n * (10 + 3 * c):].view(n, 1))
    r0, r1 = row_shard(n, world, rank)
    shards = tuple(torch.empty((r1 - r0, f.shape[1])) for f in fulls_g)
    reduce_scatter_rows(fulls_g, shards, group)
    t = splats.transforms.numpy().copy()
    sh = splats.sh_coeffs.numpy().reshape(n, 3 * c).copy()
    op = splats.raw_opacities.numpy().reshape(n, 1).copy()
    for p, g, red in [(t, shards[0], False), (sh, shards[1], True), (op, shards[2], False)]:
        pv = np.ascontiguousarray(p[r0:r1])
        orc.adam(pv, g.numpy(), np.zeros_like(pv), np.zeros(r1 - r0, np.float32) if red else np.zeros_like(pv), 1e-3,
                 None, red, grad_scale=1.0 / world)
        p[r0:r1] = pv
    fulls_p = (torch.from_numpy(t), torch.from_numpy(sh), torch.from_numpy(op))
    all_gather_rows(fulls_p, group, rank, world)
    return fulls_p[0].numpy(), fulls_p[1].numpy(), fulls_p[2].numpy()


def _worker(rank, world, port, q, die_rank, sharded=False):
    sys.path.insert(0, str(ROOT))
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import torch

    from brush_b200.dist import reduce_gradients, replicas_agree, view_for
    from oracle import oracle as orc

    torch.distributed.init_process_group("gloo", rank=rank, world_size=world,
                                         timeout=datetime.timedelta(seconds=15))
    try:
        splats, cams, size, gts = _scene()
        v = view_for(0, rank, world, len(cams))
        flat, vr = _view_grad(orc, splats, cams[v], size, gts[v])
        if rank == die_rank:
            os._exit(3)  # leaves between steps, before the collective
        if sharded:
            t, sh, op = _apply_sharded(orc, splats, flat, rank, world, torch.distributed.group.WORLD)
            rt, scale = torch.from_numpy(vr), 1.0 / world
            torch.distributed.all_reduce(rt, op=torch.distributed.ReduceOp.MAX)
        else:
            ft, rt = torch.from_numpy(flat), torch.from_numpy(vr)
            scale = reduce_gradients(ft, rt, torch.distributed.group.WORLD)
            t, sh, op = _apply(orc, splats, ft.numpy(), scale)
        agree = replicas_agree(torch.distributed.group.WORLD, torch.from_numpy(t), torch.from_numpy(sh),
                               torch.from_numpy(op))
        q.put((rank, "ok", t, sh, op, scale, agree, rt.numpy()))
    except Exception as e:  # noqa: BLE001
        q.put((rank, "error", repr(e)))
    finally:
        try:
            torch.distributed.destroy_process_group()
        except Exception:  # noqa: BLE001
            pass


def _run(world, die_rank=-1, timeout=120, sharded=False):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, die_rank, sharded)) for r in range(world)]
    for p in procs:
        p.start()
    out = []
    alive = world - (1 if die_rank >= 0 else 0)
    for _ in range(alive):
        out.append(q.get(timeout=timeout))
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    return sorted(out, key=lambda r: r[0])


@pytest.mark.parametrize("world", [2, 4])
@pytest.mark.parametrize("sharded", [False, True], ids=["allreduce", "reduce_scatter"])
def test_ranks_match_mean_of_views_step(orc, sharded, world):
    res = _run(world, sharded=sharded)
    assert all(r[1] == "ok" for r in res), res
    _, _, t0, s0, o0, _, _, r0 = res[0]
    for (_, _, t, sh, op, sc, ag, rw) in res:
        assert sc == 1.0 / world and ag
        np.testing.assert_array_equal(t, t0)
        np.testing.assert_array_equal(sh, s0)
        np.testing.assert_array_equal(op, o0)
        np.testing.assert_array_equal(rw, r0)
    # single process: every rank's view gradient summed, scaled by 1/world
    from brush_b200.dist import view_for

    splats, cams, size, gts = _scene()
    views = [view_for(0, r, world, len(cams)) for r in range(world)]
    assert sorted(views) == list(range(world))
    flats = [_view_grad(orc, splats, cams[v], size, gts[v]) for v in views]
    t, sh, op = _apply(orc, splats, np.sum([f[0] for f in flats], axis=0, dtype=np.float32), 1.0 / world)
    np.testing.assert_allclose(t0, t, rtol=0, atol=2e-6)
    np.testing.assert_allclose(s0, sh, rtol=0, atol=2e-6)
    np.testing.assert_allclose(o0, op, rtol=0, atol=2e-6)
    # the oracle's raster backward sums with OpenMP atomics, so an independent
    # recomputation agrees to rounding, not bit-for-bit
    np.testing.assert_allclose(r0, np.max([f[1] for f in flats], axis=0), rtol=1e-4, atol=1e-9)


def test_dead_rank_fails_fast_instead_of_hanging():
    res = _run(2, die_rank=1, timeout=90)
    assert len(res) == 1 and res[0][0] == 0 and res[0][1] == "error", res

"""GPU primitives against the reference's own known answers and the oracle
(crates/brush-sort/src/lib.rs:158-429, crates/brush-prefix-sum/src/lib.rs:109-220,
crates/brush-render/src/get_tile_offset.rs:88-129). Integer work: bit-exact."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _t(a):
    return torch.from_numpy(np.ascontiguousarray(np.asarray(a, dtype=np.uint32)).view(np.int32)).cuda()


def _u(t):
    return t.cpu().numpy().view(np.uint32)


def test_sort_stable_for_every_pass_count(cuda, orc):
    from brush_b200.primitives import radix_argsort

    n = 4099
    i = np.arange(n, dtype=np.uint64)
    group = ((i * 73) % 1021).astype(np.uint64)
    prod = (group * 0x9E3779B9) & 0xFFFFFFFF
    keys = ((((prod << 7) | (prod >> 25)) & 0xFFFFFFFF) ^ 0xA5A55A5A).astype(np.uint32)
    vals = np.arange(n, dtype=np.uint32)
    kt, vt = _t(keys), _t(vals)
    for bits in [0, 4, 8, 12, 13, 14, 15, 16, 20, 28, 32]:
        ko, vo = radix_argsort(kt, vt, bits)
        eko, evo = orc.radix_argsort(keys, vals, bits)
        assert (_u(ko) == eko).all() and (_u(vo) == evo).all(), bits
        assert (_u(kt) == keys).all() and (_u(vt) == vals).all()


def test_sort_small_kat(cuda):
    from brush_b200.primitives import radix_argsort

    for i in range(0, 128, 17):
        keys = np.array([5 + i * 4, i, 6, 123, 74657, 123, 999, 2**24 + 123, 6, 7, 8, 0], np.uint32)
        vals = np.arange(keys.size, dtype=np.uint32)
        ko, vo = radix_argsort(_t(keys), _t(vals), 32)
        order = np.argsort(keys, kind="stable")
        assert (_u(ko) == keys[order]).all() and (_u(vo) == order).all()


# sizes of the benchmark's depth (647,777 visible) and tile (3,140,719 intersections) sorts among them
@pytest.mark.parametrize("n,bits", [(1, 32), (4095, 32), (4097, 16), (647_777, 32), (1_000_003, 32),
                                    (1_800_001, 32), (2_400_000, 13), (3_140_719, 13), (30_000_000, 13),
                                    (70_000_000, 32)])
def test_sort_large_random(cuda, n, bits):
    from brush_b200.primitives import radix_argsort

    g = torch.Generator(device="cuda")
    g.manual_seed(n)
    keys = torch.randint(-2**31, 2**31 - 1, (n,), generator=g, device="cuda", dtype=torch.int32)
    if bits < 32:
        keys = keys & ((1 << bits) - 1)
    vals = torch.arange(n, device="cuda", dtype=torch.int32)
    ko, vo = radix_argsort(keys, vals, bits)
    k64 = keys.to(torch.int64) & 0xFFFFFFFF
    ref = torch.sort(k64, stable=True)
    assert torch.equal(ko.to(torch.int64) & 0xFFFFFFFF, ref.values)
    assert torch.equal(vo.to(torch.int64), ref.indices)


def test_empty_inputs(cuda):
    from brush_b200.primitives import prefix_sum, radix_argsort

    e = torch.zeros(0, dtype=torch.int32, device="cuda")
    ko, vo = radix_argsort(e, e, 32)
    assert ko.numel() == 0 and vo.numel() == 0
    assert prefix_sum(e).numel() == 0


def test_prefix_sum_kats(cuda):
    from brush_b200.primitives import prefix_sum

    assert list(_u(prefix_sum(_t([1, 1, 1, 1])))) == [1, 2, 3, 4]
    for n in [255, 256, 257, 4095, 4096, 4097, 1024]:
        d = (np.arange(n) % 7 + (90 if n == 1024 else 0)).astype(np.uint32)
        assert (_u(prefix_sum(_t(d))) == np.cumsum(d, dtype=np.uint64).astype(np.uint32)).all(), n
    d = np.array([2, 0, 32, 512, 30965] * (512 * 16 + 123), dtype=np.uint32)
    d[0::5] += np.arange(512 * 16 + 123, dtype=np.uint32)
    assert (_u(prefix_sum(_t(d))) == np.cumsum(d, dtype=np.uint64).astype(np.uint32)).all()


def test_prefix_sum_30m_and_unaligned(cuda):
    from brush_b200.primitives import prefix_sum

    n = 30_000_000
    d = (torch.arange(n, device="cuda", dtype=torch.int64) % 100).to(torch.int32)
    s = prefix_sum(d).to(torch.int64) & 0xFFFFFFFF
    ref = torch.cumsum(d.to(torch.int64), 0) & 0xFFFFFFFF
    assert torch.equal(s, ref)
    base = torch.arange(1, 10001, device="cuda", dtype=torch.int32)
    view = base[3:]  # 12-byte offset: scalar path
    out = prefix_sum(view.clone()) if not view.is_contiguous() else prefix_sum(view)
    assert torch.equal(out.to(torch.int64), torch.cumsum(view.to(torch.int64), 0))


def test_prefix_sum_wraps_like_u32(cuda):
    from brush_b200.primitives import prefix_sum

    d = np.full(10000, 0xF0000000, np.uint32)
    assert (_u(prefix_sum(_t(d))) == np.cumsum(d.astype(np.uint64)).astype(np.uint32)).all()


def test_tile_offsets_kat(cuda, orc):
    from brush_b200.primitives import get_tile_offsets

    runs = [31, 1, 223, 1, 1791, 1, 17, 0]
    ids = []
    for tid, rl in enumerate(runs):
        ids += [tid] * rl
    ids += [8] * 13
    ids = np.array(ids, np.uint32)
    got = _u(get_tile_offsets(_t(ids), 8)).reshape(8, 2)
    assert (got == orc.tile_offsets(ids, 8)).all()

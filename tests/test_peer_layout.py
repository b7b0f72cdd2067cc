"""Exchange-region layout of the peer-memory data-parallel step (no GPU needed):
every rank's shard fits its gradient slots, the slots start 16-byte aligned, the
region holds W slots per group, and the kernel's owner rule (rows
[n q / W, n (q + 1) / W)) matches brush_b200.peer.shard_rows."""
import pytest

from brush_b200.peer import ExchangeLayout, shard_rows


def _owner(n, g, world):
    # the device rule (common.cuh shard_owner): floor(g W / n), raised by one when needed
    q = g * world // n
    if q + 1 < world and shard_rows(n, q + 1, world)[0] <= g:
        q += 1
    return q


@pytest.mark.parametrize("n", [1, 127, 128, 40000, 40001, 1_000_003])
@pytest.mark.parametrize("world", [1, 2, 3, 4, 7, 8])
def test_slots_hold_every_shard(n, world):
    lay = ExchangeLayout(n, 16, world)
    s = lay.slot_rows
    assert s % 4 == 0
    for q in range(world):
        b, e = shard_rows(n, q, world)
        assert e - b <= s
    for name, w in lay.widths.items():
        start = lay.offsets[("grad", name)]
        # slot k of every group starts 16-byte aligned (offsets are 256-byte aligned)
        assert (start * 4) % 256 == 0
        for k in range(world):
            assert ((start + k * s * w) * 4) % 16 == 0
    # the gradient sub-buffers are large enough for W slots and are not overlapped by the next one
    keys = sorted(((v, k) for k, v in lay.offsets.items()), key=lambda x: x[0])
    for (o0, k0), (o1, _) in zip(keys, keys[1:]):
        if isinstance(k0, tuple) and k0[0] == "grad":
            assert o1 - o0 >= world * s * lay.widths[k0[1]]
        elif isinstance(k0, tuple):
            assert o1 - o0 >= n * lay.widths[k0[1]]


@pytest.mark.parametrize("n,world", [(40001, 2), (40001, 4), (1_000_000, 8), (999_999, 7), (300, 2)])
def test_owner_rule_matches_shards(n, world):
    owners = [_owner(n, g, world) for g in range(0, n, max(1, n // 5000))] + [_owner(n, n - 1, world)]
    for g, q in zip(list(range(0, n, max(1, n // 5000))) + [n - 1], owners):
        b, e = shard_rows(n, q, world)
        assert b <= g < e

"""Densification restatement in the oracle (oracle/refine.cpp) against the
reference's documented semantics (CPU only).

The sampler cases mirror the reference's own multinomial tests
(crates/brush-train/src/multinomial.rs:37-120): draws are distinct, NaN and
zero weights are never drawn, a seed repeats its draw. The split geometry
follows refine_splats (crates/brush-train/src/train.rs:1547-1700).
"""
import math

import numpy as np
import pytest

from oracle import oracle as orc


def test_sampler_without_replacement_and_in_range():
    w = np.array([0.1, 0.3, 0.4, 0.2], np.float32)
    s = orc.weighted_sample(w, 3)
    assert len(s) == 3 and len(set(s.tolist())) == 3 and all(0 <= x < 4 for x in s)
    assert orc.weighted_sample(np.array([1.0], np.float32), 1).tolist() == [0]


def test_sampler_skips_nan_and_zero_weights():
    w = np.array([0.5, np.nan, 0.3, 0.2], np.float32)
    for seed in range(50):
        s = orc.weighted_sample(w, 2, seed=seed)
        assert len(s) == 2 and 1 not in s.tolist()
    assert len(orc.weighted_sample(np.zeros(5, np.float32), 3)) == 0
    # more draws than positive weights: every positive index once
    assert sorted(orc.weighted_sample(np.array([0, 2, 0, 1], np.float32), 4).tolist()) == [1, 3]


def test_sampler_repeatable_and_stream_dependent():
    w = np.random.default_rng(0).uniform(0.1, 1.0, 1000).astype(np.float32)
    a, b = orc.weighted_sample(w, 50, seed=7, stream=3), orc.weighted_sample(w, 50, seed=7, stream=3)
    assert a.tolist() == b.tolist()
    assert a.tolist() != orc.weighted_sample(w, 50, seed=7, stream=4).tolist()


def test_sampler_first_draw_proportional_to_weight():
    w = np.array([1, 2, 3, 4], np.float32)
    counts = np.zeros(4)
    trials = 4000
    for t in range(trials):
        counts[orc.weighted_sample(w, 1, seed=t)[0]] += 1
    expected = trials * w / w.sum()
    chi2 = float(((counts - expected) ** 2 / expected).sum())
    assert chi2 < 16.3  # 3 dof, p = 0.001


def _successive_subset_probs(w, k):
    """Exact probability of every k-subset under successive weighted sampling without
    replacement (each draw proportional to the remaining weights): the distribution of
    rand::seq::index::sample_weighted, which the reference's multinomial_sample calls
    (crates/brush-train/src/multinomial.rs:1-28), by Efraimidis & Spirakis (2006)."""
    import itertools

    total = float(sum(w))
    probs = {}
    for order in itertools.permutations(range(len(w)), k):
        p, rest = 1.0, total
        for i in order:
            p *= float(w[i]) / rest
            rest -= float(w[i])
        key = tuple(sorted(order))
        probs[key] = probs.get(key, 0.0) + p
    return probs


def test_sampler_subset_distribution_matches_successive_sampling():
    """Draw-level parity with the reference's sampler is not possible (it runs StdRng);
    its distribution is: the frequency of each 3-of-6 subset over many seeds against the
    exact successive-sampling probabilities (chi-square, 19 degrees of freedom)."""
    w = np.array([0.5, 1.0, 1.5, 2.0, 4.0, 8.0], np.float32)
    probs = _successive_subset_probs(w, 3)
    trials = 20000
    counts = {key: 0 for key in probs}
    for t in range(trials):
        counts[tuple(sorted(orc.weighted_sample(w, 3, seed=t, stream=2).tolist()))] += 1
    chi2 = sum((counts[key] - trials * p) ** 2 / (trials * p) for key, p in probs.items())
    assert chi2 < 43.8  # 19 dof, p = 0.001
    # inclusion frequency of the heaviest weight, against its exact value
    inc = sum(p for key, p in probs.items() if 5 in key)
    got = sum(c for key, c in counts.items() if 5 in key) / trials
    assert abs(got - inc) < 4 * math.sqrt(inc * (1 - inc) / trials)


def _scene(n=400, c=4, seed=0):
    rng = np.random.default_rng(seed)
    t = np.zeros((n, 10), np.float32)
    t[:, 0:3] = rng.normal(0, 1, (n, 3))
    q = rng.normal(0, 1, (n, 4))
    t[:, 3:7] = q
    t[:, 7:10] = rng.normal(-3, 0.5, (n, 3))
    sh = rng.normal(0, 0.3, (n, c, 3)).astype(np.float32)
    op = rng.normal(1, 1, n).astype(np.float32)
    return t, sh, op


def test_prune_mask_bits():
    t, sh, op = _scene(8)
    t[:, 7:10] = -3.0
    t[:, 3:7] = [1, 0, 0, 0]
    op[:] = 2.0
    op[0] = -10.0                 # alpha < 1/255
    t[1, 8] = 5.0                 # scale e^5 > max_allowed 100
    t[2, 0] = 200.0               # outside the bounds (per axis)
    sh[3, 1, 2] = np.nan          # non-finite
    t[4, 9] = -30.0               # raw scale < 1e-10
    t[5, 3:7] = 1e-5              # |q|^2 < 1e-8
    cfg = orc.refine_cfg()
    m = orc.refine_prune_mask(t, sh, op, cfg, np.zeros(3, np.float32), 100.0)
    assert m.tolist() == [1, 2, 4, 8, 16, 32, 0, 0]
    cfg_off = orc.refine_cfg(min_scale_prune=0, near_zero_rotation_prune=0)
    assert orc.refine_prune_mask(t, sh, op, cfg_off, np.zeros(3, np.float32), 100.0).tolist()[4:6] == [0, 0]


def _moments(n, c, rng):
    m = (rng.normal(size=(n, 10)).astype(np.float32), rng.normal(size=(n, 3 * c)).astype(np.float32),
         rng.normal(size=n).astype(np.float32))
    v = (rng.uniform(size=(n, 10)).astype(np.float32), rng.uniform(size=n).astype(np.float32),
         rng.uniform(size=n).astype(np.float32))
    return m, v


def test_refine_split_geometry_and_moments():
    n, c = 300, 4
    rng = np.random.default_rng(1)
    t, sh, op = _scene(n, c, 1)
    rn = np.zeros(n, np.float32)
    rn[::7] = 0.01            # above the growth threshold
    vis = np.ones(n, np.float32)
    screen = np.full(n, 0.01, np.float32)
    screen[5] = 0.8           # too large on screen -> split
    moments = _moments(n, c, rng)
    cfg = orc.refine_cfg(opac_decay=0.0, scale_decay=0.0, growth_select_fraction=0.5)
    r = orc.refine(t, sh, op, (rn, vis, screen), moments, cfg, np.zeros(3, np.float32),
                   np.full(3, 10, np.float32), 10, 0, 10, 100)
    st = r["stats"]
    assert st.num_pruned == 0 and st.num_split_oversized == 1
    grow_expected = round(len(rn[::7]) * 0.5)
    assert st.num_split_high_grad in (grow_expected, grow_expected - 1)  # the oversized one may coincide
    assert st.total_splats == n + st.num_added and 5 in r["split"].tolist()
    for q, s in enumerate(r["split"].tolist()):
        child = n + q
        mean, par, chi = t[s, :3], r["transforms"][s, :3], r["transforms"][child, :3]
        np.testing.assert_allclose(par + chi, 2 * mean, atol=1e-5)
        L = int(np.argmax(t[s, 7:10]))
        off = chi - mean
        assert abs(np.linalg.norm(off) - 0.5 * math.exp(t[s, 7 + L])) <= 1e-5 * (1 + math.exp(t[s, 7 + L]))
        m_long = min(0.5, 0.5 / max(screen[s], 1e-6))
        for k in range(3):
            want = t[s, 7 + k] + (math.log(m_long) if k == L else math.log(0.85))
            assert abs(r["transforms"][child, 7 + k] - want) < 1e-5
        qn = t[s, 3:7] / np.linalg.norm(t[s, 3:7])
        np.testing.assert_allclose(r["transforms"][child, 3:7], qn, atol=1e-6)
        np.testing.assert_array_equal(r["transforms"][s, 3:7], t[s, 3:7])   # parent rotation unchanged
        np.testing.assert_array_equal(r["sh"][child], sh[s])
        sig = 1 / (1 + math.exp(-op[s]))
        assert abs(1 / (1 + math.exp(-r["opac"][child])) - sig * 0.6) < 1e-5
        for arr in r["m"] + r["v"]:
            assert not np.any(arr[s]) and not np.any(arr[child])
    untouched = np.setdiff1d(np.arange(n), r["split"])
    np.testing.assert_array_equal(r["m"][0][untouched], moments[0][0][untouched])
    np.testing.assert_array_equal(r["transforms"][untouched], t[untouched])


def test_refine_prunes_then_replaces_and_respects_max_splats():
    n, c = 200, 1
    rng = np.random.default_rng(2)
    t, sh, op = _scene(n, c, 2)
    op[:20] = -10.0           # pruned for opacity
    vis = np.ones(n, np.float32)
    vis[100:] = 0.0           # replacements only among visible splats
    rn = np.full(n, 0.01, np.float32)
    screen = np.zeros(n, np.float32)
    cfg = orc.refine_cfg(max_splats=190, growth_select_fraction=1.0)
    r = orc.refine(t, sh, op, (rn, vis, screen), _moments(n, c, rng), cfg, np.zeros(3, np.float32),
                   np.full(3, 10, np.float32), 0, 0, 0, 100)
    st = r["stats"]
    assert st.num_pruned == 20 and st.num_added == 20 and st.total_splats == 200
    assert r["keep"].tolist() == list(range(20, 200))
    # every replacement is a kept row whose original splat was visible
    assert all(r["keep"][s] < 100 for s in r["split"].tolist())
    # growth: 80 visible above the threshold, grow = 80 - 20 pruned = 60, capped by max_splats 190 - 200 = 0
    assert st.num_split_high_grad == 0
    # opacity decay at phase 0: sigmoid drops by opac_decay
    kept = r["keep"][0]
    sig_new = 1 / (1 + math.exp(-float(r["opac"][0])))
    assert abs(sig_new - (1 / (1 + math.exp(-op[kept])) - 0.004)) < 1e-5 or 0 in r["split"].tolist()


def test_refine_all_pruned_keeps_everything():
    n, c = 10, 1
    t, sh, op = _scene(n, c, 3)
    op[:] = -20.0
    r = orc.refine(t, sh, op, (np.zeros(n, np.float32), np.zeros(n, np.float32), np.zeros(n, np.float32)),
                   _moments(n, c, np.random.default_rng(0)), orc.refine_cfg(), np.zeros(3, np.float32),
                   np.ones(3, np.float32), 0, 0, 0, 100)
    assert r["stats"].num_pruned == 0 and r["stats"].total_splats == n


def test_gradient_threshold_rule_clone_split_prune():
    """The original 3DGS densification (Kerbl et al. 2023) as restated: rows that stay,
    clones, then the two children of every split row; opacity pruning; new rows have zero
    moments; children sit at mean + R(q) (s * n) with scales s / 1.6."""
    n, c = 400, 4
    rng = np.random.default_rng(5)
    t, sh, op = _scene(n, c, 5)
    t[:, 7:10] = -3.0
    t[::2, 7] = -1.0                      # even rows large (split), odd rows small (clone)
    op[:] = 1.0
    op[390:] = -8.0                       # opacity 3e-4 < 0.005: pruned
    vis = np.full(n, 2.0, np.float32)
    vis[300:310] = 0.0                    # never visible: never selected
    g2 = np.zeros(n, np.float32)
    g2[:320:4] = 2.0 * 3e-4               # average 3e-4 >= 2e-4 (rows 0, 4, 8, ...)
    g2[1:320:4] = 2.0 * 1e-4              # average 1e-4: below
    g2[3:320:8] = 2.0 * 5e-4              # odd rows above: cloned
    moments = _moments(n, c, rng)
    extent = np.full(3, 10.0, np.float32)
    # boundary: percent_dense x 10 = 0.1 between e^-3 (0.05) and e^-1 (0.37)
    cfg = orc.refine_cfg(rule=1, growth_grad_threshold=2e-4, min_opacity=0.005, percent_dense=0.01, seed=3)
    r = orc.refine(t, sh, op, (np.zeros(n, np.float32), vis, np.zeros(n, np.float32), g2), moments, cfg,
                   np.zeros(3, np.float32), extent, 0, 0, 0, 100)
    st = r["stats"]
    splits = [i for i in range(0, 320, 4) if not (300 <= i < 310)]
    clones = [i for i in range(3, 320, 8) if not (300 <= i < 310)]
    assert st.num_pruned == 10 and st.num_split_high_grad == len(splits)
    assert st.num_added - st.num_split_high_grad == len(clones)
    K = n - 10
    assert st.total_splats == K + len(clones) + len(splits)
    stay = [i for i in range(K) if i not in set(splits)]
    np.testing.assert_array_equal(r["transforms"][:len(stay)], t[stay])
    np.testing.assert_array_equal(r["m"][0][:len(stay)], moments[0][0][stay])
    base = len(stay)
    np.testing.assert_array_equal(r["transforms"][base:base + len(clones)], t[clones])
    np.testing.assert_array_equal(r["sh"][base:base + len(clones)], sh[clones])
    base += len(clones)
    S = len(splits)
    for k in range(2):
        for q, i in enumerate(splits):
            row = r["transforms"][base + k * S + q]
            np.testing.assert_allclose(row[7:10], np.log(np.exp(t[i, 7:10].astype(np.float64)) / 1.6), atol=1e-6)
            np.testing.assert_array_equal(row[3:7], t[i, 3:7])
            assert r["opac"][base + k * S + q] == op[i]
            z = orc.normal3(3, (1 << 30) + k, i)
            qn = t[i, 3:7].astype(np.float64) / np.linalg.norm(t[i, 3:7].astype(np.float64))
            w, x, y, zz = qn
            R = np.array([[1 - 2 * (y * y + zz * zz), 2 * (x * y - w * zz), 2 * (x * zz + w * y)],
                          [2 * (x * y + w * zz), 1 - 2 * (x * x + zz * zz), 2 * (y * zz - w * x)],
                          [2 * (x * zz - w * y), 2 * (y * zz + w * x), 1 - 2 * (x * x + y * y)]])
            want = t[i, :3] + R @ (np.exp(t[i, 7:10].astype(np.float64)) * z)
            np.testing.assert_allclose(row[:3], want, atol=1e-5)
    for arr in r["m"] + r["v"]:
        assert not np.any(arr[len(stay):])
    # the budget cuts clones, then splits, in row order
    r2 = orc.refine(t, sh, op, (np.zeros(n, np.float32), vis, np.zeros(n, np.float32), g2), moments,
                    orc.refine_cfg(rule=1, growth_grad_threshold=2e-4, min_opacity=0.005, max_splats=K + 5, seed=3),
                    np.zeros(3, np.float32), extent, 0, 0, 0, 100)
    assert r2["stats"].total_splats == K + 5 and r2["stats"].num_split_high_grad == 0

"""The mean-noise step (crates/brush-train/src/train.rs:1095-1169) and its generator, on the CPU.

The reference draws the normals from its device RNG; this library draws them from a
counter-based generator shared by the kernels and the oracle (SplitMix64 of the seed,
the optimizer step and the splat index, Box-Muller with a sine / cosine of its own).
Checked here: the sine / cosine against the double-precision functions at every
argument the generator produces, the normals' distribution, integer powers, and the
step's formula (gate, opacity weight, clamp) on the oracle restatement.
"""
import math

import numpy as np
import pytest


def test_sincos_2pi_accuracy(orc):
    es, ec = orc.sincos_2pi_max_err()
    assert es <= 1.5e-7 and ec <= 1.5e-7, (es, ec)
    for u, (s, c) in [(0.0, (0.0, 1.0)), (0.25, (1.0, 0.0)), (0.5, (0.0, -1.0)), (0.75, (-1.0, 0.0))]:
        got = orc.sincos_2pi(u)
        assert abs(got[0] - s) <= 1e-7 and abs(got[1] - c) <= 1e-7


def test_normals_are_standard_and_deterministic(orc):
    from scipy import stats

    z = orc.normal3_many(42, 7, 400_000)
    assert np.isfinite(z).all()
    n = z.shape[0]
    for k in range(3):
        x = z[:, k].astype(np.float64)
        assert abs(x.mean()) <= 5.0 / math.sqrt(n)
        assert abs(x.var() - 1.0) <= 5.0 * math.sqrt(2.0 / n)
        assert stats.kstest(x, "norm").pvalue > 1e-4
    c = np.corrcoef(z.T.astype(np.float64))
    assert np.abs(c - np.eye(3)).max() <= 5.0 / math.sqrt(n)
    # tails: P(|z| > 3) = 0.0027
    assert abs((np.abs(z) > 3).mean() - 0.0027) <= 0.0005
    np.testing.assert_array_equal(z[:10], orc.normal3_many(42, 7, 10))
    np.testing.assert_array_equal(orc.normal3(42, 7, 123), z[123])
    assert not np.array_equal(orc.normal3_many(42, 8, 10), z[:10])
    assert not np.array_equal(orc.normal3_many(43, 7, 10), z[:10])


@pytest.mark.parametrize("b", [0.0, 0.5, 0.9, 0.99, 0.999, 1.0])
def test_powi_150(orc, b):
    want = np.float64(np.float32(b)) ** 150
    got = orc.powi(b, 150)
    assert abs(got - want) <= 2e-5 * want + 1e-40


def test_mean_noise_step_formula(orc):
    rng = np.random.default_rng(3)
    n = 5000
    t = rng.normal(0, 1, (n, 10)).astype(np.float32)
    raw = rng.normal(-3, 2, n).astype(np.float32)
    gate = (rng.uniform(0, 1, n) < 0.7).astype(np.float32)
    scale, limit = np.float32(0.05), np.float32(0.02)
    out = orc.mean_noise_step(t, raw, gate, scale, limit, 9, 5)
    # only the means of gated splats move; the rest of every row is untouched
    np.testing.assert_array_equal(out[:, 3:], t[:, 3:])
    np.testing.assert_array_equal(out[gate == 0, :3], t[gate == 0, :3])
    d = out[:, :3].astype(np.float64) - t[:, :3]
    assert (np.abs(d) <= limit + 1e-6).all()  # the float addition rounds to the mean's ulp
    z = orc.normal3_many(9, 5, n).astype(np.float64)
    w = np.clip((1.0 - 1.0 / (1.0 + np.exp(-raw.astype(np.float64)))) ** 150, 0, 1) * gate
    want = np.clip(z * (w * float(scale))[:, None], -float(limit), float(limit))
    assert np.abs(d - want).max() <= 1e-6
    assert (np.abs(d[gate > 0]) > 0).any() and (np.abs(d) >= limit * 0.999).any()
    # opaque splats do not move: (1 - opacity)^150 underflows
    opaque = orc.mean_noise_step(t, np.full(n, 8.0, np.float32), np.ones(n, np.float32), scale, limit, 9, 5)
    np.testing.assert_array_equal(opaque, t)

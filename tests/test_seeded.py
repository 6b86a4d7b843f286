"""The seeded input generator (CPU)."""
import numpy as np


def test_deterministic_and_sliceable(pkg):
    s = pkg.seeded
    a = s.normal(123, 1, 1001)
    assert np.array_equal(a, s.normal(123, 1, 1001))
    assert np.array_equal(a[37:600], s.normal(123, 1, 563, offset=37))
    assert np.array_equal(a[1:2], s.normal(123, 1, 1, offset=1))
    assert not np.array_equal(a, s.normal(123, 2, 1001))
    assert not np.array_equal(a, s.normal(124, 1, 1001))


def test_normal_moments(pkg):
    x = pkg.seeded.normal(1, 1, 400000).astype(np.float64)
    assert abs(x.mean()) < 0.01
    assert abs(x.std() - 1.0) < 0.01
    assert np.all(np.isfinite(x))


def test_uniform_int_range(pkg):
    v = pkg.seeded.uniform_int(3, 4, 5000, 256, 8192)
    assert v.min() >= 256 and v.max() <= 8192
    assert abs(v.mean() - (256 + 8192) / 2) < 150


def test_grid_values(pkg):
    g = pkg.seeded.grid_uniform(3, 2, 10000)
    assert set(np.round(np.unique(g) * 100).astype(int)) <= set(range(-100, 100))

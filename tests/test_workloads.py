"""Synthetic workload generators against the checksums the reference publishes for its own
benchmark input (docs/benchmarks.md: input sums -8.5625 at 32768 steps and -3.234375 at 512)."""
import numpy as np

from timestral_b200 import synthetic as sy


def test_dyadic_input_checksums():
    assert float(sy.series_dyadic(32768).sum(dtype=np.float64)) == -8.5625
    assert float(sy.series_dyadic(512).sum(dtype=np.float64)) == -3.234375


def test_dyadic_input_values():
    x = sy.series_dyadic(300, V=3)
    assert x.shape == (1, 3, 300) and x.dtype == np.float32
    t = np.arange(300)
    for v in range(3):
        want = (((17 * t + 13 * v) % 257) - 128) / 64.0
        assert np.array_equal(x[0, v].astype(np.float64), want)
    assert np.isfinite(x).all()

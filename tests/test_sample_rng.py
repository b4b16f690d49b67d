"""The sampled decode's random stream (host side of libbfp200, no GPU):
numpy's legacy generator after np.random.seed(seed), one random_sample per
draw -- the stream sim_rtl_fp_hw.py's np.random.choice consumes (:17, :213)."""
import numpy as np
import pytest

from bfp200 import _lib


@pytest.mark.parametrize("seed", [0, 1, 7, 12345, 2**32 - 1])
def test_uniforms_equal_numpy_legacy(seed):
    n = 1500                                   # crosses the 624-word state refills
    out = np.empty(n, np.float64)
    _lib.check(_lib.lib().bfp200_sample_uniforms(seed, n, _lib.ptr(out)))
    rs = np.random.RandomState(seed)
    assert np.array_equal(out, rs.random_sample(n))


def test_choice_uses_one_uniform_per_draw():
    """np.random.choice(n, p=p) == searchsorted(cumsum(p)/cumsum(p)[-1], u, 'right')."""
    p = np.random.default_rng(3).random(1000)
    p /= p.sum()
    np.random.seed(5)
    draws = [int(np.random.choice(len(p), p=p)) for _ in range(40)]
    u = np.empty(40, np.float64)
    _lib.check(_lib.lib().bfp200_sample_uniforms(5, 40, _lib.ptr(u)))
    cdf = np.cumsum(p)
    cdf /= cdf[-1]
    assert draws == [int(np.searchsorted(cdf, x, side="right")) for x in u]

"""The reference's own sketch unit tests (src/data/sketch.rs:565-780), run on
the CPU oracle and on the engine's host sketch (fb_sketch_features, the path
weighted data and max_bin > 1024 take; the device sketch is checked bit for
bit against the oracle on the GPU): quantile accuracy on sorted and shuffled
data, weights shifting quantiles, strictly increasing cuts on skewed data,
constant and low-cardinality features, finite cuts over the full f32 range,
and per-feature bin counts."""
import ctypes as C

import numpy as np
import pytest

from ferrisboost_b200 import _lib


def engine_sketch(X, max_bin, w=None):
    X = np.ascontiguousarray(X, np.float32)
    n, F = X.shape
    cap = F * (max_bin + 2)
    cuts = np.zeros(cap, np.float32)
    counts = np.zeros(F, np.uint32)
    feats = np.arange(F, dtype=np.uint32)
    w = None if w is None else np.ascontiguousarray(w, np.float32)
    k = _lib.load().fb_sketch_features(_lib.ptr(X, C.c_float), n, F, max_bin, _lib.ptr(w, C.c_float), None,
                                       _lib.ptr(feats, C.c_uint32), F, 0, _lib.ptr(cuts, C.c_float),
                                       _lib.ptr(counts, C.c_uint32), cap)
    assert k >= 0
    off = np.concatenate([[0], np.cumsum(counts)]).astype(np.uint32)
    return cuts[:k].copy(), off


@pytest.fixture(params=["oracle", "engine"])
def sketch(request, oracle):
    if request.param == "oracle":
        return lambda X, mb, w=None: oracle.sketch(X, mb, w)
    return engine_sketch


def max_quantile_err(cuts, max_bins):  # sketch.rs:559-567
    return max(abs(v - (k + 1) / max_bins) for k, v in enumerate(cuts))


def test_uniform_quantiles(sketch):
    n, mb = 100_000, 16
    sorted_x = (np.arange(n, dtype=np.float32) / np.float32(n))[:, None]
    shuffled = (((np.arange(n) * 7919) % n).astype(np.float32) / np.float32(n))[:, None]
    for X in (sorted_x, shuffled):
        cuts, off = sketch(X, mb)
        assert len(cuts) < mb
        assert max_quantile_err(cuts, mb) < 0.02


def test_weights_shift_quantiles(sketch):
    v = np.arange(1000, dtype=np.float32)[:, None]
    cu, _ = sketch(v, 8)
    cw, _ = sketch(v, 8, np.where(v[:, 0] > 500, 10.0, 1.0).astype(np.float32))
    assert cw[3] > cu[3]


def test_skewed_cuts_strictly_increasing(sketch):
    i = np.arange(100_000)
    X = np.where(i % 100 == 0, i, 0).astype(np.float32)[:, None]
    cuts, _ = sketch(X, 16)
    assert np.all(np.diff(cuts) > 0)


def test_constant_and_low_cardinality(sketch):
    cuts, off = sketch(np.full((1000, 1), 42.0, np.float32), 256)
    assert off[-1] == 0
    X = np.tile(np.array([1.0, 2.0, 3.0, 5.0], np.float32), 1000)[:, None]
    cuts, off = sketch(X, 256)
    assert list(cuts) == [1.5, 2.5, 4.0]
    assert list(np.searchsorted(cuts, [1.0, 2.0, 3.0, 5.0], side="right")) == [0, 1, 2, 3]


def test_wide_range_gives_finite_cuts(sketch):
    X = np.array([-3.0e38, -2.0e38, 0.0, 2.0e38, np.finfo(np.float32).max], np.float32)[:, None]
    cuts, off = sketch(X, 16)
    assert off[-1] + 1 == 5  # n_bins == 5
    assert np.all(np.isfinite(cuts)) and np.all(np.diff(cuts) > 0)


def test_per_feature_bin_counts(sketch):
    i = np.arange(1000, dtype=np.float32)
    X = np.stack([i, i % 3, np.full(1000, 7.0, np.float32)], axis=1)
    cuts, off = sketch(X, 8)
    nb = np.diff(off) + 1
    assert nb[0] > 4 and nb[1] == 3 and nb[2] == 1


def test_engine_host_sketch_equals_oracle(oracle):
    rng = np.random.default_rng(12)
    X = rng.standard_normal((30000, 5)).astype(np.float32)
    X[rng.random(X.shape) < 0.05] = np.nan
    w = rng.uniform(0.1, 2.0, 30000).astype(np.float32)
    for mb in (16, 256, 2000):
        for ww in (None, w):
            a = engine_sketch(X, mb, ww)
            b = oracle.sketch(X, mb, ww)
            assert np.array_equal(a[0].view(np.uint32), b[0].view(np.uint32)) and np.array_equal(a[1], b[1])

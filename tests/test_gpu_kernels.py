"""Device kernels against the CPU oracle, bit for bit (integer histograms,
split packets, stable partitions)."""
import numpy as np
import pytest

from gpu_util import Ctx, random_bins

pytestmark = pytest.mark.gpu

FLT_MAX = 3.4028234663852886e38


def oracle_missing(widths):
    return np.array([65535 if w == 2 else 255 for w in widths], dtype=np.uint16)


@pytest.mark.parametrize("seed", [0, 1, 2])
def test_histogram_matches_oracle(oracle, seed):
    rng = np.random.default_rng(seed)
    n = 70000
    nbins = [256, 300, 17, 1024, 255, 2, 64]
    bins, widths = random_bins(rng, n, nbins)
    ctx = Ctx(bins, nbins, widths)
    fixed = rng.integers(-(1 << 40), 1 << 40, (n, 2), dtype=np.int64)
    fixed[:, 1] = np.abs(fixed[:, 1])
    off = np.concatenate([[0], np.cumsum(nbins)]).astype(np.uint32)
    miss = oracle_missing(widths)
    want = oracle.hist(bins, off, miss, fixed)
    assert np.array_equal(ctx.histogram(fixed), want)
    rows = np.sort(rng.choice(n, 12345, replace=False)).astype(np.uint32)
    assert np.array_equal(ctx.histogram(fixed, rows), oracle.hist(bins, off, miss, fixed, rows))
    rng.shuffle(rows)  # order independence (reference tests/bit_exact_vs_xgboost.rs:285-357)
    assert np.array_equal(ctx.histogram(fixed, rows), oracle.hist(bins, off, miss, fixed, rows))


def test_histogram_low_word_carries(oracle):
    # values just below 2^32 force a carry on almost every 32-bit low-plane add
    # (reference tests/gpu_histogram.rs:1272 low-word carry overflow)
    rng = np.random.default_rng(11)
    n = 40000
    nbins = [3, 256]
    bins, widths = random_bins(rng, n, nbins, miss_rate=0.0)
    ctx = Ctx(bins, nbins, widths)
    fixed = np.empty((n, 2), dtype=np.int64)
    fixed[:, 0] = (1 << 32) - 1 - rng.integers(0, 7, n)
    fixed[:, 1] = -((1 << 33) + rng.integers(0, 1 << 31, n))
    off = np.concatenate([[0], np.cumsum(nbins)]).astype(np.uint32)
    assert np.array_equal(ctx.histogram(fixed), oracle.hist(bins, off, oracle_missing(widths), fixed))


def _node_case(oracle, rng, n, nbins, categorical=None):
    bins, widths = random_bins(rng, n, nbins)
    g = rng.standard_normal(n).astype(np.float32) * 0.5
    h = rng.uniform(0.05, 0.25, n).astype(np.float32)
    gp = np.stack([g, h], axis=1)
    scales = oracle.quantizer(gp, n)
    fixed, s = oracle.to_fixed(gp, scales)
    off = np.concatenate([[0], np.cumsum(nbins)]).astype(np.uint32)
    hist = oracle.hist(bins, off, oracle_missing(widths), fixed)
    return bins, widths, hist, s, scales, off


def _same(a, b):
    assert a.found == b.found
    if not a.found:
        return
    assert (a.feat, a.bin, a.missing_left) == (b.feat, b.bin, b.missing_left)
    assert np.float32(a.gain).view(np.uint32) == np.float32(b.gain).view(np.uint32)
    assert (a.left_grad, a.left_hess, a.right_grad, a.right_hess) == (b.left_g, b.left_h, b.right_g, b.right_h)


@pytest.mark.parametrize("seed", range(6))
def test_split_matches_oracle(oracle, seed):
    rng = np.random.default_rng(100 + seed)
    nbins = [256, 40, 256, 1024, 7, 256]
    bins, widths, hist, s, scales, off = _node_case(oracle, rng, 3000, nbins)
    ctx = Ctx(bins, nbins, widths)
    kw = dict(min_child_weight=[1.0, 0.0, 5.0][seed % 3], gamma=[0.0, 0.5][seed % 2],
              alpha=[0.0, 0.3][seed % 2], max_delta_step=[0.0, 0.7][seed % 2])
    _same(ctx.eval_split(hist, s, scales, **kw), oracle.best_split(hist, off, s, scales, **kw))
    en = (rng.random(len(nbins)) < 0.5).astype(np.uint8)
    en[0] = 1
    _same(ctx.eval_split(hist, s, scales, enabled=en, **kw), oracle.best_split(hist, off, s, scales, enabled=en, **kw))
    mono = rng.integers(-1, 2, len(nbins)).astype(np.int8)
    for lo, hi in ((-FLT_MAX, FLT_MAX), (-0.05, 0.3)):
        _same(ctx.eval_split(hist, s, scales, lower=lo, upper=hi, monotone=mono, **kw),
              oracle.best_split(hist, off, s, scales, lower=lo, upper=hi, monotone_constraints=mono, **kw))


def test_split_ties_go_to_the_lower_feature(oracle):
    rng = np.random.default_rng(5)
    bins, widths, hist, s, scales, off = _node_case(oracle, rng, 2000, [64])
    nbins = [64, 64, 64]
    hist3 = np.concatenate([hist, hist, hist])
    bins3 = np.concatenate([bins, bins, bins])
    ctx = Ctx(bins3, nbins, [1, 1, 1])
    a = ctx.eval_split(hist3, s, scales)
    assert a.found and a.feat == 0
    off3 = np.array([0, 64, 128, 192], np.uint32)
    _same(a, oracle.best_split(hist3, off3, s, scales))


@pytest.mark.parametrize("seed", range(4))
def test_categorical_split_matches_oracle(oracle, seed):
    rng = np.random.default_rng(200 + seed)
    nbins = [3, 64, 256, 12]  # one-hot (< 4), partition, a numeric, partition
    cat = np.array([1, 1, 0, 1], np.uint8)
    bins, widths, hist, s, scales, off = _node_case(oracle, rng, 4000, nbins)
    ctx = Ctx(bins, nbins, widths, categorical=cat)
    for mct in (64, 5):
        got = ctx.eval_split(hist, s, scales, max_cat_threshold=mct)
        want = oracle.best_split(hist, off, s, scales, categorical=cat, max_cat_threshold=mct)
        _same(got, want)
        if got.found and got.categorical:
            assert list(got.cats) == list(want.cats)
    en = np.array([1, 1, 0, 1], np.uint8)
    got = ctx.eval_split(hist, s, scales, enabled=en)
    want = oracle.best_split(hist, off, s, scales, categorical=cat, enabled=en)
    _same(got, want)
    assert got.found and got.categorical and list(got.cats) == list(want.cats)


@pytest.mark.parametrize("n", [1, 4095, 4096, 4097, 100000])
def test_partition_is_stable(n):
    rng = np.random.default_rng(n)
    nbins = [256, 300]
    bins, widths = random_bins(rng, max(n, 10), nbins)
    ctx = Ctx(bins, nbins, widths)
    rows = np.sort(rng.choice(bins.shape[1], n, replace=False)).astype(np.uint32)
    for feat, b, ml in ((0, 100, False), (1, 7, True), (0, 0, True), (1, 301, False)):
        out, nl = ctx.partition(rows, feat, b, ml)
        v = bins[feat][rows]
        miss = 65535 if widths[feat] == 2 else 255
        left = np.where(v == miss, ml, v < b)
        want = np.concatenate([rows[left], rows[~left]])
        assert nl == left.sum()
        assert np.array_equal(out, want)


def test_categorical_partition_sends_the_set_right():
    rng = np.random.default_rng(9)
    bins, widths = random_bins(rng, 9000, [64])
    ctx = Ctx(bins, [64], widths, categorical=[1])
    cats = np.zeros(8, np.uint32)
    for c in (1, 5, 33, 63):
        cats[c // 32] |= np.uint32(1 << (c % 32))
    rows = np.arange(9000, dtype=np.uint32)
    out, nl = ctx.partition(rows, 0, 0, True, cats)
    v = bins[0]
    inset = np.isin(v, [1, 5, 33, 63])
    left = np.where(v == 255, True, ~inset)
    assert nl == left.sum() and np.array_equal(out, np.concatenate([rows[left], rows[~left]]))


def test_multiclass_gradients_and_quantize_match_oracle(oracle):
    # tests/gpu_histogram.rs:2666-2720: class-major K base margins, softmax
    # gradients of all classes, then per class the sampled bounds, scales and
    # root sum (the tree index keys the row sampling)
    import ctypes as C
    from gpu_util import check, lib
    from ferrisboost_b200 import _lib
    from test_multiclass_oracle import fixture
    K, n = 5, 3000
    _, y, w = fixture(n, 4, K)
    rng = np.random.default_rng(4)
    bins, widths = random_bins(rng, n, [8, 8])
    margins = np.array([0.3 * c - 0.7 for c in range(K)], np.float32)
    ctx = Ctx(bins, [8, 8], widths)
    yy = np.ascontiguousarray(y, np.float32)
    ww = np.ascontiguousarray(w, np.float32)
    check(lib().fbgpu_set_labels(ctx.h, _lib.ptr(yy, C.c_float), _lib.ptr(ww, C.c_float), None, 0.0), ctx.h)
    check(lib().fbgpu_set_outputs(ctx.h, K, _lib.ptr(margins, C.c_float)), ctx.h)
    check(lib().fbgpu_multiclass_gradients(ctx.h, 0), ctx.h)
    grads = oracle.softmax_gradients(np.repeat(margins[:, None], n, axis=1), y, w)
    for rate, cls, tree in ((1.0, 0, 0), (1.0, 3, 3), (0.6, 2, 7)):
        th = (1 << 64) - 1 if rate >= 1.0 else int(rate * (1 << 53))
        sc = np.zeros(2, np.float64)
        sm = np.zeros(2, np.int64)
        check(lib().fbgpu_quantize_class(ctx.h, cls, th, 6, tree, 0, _lib.ptr(sc, C.c_double),
                                         _lib.ptr(sm, C.c_int64)), ctx.h)
        g = grads[cls].copy()
        if rate < 1.0:  # data/subsample.rs:45-78 row hash keyed by the tree index
            def mix(z):
                z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9 & (2**64 - 1)
                z = (z ^ (z >> 27)) * 0x94D049BB133111EB & (2**64 - 1)
                return z ^ (z >> 31)
            rot = lambda x, r: ((x << r) | (x >> (64 - r))) & (2**64 - 1)
            for i in range(n):
                hsh = mix(6 ^ rot(tree * 0x9E3779B97F4A7C15 & (2**64 - 1), 23) ^ (i * 0xD6E8FEB86659FD93 & (2**64 - 1)))
                if (hsh >> 11) >= th:
                    g[i] = 0.0
        want_sc = oracle.quantizer(g.reshape(-1, 2), n)
        _, want_sum = oracle.to_fixed(g.reshape(-1, 2), want_sc)
        assert np.array_equal(sc, want_sc), (cls, sc, want_sc)
        assert np.array_equal(sm, want_sum), (cls, sm, want_sum)
    out = np.zeros((K, n), np.float32)
    check(lib().fbgpu_download_margins(ctx.h, _lib.ptr(out, C.c_float)), ctx.h)
    assert np.array_equal(out, np.repeat(margins[:, None], n, axis=1))
    assert lib().fbgpu_set_output_column(ctx.h, K) != 0

"""The reference's histogram unit tests (src/training/hist.rs tests) on the
CPU oracle's histogram and quantizer: a per-row scalar reference, row
subsets, row order, missing rows kept out of every bin but inside the node
sum, sibling subtraction, 8- and 16-bit codes alike, and fixed point that
neither overflows nor loses the signal when gradients grow or shrink by six
orders of magnitude; and the quantizer's known answers and its refusal of
non-finite pairs (tests/numerical_guards.rs).  The device histogram and
quantize kernels equal the oracle's bit for bit (the GPU kernel tests), so
these properties hold for them too."""
import numpy as np
import pytest

MISS8, MISS16 = 255, 65535


def _block(rng, n, nbins, miss_code, missing_pct=0.1):
    off = np.concatenate([[0], np.cumsum(nbins)]).astype(np.uint32)
    b = np.zeros((len(nbins), n), np.uint16)
    for f, nb in enumerate(nbins):
        b[f] = rng.integers(0, nb, n)
        b[f][rng.random(n) < missing_pct] = miss_code
    return b, off


def _fixed(oracle, rng, n, mult=1.0):
    g = np.stack([rng.uniform(-1, 1, n) * mult, rng.uniform(0.05, 1, n) * mult], 1).astype(np.float32)
    fixed, total = oracle.to_fixed(g, oracle.quantizer(g))
    return fixed, total


def _scalar(b, off, miss, fixed, rows=None):
    """The per-row reference: each row adds its pair to its bin of every
    feature it is not missing in (two's-complement sums)."""
    out = np.zeros((int(off[-1]), 2), np.uint64)
    rows = range(b.shape[1]) if rows is None else rows
    for r in rows:
        for f in range(b.shape[0]):
            if b[f, r] != miss[f]:
                out[off[f] + b[f, r]] += fixed[r].astype(np.uint64)
    return out.astype(np.int64)


def test_all_rows_and_subsets_match_the_scalar_reference(oracle):
    rng = np.random.default_rng(0)
    n = 700
    b, off = _block(rng, n, [4, 7, 2, 16], MISS8)
    miss = np.full(4, MISS8, np.uint16)
    fixed, _ = _fixed(oracle, rng, n)
    assert np.array_equal(oracle.hist(b, off, miss, fixed), _scalar(b, off, miss, fixed))
    rows = np.sort(rng.choice(n, 211, replace=False)).astype(np.uint32)
    assert np.array_equal(oracle.hist(b, off, miss, fixed, rows), _scalar(b, off, miss, fixed, rows))
    # none and the full row list agree
    assert np.array_equal(oracle.hist(b, off, miss, fixed, np.arange(n, dtype=np.uint32)),
                          oracle.hist(b, off, miss, fixed))


def test_row_order_does_not_change_the_result(oracle):
    rng = np.random.default_rng(1)
    n = 2000
    b, off = _block(rng, n, [5, 9, 3], MISS8)
    miss = np.full(3, MISS8, np.uint16)
    fixed, _ = _fixed(oracle, rng, n)
    rows = np.arange(n, dtype=np.uint32)
    want = oracle.hist(b, off, miss, fixed, rows)
    for seed in range(3):
        perm = np.random.default_rng(seed).permutation(rows).astype(np.uint32)
        assert np.array_equal(oracle.hist(b, off, miss, fixed, perm), want)


def test_missing_rows_are_excluded_from_every_bin_and_kept_in_the_node_sum(oracle):
    rng = np.random.default_rng(2)
    n = 1500
    b, off = _block(rng, n, [4, 6, 4], MISS8, missing_pct=0.0)
    b[2, [0, 2, 17]] = MISS8
    miss = np.full(3, MISS8, np.uint16)
    fixed, total = _fixed(oracle, rng, n)
    h = oracle.hist(b, off, miss, fixed)
    per_feat = [h[off[f]:off[f + 1]].astype(np.uint64).sum(axis=0).astype(np.int64) for f in range(3)]
    assert np.array_equal(per_feat[0], total)  # no missing: every row is binned
    missing = fixed[[0, 2, 17]].astype(np.uint64).sum(axis=0).astype(np.int64)
    # node sum - sum of a feature's bins = its missing rows, exactly
    assert np.array_equal((total.astype(np.uint64) - per_feat[2].astype(np.uint64)).astype(np.int64), missing)


def test_siblings_subtract_to_the_parent(oracle):
    rng = np.random.default_rng(3)
    n = 3000
    b, off = _block(rng, n, [8, 3, 12, 5], MISS8)
    miss = np.full(4, MISS8, np.uint16)
    fixed, _ = _fixed(oracle, rng, n)
    left = np.flatnonzero(rng.random(n) < 0.4).astype(np.uint32)
    right = np.setdiff1d(np.arange(n), left).astype(np.uint32)
    parent = oracle.hist(b, off, miss, fixed)
    lh = oracle.hist(b, off, miss, fixed, left)
    derived = (parent.astype(np.uint64) - lh.astype(np.uint64)).astype(np.int64)
    assert np.array_equal(derived, oracle.hist(b, off, miss, fixed, right))


def test_sixteen_bit_codes_accumulate_like_eight_bit_codes(oracle):
    rng = np.random.default_rng(4)
    n = 1200
    b8, off = _block(rng, n, [6, 200, 3], MISS8)
    b16 = b8.copy()
    b16[b16 == MISS8] = MISS16
    fixed, _ = _fixed(oracle, rng, n)
    a = oracle.hist(b8, off, np.full(3, MISS8, np.uint16), fixed)
    c = oracle.hist(b16, off, np.full(3, MISS16, np.uint16), fixed)
    assert np.array_equal(a, c)
    # wide features: codes above 255 land in their own bins
    wide, woff = _block(rng, n, [300, 1024], MISS16)
    wm = np.full(2, MISS16, np.uint16)
    assert np.array_equal(oracle.hist(wide, woff, wm, fixed), _scalar(wide, woff, wm, fixed))


@pytest.mark.parametrize("mult", [1e-6, 1.0, 1e6])
def test_extreme_gradient_magnitudes_neither_overflow_nor_lose_the_signal(oracle, mult):
    n = 1000
    i = np.arange(n)
    g = np.stack([((i % 17) - 8.0) * mult, ((i % 5) + 1.0) * mult], 1).astype(np.float32)
    scales = oracle.quantizer(g)
    fixed, total = oracle.to_fixed(g, scales)
    grad, hess = total[0] / scales[0], total[1] / scales[1]
    want_g = g[:, 0].astype(np.float64).sum()
    want_h = g[:, 1].astype(np.float64).sum()
    tol = 1e-9 * max(abs(want_h), 1e-30 * mult)
    assert abs(grad - want_g) <= max(tol, 1e-9 * abs(want_g)), (mult, grad, want_g)
    assert abs(hess - want_h) <= max(tol, 1e-9 * abs(want_h)), (mult, hess, want_h)


def test_quantizer_known_answers(oracle):
    """tests/numerical_guards.rs:119-149: scale = 2^floor(log2((2^62 / n_rows)
    / max|v|)) per channel; with 4 rows, max|g| = 2 and max|h| = 0.25 that is
    2^59 and 2^62, and the fixed-point values are exact."""
    g = np.array([[1.5, 0.125], [-2.0, 0.25]], np.float32)
    scales = oracle.quantizer(g, 4)
    assert scales[0] == 2.0 ** 59 and scales[1] == 2.0 ** 62
    fixed, _ = oracle.to_fixed(g, scales)
    assert fixed.tolist() == [[864_691_128_455_135_232, 576_460_752_303_423_488],
                              [-1_152_921_504_606_846_976, 1_152_921_504_606_846_976]]
    tiny = np.array([[np.finfo(np.float32).tiny, np.finfo(np.float32).tiny]], np.float32)
    s = oracle.quantizer(tiny, 1)
    assert np.all(np.isfinite(s)) and np.all(s > 0)


@pytest.mark.parametrize("bad", [np.nan, np.inf, -np.inf])
def test_quantizer_rejects_nonfinite_pairs(oracle, bad):
    """tests/numerical_guards.rs:77-101."""
    for pair in ([bad, 1.0], [1.0, bad]):
        with pytest.raises(ValueError, match="non-finite"):
            oracle.quantizer(np.array([pair], np.float32), 1)

"""The default base score's label mean (objective.rs:41-61): an f64 sum of
label / n in row order.  For labels with one value besides zero the library
evaluates that sequence by whole binades instead of one addition per row;
these cases check that it lands on the row loop's f64 value exactly
(np.add.accumulate is the row loop: a strictly sequential f64 sum)."""
import ctypes as C

import numpy as np
import pytest

from ferrisboost_b200 import _lib, lib


def _row_loop(y):
    terms = y.astype(np.float64) / np.float64(len(y))
    return float(np.add.accumulate(terms)[-1]) if len(y) else 0.0


def _lib_f64(y):
    y = np.ascontiguousarray(y, dtype=np.float32)
    return lib().fb_label_mean_f64(_lib.ptr(y, C.c_float), len(y))


@pytest.mark.parametrize("n", [1, 2, 3, 7, 64, 1000, 4097, 1 << 20, (1 << 20) + 1, 3_000_017])
@pytest.mark.parametrize("v", [1.0, 0.3, -2.5, 3.0, 1e30, 1.5e-38, 0.1])
@pytest.mark.parametrize("frac", [0.0, 0.001, 0.37, 0.5, 1.0])
def test_two_valued_labels_match_the_row_loop(n, v, frac):
    rng = np.random.default_rng(n ^ int(frac * 1000))
    y = np.where(rng.random(n) < frac, np.float32(v), np.float32(0)).astype(np.float32)
    if n > 5:
        y[rng.integers(0, n, 3)] = np.float32(-0.0)  # signed zeros are zero terms too
    assert _lib_f64(y) == _row_loop(y)


def test_configs1_sized_binary_labels():
    rng = np.random.default_rng(0)
    n = 11_000_000
    y = (rng.random(n) < 0.53).astype(np.float32)
    want = _row_loop(y)
    assert _lib_f64(y) == want
    got32 = lib().fb_label_mean(_lib.ptr(y, C.c_float), None, n)
    assert np.float32(got32) == np.float32(want)


@pytest.mark.parametrize("case", ["three_values", "negative_and_positive", "nan", "inf", "all_zero", "empty"])
def test_other_labels_take_the_row_loop(case):
    rng = np.random.default_rng(1)
    n = 100_003
    y = rng.integers(0, 2, n).astype(np.float32)
    if case == "three_values":
        y[::7] = 2.0
    elif case == "negative_and_positive":
        y[::5] = -1.0
    elif case == "nan":
        y[10] = np.nan
    elif case == "inf":
        y[10] = np.inf
    elif case == "all_zero":
        y[:] = 0.0
    else:
        y = y[:0]
    got, want = _lib_f64(y), _row_loop(y)
    assert got == want or (np.isnan(got) and np.isnan(want))


def test_powers_of_two_and_ties():
    # n a power of two makes 1 / n exact, so the terms sit on binade grids and
    # the sums meet round-half cases
    for n in (2, 8, 1 << 10, 1 << 24, (1 << 24) + 2):
        for v in (1.0, 3.0, 5.0, 0.75):
            y = np.full(n, np.float32(v), np.float32)
            y[::3] = 0.0
            assert _lib_f64(y) == _row_loop(y), (n, v)


def test_random_values_and_sizes():
    rng = np.random.default_rng(7)
    for _ in range(200):
        n = int(rng.integers(1, 200_000))
        v = np.float32(rng.choice([-1, 1]) * 10.0 ** rng.uniform(-30, 30))
        y = np.where(rng.random(n) < rng.random(), v, np.float32(0)).astype(np.float32)
        assert _lib_f64(y) == _row_loop(y), (n, v)

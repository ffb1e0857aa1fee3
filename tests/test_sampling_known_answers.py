"""The reference's sampling unit tests on the CPU oracle's samplers:
colsample_bytree (src/data/colsample.rs tests: the XGBoost count rule,
identity at rate 1, sorted distinct ids, reproducibility and sensitivity to
seed and round) and subsample (src/data/subsample.rs tests: per-row Bernoulli
draws, independent of traversal order, a realised count that varies by tree,
a kept fraction that tracks the rate).  The device kernels are held to these
samplers through byte-identical models trained with subsample and
colsample_bytree (the GPU training tests)."""
import numpy as np
import pytest


@pytest.mark.parametrize("nf,rate,want", [
    (300, 0.1, 30), (300, 0.3, 90), (28, 0.7, 19), (10, 0.99, 9),  # truncation, not rounding
    (300, 0.0001, 1), (300, 0.0, 1), (1, 0.5, 1),  # at least one feature
])
def test_count_truncates_and_keeps_at_least_one(oracle, nf, rate, want):
    """colsample.rs: max(1, (int)(rate * n)), as XGBoost does."""
    assert len(oracle.sample_features(nf, rate, 7, 0)) == want


def test_rate_one_returns_every_feature_in_order(oracle):
    assert np.array_equal(oracle.sample_features(64, 1.0, 7, 3), np.arange(64))


def test_sample_is_sorted_distinct_and_right_sized(oracle):
    for rnd in range(8):
        s = oracle.sample_features(300, 0.1, 42, rnd)
        assert len(s) == 30 and np.all(np.diff(s.astype(np.int64)) > 0) and s.max() < 300


def test_same_seed_and_round_reproduce_and_others_differ(oracle):
    a = oracle.sample_features(300, 0.3, 11, 5)
    assert np.array_equal(a, oracle.sample_features(300, 0.3, 11, 5))
    assert not np.array_equal(a, oracle.sample_features(300, 0.3, 12, 5))
    assert not np.array_equal(a, oracle.sample_features(300, 0.3, 11, 6))


def test_features_are_drawn_uniformly(oracle):
    """Fisher-Yates over the ids: every feature is picked about as often."""
    counts = np.zeros(20, np.int64)
    for rnd in range(4000):
        counts[oracle.sample_features(20, 0.25, 3, rnd)] += 1
    assert counts.sum() == 4000 * 5
    assert np.all(np.abs(counts / 4000 - 0.25) < 0.03), counts


def test_rate_one_keeps_every_row(oracle):
    assert oracle.rows_selected(64, 1.0, 9, 5).all()


def test_row_draws_reproduce_and_depend_on_tree_and_seed(oracle):
    a = oracle.rows_selected(500, 0.5, 11, 2)
    assert np.array_equal(a, oracle.rows_selected(500, 0.5, 11, 2))
    assert not np.array_equal(a, oracle.rows_selected(500, 0.5, 11, 3))
    assert not np.array_equal(a, oracle.rows_selected(500, 0.5, 12, 2))


def test_row_draw_is_per_row(oracle):
    """A row's draw depends on its index only, so a prefix of the rows gets
    the same draws as the whole (any traversal or split of the rows)."""
    full = oracle.rows_selected(1000, 0.3, 5, 1)
    assert np.array_equal(oracle.rows_selected(300, 0.3, 5, 1), full[:300])


def test_realized_count_varies_by_tree(oracle):
    counts = [int(oracle.rows_selected(10_000, 0.5, 1, t).sum()) for t in range(8)]
    assert len(set(counts)) > 1, counts
    assert all(4700 <= c < 5300 for c in counts), counts


@pytest.mark.parametrize("rate", [0.1, 0.25, 0.5, 0.9])
def test_kept_fraction_tracks_the_rate(oracle, rate):
    frac = oracle.rows_selected(200_000, rate, 3, 0).mean()
    assert abs(frac - rate) < 0.01, (rate, frac)

"""The reference's extreme-value tests (tests/extreme_split.rs) on the CPU
oracle and the engine's host data path: a feature of one bin whose values
sit next to f32::MAX (or at f32::MIN) still splits from its missing values,
with the same gain, covers and leaf values; the engine bins such values as
the oracle does; f32::MAX itself, reserved as the upper split sentinel, and
+-inf are refused by every dense entry point; the models load and write back
byte for byte."""
import json

import numpy as np
import pytest

import ferrisboost_b200 as fb

F32_MAX = np.finfo(np.float32).max
BELOW_MAX = np.nextafter(F32_MAX, np.float32(0), dtype=np.float32)
F32_MIN = np.finfo(np.float32).min
LABELS = np.array([1.0, 1.0, 0.0, 0.0], np.float32)


def _train_one_feature(oracle, value, n_rounds=1, eta=1.0):
    """extreme_split.rs:11-38: 4 rows (two of `value`, two missing), max_bin
    1, depth 1, lambda 1, min_child_weight 0, squared error, base_score 0.5."""
    X = np.array([[value], [value], [np.nan], [np.nan]], np.float32)
    return X, oracle.train(X, LABELS, objective="reg:squarederror", n_rounds=n_rounds, max_depth=1, max_bin=1,
                           eta=eta, reg_lambda=1.0, min_child_weight=0.0, base_score=0.5, nthread=1)


def _tree(ref, t=0):
    return json.loads(ref.json())["learner"]["gradient_booster"]["model"]["trees"][t]


@pytest.mark.parametrize("value", [BELOW_MAX, F32_MIN])
def test_one_bin_feature_still_splits_from_missing(oracle, value):
    """extreme_split.rs:40-101 assert_binary_split."""
    X, ref = _train_one_feature(oracle, value)
    t = _tree(ref)
    assert ref.num_trees == 1 and len(t["left_children"]) == 3
    assert (t["left_children"][0], t["right_children"][0]) == (1, 2)
    assert t["left_children"][1] == t["left_children"][2] == -1
    assert abs(t["loss_changes"][0] - 2.0 / 3.0) < 1e-6
    assert t["sum_hessian"][0] == 4.0
    assert abs(t["sum_hessian"][1] - 2.0) < 1e-6 and abs(t["sum_hessian"][2] - 2.0) < 1e-6
    m = ref.predict_margin(X)
    assert abs(m[0] - 0.8333333) < 1e-6 and abs(m[2] - 0.16666666) < 1e-6
    # the engine writes the oracle's model back byte for byte
    assert fb.Model.load_model(ref.json()).to_json() == ref.json()


@pytest.mark.parametrize("value", [BELOW_MAX, F32_MIN])
def test_engine_bins_extreme_values_like_the_oracle(oracle, value):
    X = np.array([[value], [value], [np.nan], [np.nan]], np.float32)
    ds = fb.Dataset(X, max_bin=1)
    cuts, off = ds.cuts()
    rc, ro = oracle.sketch(X, 1)
    assert np.array_equal(off, ro) and np.array_equal(cuts.view(np.uint32), rc.view(np.uint32))
    assert off[1] - off[0] == 0  # one bin: no interior cut
    col = ds.column(0)
    assert np.array_equal(col, oracle.quantize(X, rc, ro)[0])
    assert col[0] == col[1] and col[2] == col[3] and col[0] != col[2]


def test_multiround_extreme_model_separates_and_round_trips(oracle):
    """extreme_split.rs:103-150: three rounds at eta 0.5; the finite value
    scores above the missing one; the saved model reads back to the same
    bytes."""
    X, ref = _train_one_feature(oracle, BELOW_MAX, n_rounds=3, eta=0.5)
    assert ref.num_trees == 3
    m = ref.predict_margin(X)
    assert m[0] > m[2]
    assert fb.Model.load_model(ref.json()).to_json() == ref.json()


def test_exact_f32_max_is_rejected_by_dense_entry_points():
    """extreme_split.rs:56-73: f32::MAX is the finite upper split sentinel, so
    a feature value equal to it is refused, whether the cuts are sketched or
    given."""
    X = np.array([[F32_MAX], [F32_MAX], [np.nan], [np.nan]], np.float32)
    with pytest.raises(ValueError, match="f32::MAX"):
        fb.Dataset(X, max_bin=1)
    given = (np.array([0.0], np.float32), np.array([0, 1], np.uint32))
    with pytest.raises(ValueError, match="f32::MAX"):
        fb.Dataset(X, max_bin=1, cuts=given)


def test_infinite_training_features_are_rejected():
    """python/mod.rs:4063-4073 reject_inf: training data (and validation sets,
    binned with given cuts) cannot hold +-inf; missing values are NaN."""
    for v in (np.inf, -np.inf):
        X = np.array([[1.0], [2.0], [v], [np.nan]], np.float32)
        with pytest.raises(ValueError, match="inf"):
            fb.Dataset(X, max_bin=4)
        with pytest.raises(ValueError, match="inf"):
            fb.Dataset(X, cuts=(np.array([1.5], np.float32), np.array([0, 1], np.uint32)))


def test_find_bin_does_not_wrap_above_255_bins(oracle):
    """columns.rs width_grouping_tests find_bin_does_not_wrap_above_255_bins:
    599 cuts (600 bins, 16-bit codes); 0.5, 300 and 1e9 fall in bins 0, 300
    and 599, with the cuts given, in the engine and the oracle."""
    cuts = np.arange(1, 600, dtype=np.float32)
    off = np.array([0, 599], np.uint32)
    X = np.array([[0.5], [300.0], [1e9], [np.nan]], np.float32)
    ds = fb.Dataset(X, cuts=(cuts, off))
    col = ds.column(0)
    assert col[:3].tolist() == [0, 300, 599]
    assert np.array_equal(col, oracle.quantize(X, cuts, off)[0])

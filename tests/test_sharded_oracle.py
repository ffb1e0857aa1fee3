"""The multi-GPU training algorithm, with threads as ranks on the CPU
(oracle rc_train_sharded): rows sharded over N ranks, per-level partial
histograms summed by a fake collective, the accumulated child chosen by the
children's global hessian sums instead of row counts, and optionally the
split search sharded by feature range with the per-node winners gathered.
Integer sums do not depend on how the rows are split, so every variant must
give the unsharded model byte for byte (north_star: exact-mode models
identical at any GPU count)."""
import numpy as np
import pytest


def _data(seed, n=6000, F=9, missing=0.03):
    rng = np.random.default_rng(seed)
    X = rng.standard_normal((n, F)).astype(np.float32)
    X[rng.random(X.shape) < missing] = np.nan
    z = np.nan_to_num(X[:, 0]) - 0.7 * np.nan_to_num(X[:, 1]) * np.nan_to_num(X[:, 2]) + 0.3 * np.nan_to_num(X[:, 3])
    y = (rng.random(n) < 1 / (1 + np.exp(-z))).astype(np.float32)
    return X, y


CASES = {
    "logistic": dict(objective="binary:logistic", max_depth=6, eta=0.3, max_bin=64),
    "squared_error_weights": dict(objective="reg:squarederror", max_depth=5, eta=0.2, max_bin=32),
    "colsample_subsample": dict(objective="binary:logistic", max_depth=6, eta=0.3, max_bin=64,
                                colsample_bytree=0.6, subsample=0.8, seed=3),
    "max_leaves": dict(objective="binary:logistic", max_depth=7, eta=0.3, max_bin=64, max_leaves=20),
    "monotone": dict(objective="binary:logistic", max_depth=5, eta=0.3, max_bin=32,
                     monotone_constraints=[1, -1, 0, 0, 0, 0, 0, 0, 0]),
    "categorical": dict(objective="reg:squarederror", max_depth=6, eta=0.3, max_bin=64),
}


@pytest.mark.parametrize("name", sorted(CASES))
@pytest.mark.parametrize("ranks", [2, 3, 8])
@pytest.mark.parametrize("feature_sharded", [False, True])
def test_sharded_training_equals_single(oracle, name, ranks, feature_sharded):
    X, y = _data(sum(map(ord, name)))
    p = dict(CASES[name])
    w = None
    if name == "squared_error_weights":
        w = np.random.default_rng(1).uniform(0.2, 3.0, len(y)).astype(np.float32)
        y = (np.nan_to_num(X[:, 0]) + np.random.default_rng(2).normal(0, 0.3, len(y))).astype(np.float32)
    if name == "categorical":
        X[:, 7] = np.random.default_rng(4).integers(0, 40, len(X))
        X[:, 8] = np.random.default_rng(5).integers(0, 3, len(X))
        y = (np.nan_to_num(X[:, 0]) + np.sin(X[:, 7])).astype(np.float32)
        p["categorical"] = np.array([0] * 7 + [1, 1], np.uint8)
    want = oracle.train(X, y, w, n_rounds=6, **p).json()
    got = oracle.train_sharded(X, y, w, ranks=ranks, feature_sharded=feature_sharded, n_rounds=6, **p).json()
    assert got == want


def test_hessian_choice_differs_from_row_counts_yet_models_agree(oracle):
    # weights make the child with fewer rows the heavier one, so the sharded
    # rule (smaller hessian sum) accumulates the other child than the
    # reference's rule (fewer rows); the integers, hence the model, agree
    X, y = _data(9, n=4000)
    w = np.where(np.nan_to_num(X[:, 0]) > 0.5, 20.0, 0.1).astype(np.float32)
    p = dict(objective="binary:logistic", max_depth=6, eta=0.3, max_bin=64)
    want = oracle.train(X, y, w, n_rounds=4, **p).json()
    for ranks in (1, 2, 5):
        assert oracle.train_sharded(X, y, w, ranks=ranks, n_rounds=4, **p).json() == want

"""The reference's training unit tests (src/training/mod.rs tests) on the
CPU oracle and the engine's host base score: the default base score is the
label mean (f64, row order) or the weighted mean, 0.5 when every weight is
zero, and 1 for all-positive logistic labels with a finite margin; a
root-only round feeds the next round's gradients; leaf Hessians sum back to
the root; trees keep max_depth; nothing to learn gives a single leaf; and
training is reproducible."""
import json
import math

import numpy as np
import pytest

import ferrisboost_b200 as fb
from ferrisboost_b200 import _lib


def _learner(ref):
    return json.loads(ref.json())["learner"]


def _base_score(ref):
    return np.float32(float(_learner(ref)["learner_model_param"]["base_score"]))


def _trees(ref):
    return _learner(ref)["gradient_booster"]["model"]["trees"]


def _label_mean(y, w=None):
    """objective.rs:41-61 FitInterceptGlmLike: sum of y/n (or y/sw * w) in
    f64, row order, rounded to f32; 0.5 when the weights sum to zero."""
    if w is None:
        acc = 0.0
        for v in y:
            acc += float(v) / len(y)
        return np.float32(acc)
    sw = 0.0
    for v in w:
        sw += float(v)
    if sw <= 0.0:
        return np.float32(0.5)
    acc = 0.0
    for v, wi in zip(y, w):
        acc += float(v) / sw * float(wi)
    return np.float32(acc)


def _engine_mean(y, w=None):
    y = np.ascontiguousarray(y, np.float32)
    w = None if w is None else np.ascontiguousarray(w, np.float32)
    return np.float32(fb.lib().fb_label_mean(_lib.ptr(y, _lib.C.c_float), _lib.ptr(w, _lib.C.c_float), len(y)))


@pytest.mark.parametrize("objective", ["reg:squarederror", "binary:logistic"])
def test_default_base_score_is_the_weighted_label_mean(oracle, objective):
    """mod.rs:5597-5649."""
    i = np.arange(40)
    X = (i % 7).astype(np.float32)[:, None]
    y = (i % 3 == 0).astype(np.float32)
    w = np.where(i % 3 == 0, 3.0, 0.5 + (i % 4)).astype(np.float32)
    m = oracle.train(X, y, objective=objective, max_depth=2, n_rounds=1, max_bin=255)
    assert _base_score(m) == _label_mean(y) == _engine_mean(y)
    mw = oracle.train(X, y, w, objective=objective, max_depth=2, n_rounds=1, max_bin=255)
    assert _base_score(mw) == _label_mean(y, w) == _engine_mean(y, w)
    assert _base_score(mw) != _label_mean(y)
    assert _label_mean(y, np.zeros(40, np.float32)) == _engine_mean(y, np.zeros(40, np.float32)) == 0.5


def test_all_positive_logistic_labels_give_a_clamped_finite_margin(oracle):
    X = (np.arange(40) % 7).astype(np.float32)[:, None]
    m = oracle.train(X, np.ones(40, np.float32), objective="binary:logistic", max_depth=2, n_rounds=1)
    assert _base_score(m) == 1.0
    assert np.isfinite(m.predict_margin(X)).all()


def test_root_only_tree_updates_the_next_round(oracle):
    """mod.rs:5651-5674: with max_depth 0 the root is the leaf; round two
    sees round one's predictions, so its leaf is smaller but still positive."""
    X = np.zeros((8, 1), np.float32)
    m = oracle.train(X, np.ones(8, np.float32), objective="reg:squarederror", max_depth=0, n_rounds=2, eta=0.3,
                     base_score=0.5)
    t0, t1 = _trees(m)
    first, second = t0["split_conditions"][0], t1["split_conditions"][0]
    assert 0.0 < second < first


def _step_data(n):
    rng = np.random.default_rng(0)
    X = rng.uniform(0, 1, (n, 3)).astype(np.float32)
    y = (X[:, 0] > 0.5).astype(np.float32)
    return X, y


def test_leaf_hessians_sum_back_to_the_root(oracle):
    X, y = _step_data(100)
    m = oracle.train(X, y, objective="binary:logistic", max_depth=4, n_rounds=3)
    for k, t in enumerate(_trees(m)):
        root = t["sum_hessian"][0]
        leaves = sum(h for h, c in zip(t["sum_hessian"], t["left_children"]) if c == -1)
        assert abs(leaves - root) < 1e-3 * max(root, 1.0), k


def _depth(t, i=0):
    if t["left_children"][i] == -1:
        return 0
    return 1 + max(_depth(t, t["left_children"][i]), _depth(t, t["right_children"][i]))


def test_respects_max_depth(oracle):
    X, y = _step_data(100)
    for d in (0, 1, 2, 4):
        m = oracle.train(X, y, objective="binary:logistic", max_depth=d, n_rounds=2)
        assert all(_depth(t) <= d for t in _trees(m)), d


def test_nothing_to_learn_gives_a_single_leaf(oracle):
    X = np.random.default_rng(1).standard_normal((64, 3)).astype(np.float32)
    m = oracle.train(X, np.full(64, 0.7, np.float32), objective="reg:squarederror", max_depth=4, n_rounds=2)
    assert all(len(t["left_children"]) == 1 for t in _trees(m))


def test_training_is_reproducible(oracle):
    X, y = _step_data(500)
    kw = dict(objective="binary:logistic", max_depth=4, n_rounds=4, subsample=0.7, colsample_bytree=0.67, seed=3)
    assert oracle.train(X, y, **kw).json() == oracle.train(X, y, **kw).json()


def _weight_toy(n=400, m=5, seed=0):
    """python/tests/test_weights.py toy: integer features, so dropping rows
    or zeroing their weights leaves the bins unchanged."""
    rng = np.random.default_rng(seed)
    x = rng.integers(0, 8, size=(n, m)).astype(np.float32)
    y = (x[:, 0] - x[:, 1] + rng.normal(0, 0.5, n) > 0).astype(np.float32)
    w = rng.uniform(0.1, 3.0, n).astype(np.float32)
    return x, y, w


_WKW = dict(objective="binary:logistic", max_depth=3, eta=0.3, nthread=1, n_rounds=5)


def test_all_ones_weight_is_byte_identical_and_weights_change_the_model(oracle):
    """test_weights.py:34-46."""
    x, y, w = _weight_toy()
    plain = oracle.train(x, y, **_WKW).json()
    assert oracle.train(x, y, np.ones(len(y), np.float32), **_WKW).json() == plain
    assert oracle.train(x, y, w, **_WKW).json() != plain


def test_zero_weight_rows_match_dropping_them(oracle):
    """test_weights.py:48-55: predictions equal (here the models are equal
    byte for byte too)."""
    x, y, w = _weight_toy()
    keep = np.arange(len(y)) % 3 != 0
    zeroed = oracle.train(x, y, np.where(keep, w, 0.0).astype(np.float32), **_WKW)
    dropped = oracle.train(x[keep], y[keep], w[keep], **_WKW)
    assert np.array_equal(zeroed.predict_margin(x), dropped.predict_margin(x))
    assert zeroed.json() == dropped.json()


def _newton_base_score(objective, y, w, spw):
    """objective.rs:403-493 with scale_pos_weight != 1: pairs at margin 0
    times the gradient weights in f32, summed in f64; -G / max(H, 1e-6f) to
    f32, through the transform."""
    y = np.asarray(y, np.float32)
    gw = (np.ones_like(y) if w is None else np.asarray(w, np.float32)) * np.where(y == 1.0, np.float32(spw),
                                                                               np.float32(1.0)).astype(np.float32)
    gw = gw.astype(np.float32)
    if objective == "binary:logistic":
        g, h = (np.float32(0.5) - y), np.full_like(y, np.float32(0.25))
    else:
        g, h = (np.float32(0.0) - y), np.ones_like(y)
    sg = sh = 0.0
    for gi, hi in zip((g * gw).astype(np.float32), (h * gw).astype(np.float32)):
        sg += float(gi)
        sh += float(hi)
    m = np.float32(-sg / max(sh, float(np.float32(1e-6))))
    if objective == "binary:logistic":
        e = np.float32(math.exp(-float(m)))  # expf, correctly rounded (glibc's, which Rust's f32::exp calls)
        return np.float32(np.float32(1.0) / (np.float32(1.0) + e))
    return m


@pytest.mark.parametrize("objective", ["binary:logistic", "reg:squarederror"])
@pytest.mark.parametrize("spw", [0.3, 4.0, 1.0])
@pytest.mark.parametrize("weighted", [False, True])
def test_scale_pos_weight_base_score(oracle, objective, spw, weighted):
    """python/tests/test_regularization.py:79-91: with scale_pos_weight != 1
    the default base score is XGBoost's one-step Newton estimate
    (FitIntercept), with 1 it is the label mean; the oracle's model, the
    engine's host estimate and an independent statement agree bit for bit."""
    rng = np.random.default_rng(5)
    n = 2001
    X = rng.integers(0, 6, (n, 3)).astype(np.float32)
    y = (X[:, 0] + rng.normal(0, 1, n) > 2.5).astype(np.float32)
    w = rng.uniform(0.2, 3, n).astype(np.float32) if weighted else None
    want = _newton_base_score(objective, y, w, spw) if spw != 1.0 else _label_mean(y, w)
    m = oracle.train(X, y, w, objective=objective, scale_pos_weight=spw, max_depth=2, n_rounds=1)
    got = fb.lib().fb_initial_base_score(1 if objective == "binary:logistic" else 0, _lib.ptr(y, _lib.C.c_float),
                                         _lib.ptr(w, _lib.C.c_float), n, spw)
    assert _base_score(m) == np.float32(got) == want, (_base_score(m), got, want)
    if spw != 1.0:
        assert want != _label_mean(y, w)


def test_max_delta_step_bounds_every_leaf(oracle):
    """python/tests/test_regularization.py:104-115: |leaf| <= max_delta_step x
    eta with lambda 0."""
    rng = np.random.default_rng(6)
    X = rng.integers(0, 5, (2000, 4)).astype(np.float32)
    y = (X[:, 0] - X[:, 1] + rng.normal(0, 1, 2000) > 0).astype(np.float32)
    eta, mds = 0.3, 0.2
    m = oracle.train(X, y, objective="binary:logistic", max_delta_step=mds, eta=eta, reg_lambda=0.0, n_rounds=5,
                     max_depth=6)
    for t in _trees(m):
        leaves = [v for v, c in zip(t["split_conditions"], t["left_children"]) if c == -1]
        assert max(abs(v) for v in leaves) <= mds * eta * (1 + 1e-6)


def _wiggly(n=800, m=4, seed=0, missing=0.08):
    """python/tests/test_monotone.py:8-15: a non-monotone truth."""
    rng = np.random.default_rng(seed)
    x = rng.uniform(-2, 2, size=(n, m)).astype(np.float32)
    signal = np.sin(1.7 * x[:, 0]) + 0.8 * np.cos(3 * x[:, 1]) - 0.5 * x[:, 2]
    y = (signal + rng.normal(0, 0.3, n) > 0).astype(np.float32)
    x[rng.random(x.shape) < missing] = np.nan
    return x, y


def _sweep_is_monotone(m, x, constraints):
    grid = np.linspace(-2.2, 2.2, 61, dtype=np.float32)
    for base in x[::23][:30]:
        for f, c in enumerate(constraints):
            if c == 0:
                continue
            rows = np.repeat(base[None, :], len(grid), axis=0)
            rows[:, f] = grid
            d = np.diff(m.predict_margin(rows))
            if (c > 0 and (d < 0).any()) or (c < 0 and (d > 0).any()):
                return False
    return True


def test_monotone_constraints_hold_and_zeros_change_nothing(oracle):
    """python/tests/test_monotone.py:41-58: the unconstrained model breaks
    monotonicity on this data, the constrained one keeps it; all-zero
    constraints give the unconstrained bytes."""
    x, y = _wiggly()
    kw = dict(objective="binary:logistic", max_depth=5, eta=0.3, nthread=1)
    mc = [1, -1, 0, 0]
    free = oracle.train(x, y, n_rounds=20, **kw)
    tied = oracle.train(x, y, n_rounds=20, monotone_constraints=mc, **kw)
    assert not _sweep_is_monotone(free, x, mc)
    assert _sweep_is_monotone(tied, x, mc)
    assert oracle.train(x, y, n_rounds=4, monotone_constraints=[0, 0, 0, 0], **kw).json() == \
        oracle.train(x, y, n_rounds=4, **kw).json()

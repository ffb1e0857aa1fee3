"""Multiclass training and prediction on the device (multi:softprob /
multi:softmax; src/training/mod.rs:2564-2800, objective.rs:1175-1333): exact
mode byte-identical to the CPU oracle's model JSON and margins, the
reference's own multiclass test matrix (tests/gpu_histogram.rs:2828-2914:
K in {2, 3, 7}; weights, row and column sampling, monotone constraints; fast
mode deterministic and within 5e-3 of exact), prediction transforms and
per-class SHAP groups."""
import numpy as np
import pytest

import ferrisboost_b200 as fb
from test_multiclass_oracle import fixture

pytestmark = pytest.mark.gpu


def _params(K, objective="multi:softprob", **kw):
    return dict(dict(objective=objective, num_class=K, max_depth=4, max_bin=32, seed=6), **kw)


CASES = [
    # (K, weighted, subsample, colsample, monotone)
    (2, False, 1.0, 1.0, None),
    (3, True, 0.75, 0.7, None),
    (7, True, 1.0, 1.0, [1, -1, 0, 0, 0, 1]),
    (3, False, 1.0, 1.0, None),
]


@pytest.mark.parametrize("case", range(len(CASES)))
def test_exact_multiclass_byte_identical(oracle, case):
    K, weighted, subsample, colsample, mono = CASES[case]
    X, y, w = fixture(2400, 6, K)
    p = _params(K, subsample=subsample, colsample_bytree=colsample)
    if mono:
        p["monotone_constraints"] = mono
    ww = w if weighted else None
    m = fb.train(p, X, label=y, weight=ww, num_boost_round=4)
    ref = oracle.train(X, y, ww, n_rounds=4, **p)
    assert m.num_trees == 4 * K and m.num_outputs == K
    assert m.to_json() == ref.json()
    got = m.predict(X, output_margin=True)
    assert got.shape == (len(X), K)
    assert np.array_equal(got.view(np.uint32), ref.predict_margin(X).view(np.uint32))


def test_multiclass_larger_mixed_and_lossguide(oracle):
    rng = np.random.default_rng(3)
    n, K = 40000, 5
    X = rng.standard_normal((n, 10)).astype(np.float32)
    X[rng.random(X.shape) < 0.05] = np.nan
    X[:, 8] = rng.integers(0, 12, n)
    z = np.nan_to_num(X[:, :K]) + 0.3 * (X[:, 8:9] % 3)
    y = np.argmax(z + rng.gumbel(size=z.shape), axis=1).astype(np.float32)
    ft = ["q"] * 8 + ["c", "q"]
    cat = np.array([f == "c" for f in ft], np.uint8)
    for p in (_params(K, objective="multi:softmax", max_depth=6, max_bin=256, eta=0.3),
              _params(K, grow_policy="lossguide", max_leaves=12, max_depth=8, max_bin=128, eta=0.2),
              _params(K, base_score=0.5, max_depth=5, max_bin=1024)):
        m = fb.train(p, X, label=y, num_boost_round=5, feature_types=ft)
        ref = oracle.train(X, y, n_rounds=5, categorical=cat, **p)
        assert m.to_json() == ref.json(), p
        assert np.array_equal(m.predict(X[:3000], output_margin=True), ref.predict_margin(X[:3000]))


def test_fast_multiclass_deterministic_and_close_to_exact():
    for K in (2, 3, 7):
        X, y, w = fixture(2400, 6, K)
        p = _params(K, subsample=0.75, colsample_bytree=0.7)
        exact = fb.train(p, X, label=y, weight=w, num_boost_round=4)
        fast = fb.train(dict(p, gpu_math="fast"), X, label=y, weight=w, num_boost_round=4)
        again = fb.train(dict(p, gpu_math="fast"), X, label=y, weight=w, num_boost_round=4)
        assert fast.to_json() == again.to_json()
        assert fast.num_trees == 4 * K
        a = exact.predict(X, output_margin=True).astype(np.float64)
        b = fast.predict(X, output_margin=True).astype(np.float64)
        assert np.abs(b - a).max() < 5e-3, K

        def softmax(m):
            e = np.exp(m - m.max(axis=1, keepdims=True))
            return e / e.sum(axis=1, keepdims=True)
        pa, pb = softmax(a), softmax(b)
        yi = y.astype(np.int64)
        mll = [float(-np.mean(w * np.log(p[np.arange(len(yi)), yi])) / np.mean(w)) for p in (pa, pb)]
        assert abs(mll[1] - mll[0]) < 1e-4, (K, mll)
        rel = np.abs(pb - pa) / pa
        # north_star: fast-mode predictions within 1e-5 relative of exact mode
        assert rel.max() <= 1e-5, (K, f"max {rel.max():.3e}, median {np.median(rel):.3e}, "
                                      f"over {np.count_nonzero(rel > 1e-5)} of {rel.size}")


def test_transforms_shap_and_leaves(oracle):
    K = 4
    X, y, w = fixture(3000, 6, K, seed=9)
    p = _params(K)
    m = fb.train(p, X, label=y, num_boost_round=5)
    ref = oracle.train(X, y, n_rounds=5, **p)
    margins = m.predict(X, output_margin=True)
    prob = m.predict(X)
    # objective.rs:1308-1322: exp(m - max) / (f32) sum in f64
    mx = margins.max(axis=1, keepdims=True)
    e = np.exp((margins - mx).astype(np.float32))
    want = e / e.astype(np.float64).sum(axis=1, keepdims=True).astype(np.float32)
    np.testing.assert_allclose(prob, want, rtol=2e-6, atol=1e-7)
    np.testing.assert_allclose(prob.sum(axis=1), 1.0, atol=1e-5)
    msx = fb.train(dict(p, objective="multi:softmax"), X, label=y, num_boost_round=5)
    cls = msx.predict(X)
    assert cls.shape == (len(X),)
    assert np.array_equal(cls, np.argmax(msx.predict(X, output_margin=True), axis=1).astype(np.float32))
    # SHAP: one group per class, within 1e-5 of the oracle, summing to the class margins
    sh = m.predict(X[:500], pred_contribs=True)
    assert sh.shape == (500, K, X.shape[1] + 1)
    assert np.max(np.abs(sh - ref.shap(X[:500]))) <= 1e-5
    np.testing.assert_allclose(sh.sum(axis=2), margins[:500], atol=1e-4)
    inter = m.predict(X[:50], pred_interactions=True)
    assert inter.shape == (50, K, X.shape[1] + 1, X.shape[1] + 1)
    np.testing.assert_allclose(inter.sum(axis=3), sh[:50], atol=1e-4)
    leaves = m.predict(X[:100], pred_leaf=True)
    assert leaves.shape == (100, 5 * K)
    assert np.array_equal(leaves, ref.pred_leaf(X[:100]))


def test_multiclass_input_errors():
    X, y, w = fixture(500, 4, 3)
    with pytest.raises(ValueError, match="num_class"):
        fb.train({"objective": "multi:softprob"}, X, label=y, num_boost_round=1)
    with pytest.raises(ValueError, match="integers"):
        fb.train(_params(3), X, label=y + 0.5, num_boost_round=1)
    with pytest.raises(ValueError, match="integers"):
        fb.train(_params(2), X, label=y, num_boost_round=1)  # label 2 with num_class 2


def test_repeated_predictions_on_alternating_rows_agree():
    """The rows of a multiclass prediction go to the device once and every
    class's model reads them on its own stream: each call must see its own
    rows, also when the device block it gets last held another call's rows."""
    K = 3
    X, y, _ = fixture(40_000, 8, K, seed=4)
    m = fb.train(_params(K), X, label=y, num_boost_round=4)
    rng = np.random.default_rng(11)
    X2 = rng.standard_normal(X.shape).astype(np.float32)
    first = {0: m.predict(X, output_margin=True), 1: m.predict(X2, output_margin=True)}
    for i in range(12):
        which = i % 2
        got = m.predict(X2 if which else X, output_margin=True)
        assert np.array_equal(got, first[which]), f"call {i}"
    # the probabilities are the softmax of the same call's margins
    prob = m.predict(X)
    e = np.exp((first[0] - first[0].max(axis=1, keepdims=True)).astype(np.float32))
    want = e / e.astype(np.float64).sum(axis=1, keepdims=True).astype(np.float32)
    np.testing.assert_allclose(prob, want, rtol=2e-6, atol=1e-7)

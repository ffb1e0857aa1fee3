"""The oracle's multiclass restatement (multi:softprob / multi:softmax,
src/training/mod.rs:2564-2800 train_multiclass_rounds, objective.rs:1175-1247
softmax_gradients and initial_class_margins, tree.rs:600-750 multi-output
JSON).  The reference ships no multiclass golden vectors, so these checks pin
each piece against an independent statement: the gradient and the base
margins against numpy, the JSON's per-class bookkeeping against its own
trees, the margins against a tree walk of the JSON, and SHAP groups against
their margins."""
import json
import math

import numpy as np
import pytest


def fixture(n, F, K, seed=0):
    """The reference's multiclass test shape (tests/gpu_histogram.rs:2630-2660):
    integer-valued features with a NaN pattern, labels from a row formula,
    weights cycling through 5 values."""
    r = np.arange(n)[:, None]
    f = np.arange(F)[None, :]
    X = ((r * 13 + f * 11) % 41).astype(np.float32)
    X[(r * 7 + f) % 29 == 0] = np.nan
    s = (np.arange(n) * 13) % 41 + (np.arange(n) * 5) % 7
    y = np.minimum(s * K // 48, K - 1).astype(np.float32)
    w = np.array([0.5, 1.0, 2.0, 0.25, 3.0], np.float32)[(np.arange(n) * 3) % 5]
    if seed:
        rng = np.random.default_rng(seed)
        X = X + rng.standard_normal(X.shape).astype(np.float32)
    return X, y, w


def _softmax_ref(m, y, w):
    K, n = m.shape
    wmax = np.maximum(m.max(axis=0), np.finfo(np.float32).tiny)
    e = np.exp((m - wmax).astype(np.float32)).astype(np.float32)
    wsum = e.astype(np.float64).sum(axis=0).astype(np.float32)
    p = (e / wsum).astype(np.float32)
    wt = np.ones(n, np.float32) if w is None else w
    h = np.maximum(((np.float32(2.0) * p) * (np.float32(1.0) - p)) * wt, np.float32(1e-16))
    p = p - (y[None, :] == np.arange(K)[:, None]).astype(np.float32)
    return np.stack([p * wt, h], axis=-1)


@pytest.mark.parametrize("weighted", [False, True])
def test_softmax_gradients_against_numpy(oracle, weighted):
    rng = np.random.default_rng(1)
    K, n = 5, 4000
    m = rng.normal(0, 2, (K, n)).astype(np.float32)
    m[:, :50] = -3.0  # all margins negative: wmax is the smallest positive normal
    y = rng.integers(0, K, n).astype(np.float32)
    w = rng.uniform(0.1, 3, n).astype(np.float32) if weighted else None
    got = oracle.softmax_gradients(m, y, w)
    want = _softmax_ref(m, y, w)
    # numpy's float32 exp and the C library's expf may differ in the last place
    np.testing.assert_allclose(got, want, rtol=4e-7, atol=5e-7)
    assert np.all(got[..., 1] >= 1e-16)


def test_initial_class_margins(oracle):
    rng = np.random.default_rng(2)
    for K, weighted in ((3, False), (7, True), (2, True)):
        y = rng.integers(0, K, 5000).astype(np.float32)
        w = rng.uniform(0, 2, 5000).astype(np.float32) if weighted else None
        got = oracle.class_margins(y, K, w)
        bins = np.zeros(K, np.float32)
        for i in range(len(y)):  # f32 counts in row order
            bins[int(y[i])] += np.float32(1.0) if w is None else w[i]
        sw = float(len(y)) if w is None else math.fsum(float(v) for v in w)
        logs = np.array([np.log(np.float32(b * (1.0 / sw)) + np.float32(1e-6)) for b in bins], np.float32)
        mean = np.float32(0.0)
        for v in logs:
            mean = np.float32(mean + v / np.float32(K))
        np.testing.assert_allclose(got, logs - mean, rtol=0, atol=2e-7)
    assert np.array_equal(oracle.class_margins(np.zeros(3, np.float32), 4, np.zeros(3, np.float32)), np.zeros(4))


def _trees(js):
    out = []
    for t in js["learner"]["gradient_booster"]["model"]["trees"]:
        out.append(dict(left=t["left_children"], right=t["right_children"], feat=t["split_indices"],
                        cond=np.array(t["split_conditions"], np.float32), dleft=t["default_left"]))
    return out


def _leaf(t, x):
    i = 0
    while t["left"][i] >= 0:
        v = x[t["feat"][i]]
        left = bool(t["dleft"][i]) if math.isnan(v) else v < t["cond"][i]
        i = t["left"][i] if left else t["right"][i]
    return t["cond"][i]


@pytest.mark.parametrize("K,objective", [(3, "multi:softprob"), (5, "multi:softmax")])
def test_multiclass_model_json_and_margins(oracle, K, objective):
    X, y, w = fixture(2400, 6, K)
    rounds = 4
    m = oracle.train(X, y, w, objective=objective, num_class=K, n_rounds=rounds, max_depth=4, max_bin=32, seed=6)
    js = json.loads(m.json())
    gb = js["learner"]["gradient_booster"]["model"]
    assert m.num_trees == rounds * K and m.num_outputs == K
    assert gb["tree_info"] == [i % K for i in range(rounds * K)]
    assert gb["iteration_indptr"] == list(range(0, rounds * K + 1, K))
    lp = js["learner"]["learner_model_param"]
    assert lp["num_class"] == str(K)
    base = [float(v) for v in lp["base_score"].strip("[]").split(",")]
    assert len(base) == K
    assert js["learner"]["objective"] == {"name": objective, "softmax_multiclass_param": {"num_class": str(K)}}
    margins = m.predict_margin(X[:200])
    trees = _trees(js)
    base32 = oracle.class_margins(y, K, w)
    assert np.array_equal(np.array(base, np.float32), base32)
    for r in range(0, 200, 17):
        want = base32.copy()
        for t, tree in enumerate(trees):
            want[t % K] = np.float32(want[t % K] + _leaf(tree, X[r]))
        assert np.array_equal(margins[r], want)
    # the classes are learned
    acc = np.mean(np.argmax(m.predict_margin(X), axis=1) == y)
    assert acc > 1.5 / K
    # SHAP: one group per class, each summing to its margin
    sh = m.shap(X[:100])
    assert sh.shape == (100, K, X.shape[1] + 1)
    np.testing.assert_allclose(sh.sum(axis=2), m.predict_margin(X[:100]), atol=2e-4)


def test_multiclass_base_score_and_label_checks(oracle):
    X, y, w = fixture(600, 4, 3)
    m = oracle.train(X, y, objective="multi:softprob", num_class=3, n_rounds=2, base_score=0.25, max_depth=3)
    assert json.loads(m.json())["learner"]["learner_model_param"]["base_score"] == "[0.25,0.25,0.25]"
    with pytest.raises(RuntimeError, match="integers"):
        oracle.train(X, y + 0.5, objective="multi:softprob", num_class=3, n_rounds=1)
    with pytest.raises(RuntimeError, match="num_class"):
        oracle.train(X, y, objective="multi:softprob", num_class=1, n_rounds=1)


def test_engine_class_margins_equal_the_oracle(oracle):
    # the engine's host restatement (fb_class_margins, used by row-sharded
    # multiclass training) against the oracle's, bit for bit
    import ctypes as C
    from ferrisboost_b200 import _lib
    lib = _lib.load()
    rng = np.random.default_rng(11)
    for K, weighted in ((2, False), (5, True), (9, True)):
        y = rng.integers(0, K, 20000).astype(np.float32)
        w = rng.uniform(0, 3, 20000).astype(np.float32) if weighted else None
        out = np.zeros(K, np.float32)
        assert lib.fb_class_margins(_lib.ptr(y, C.c_float), _lib.ptr(w, C.c_float), len(y), K,
                                    _lib.ptr(out, C.c_float)) == 0
        assert np.array_equal(out.view(np.uint32), oracle.class_margins(y, K, w).view(np.uint32))
    bad = np.array([0, 1, 2.5], np.float32)
    out = np.zeros(3, np.float32)
    assert lib.fb_class_margins(_lib.ptr(bad, C.c_float), None, 3, 3, _lib.ptr(out, C.c_float)) != 0

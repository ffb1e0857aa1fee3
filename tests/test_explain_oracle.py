"""The oracle's explanation kinds beyond SHAP values (leaf indices, Saabas
contributions, SHAP interaction values) against the reference's own checks
(src/model/explain.rs tests): brute-force Shapley values and interaction
values on small models (2e-5 / 5e-5), interaction rows summing to the SHAP
values (1e-4), symmetric interaction matrices, Saabas rows summing to the
margin, and leaf indices that the model's own traversal lands on; with
categorical splits, per-class groups of a multiclass model, root-only trees
and any thread count."""
import json
import math

import numpy as np
import pytest


def _trees(js):
    out = []
    for t in json.loads(js)["learner"]["gradient_booster"]["model"]["trees"]:
        cats = {n: set(t["categories"][s:s + k])
                for n, s, k in zip(t["categories_nodes"], t["categories_segments"], t["categories_sizes"])}
        out.append(dict(left=t["left_children"], right=t["right_children"], feat=t["split_indices"],
                        cond=np.array(t["split_conditions"], np.float32), dleft=t["default_left"],
                        val=np.array(t["base_weights"], np.float32), hess=np.array(t["sum_hessian"], np.float32),
                        cats=cats))
    return out


def _goes_left(t, i, v):
    """tree.rs:84-96 goes_left: missing follows the default direction; a
    categorical split sends a value in [0, 2^24) right when its code,
    truncated toward zero, is in the split's set, and everything else left
    (categorical.rs:330-345, XGBoost's Decision); a numeric split goes left
    when v < cond."""
    if math.isnan(v):
        return bool(t["dleft"][i])
    if i in t["cats"]:
        return not (0 <= v < 16777216 and int(v) in t["cats"][i])
    return v < t["cond"][i]


def test_categorical_decision_known_answers():
    """categorical.rs:334-352 decision_matches_xgboost, on the rule the
    brute-force explanations use."""
    t = {"cats": {0: {1, 4, 33}}, "dleft": [1], "cond": [0.0]}
    for v in (1.0, 4.0, 33.0, 4.9):
        assert not _goes_left(t, 0, v), v
    for v in (0.0, 2.0, 1000.0, -1.0, -0.5, 16777216.0, math.inf, -math.inf):
        assert _goes_left(t, 0, v), v
    assert _goes_left(t, 0, math.nan)


def _tree_value(t, i, x, known):
    """explain.rs tests tree_value: conditional expectation with the features
    in `known` fixed to x and the others averaged by cover."""
    if t["left"][i] < 0:
        return float(t["val"][i])
    f = t["feat"][i]
    l, r = t["left"][i], t["right"][i]
    if known >> f & 1:
        return _tree_value(t, l if _goes_left(t, i, x[f]) else r, x, known)
    hl, hr = float(t["hess"][l]), float(t["hess"][r])
    return (_tree_value(t, l, x, known) * hl + _tree_value(t, r, x, known) * hr) / (hl + hr)


def _brute(trees, x, m):
    value = {s: sum(_tree_value(t, 0, x, s) for t in trees) for s in range(1 << m)}
    fact = math.factorial
    phi = np.zeros(m)
    inter = np.zeros((m, m))
    for i in range(m):
        for s in range(1 << m):
            if s >> i & 1:
                continue
            size = bin(s).count("1")
            phi[i] += fact(size) * fact(m - size - 1) / fact(m) * (value[s | 1 << i] - value[s])
        for j in range(m):
            if j == i:
                continue
            for s in range(1 << m):
                if s >> i & 1 or s >> j & 1:
                    continue
                size = bin(s).count("1")
                w = fact(size) * fact(m - size - 2) / (2.0 * fact(m - 1))
                inter[i, j] += w * (value[s | 1 << i | 1 << j] - value[s | 1 << i] - value[s | 1 << j] + value[s])
    return phi, inter


def _model(oracle, seed, F=5, depth=4, rounds=6, missing=0.1):
    rng = np.random.default_rng(seed)
    X = rng.standard_normal((3000, F)).astype(np.float32)
    X[rng.random(X.shape) < missing] = np.nan
    z = np.nan_to_num(X[:, 0]) + np.nan_to_num(X[:, 1]) * np.nan_to_num(X[:, 2])
    y = (rng.random(3000) < 1 / (1 + np.exp(-z))).astype(np.float32)
    m = oracle.train(X, y, objective="binary:logistic", max_depth=depth, eta=0.5, max_bin=32, n_rounds=rounds,
                     min_child_weight=0.0)
    return m, X


@pytest.mark.parametrize("seed", [0, 1])
def test_shap_and_interactions_match_brute_force(oracle, seed):
    F = 5
    m, X = _model(oracle, seed, F=F)
    trees = _trees(m.json())
    rows = X[:12]
    shap = m.shap(rows)
    inter = m.interactions(rows)
    for r in range(len(rows)):
        phi, brute = _brute(trees, rows[r], F)
        assert np.max(np.abs(shap[r, :F] - phi)) < 2e-5
        off = ~np.eye(F, dtype=bool)
        assert np.max(np.abs(inter[r, :F, :F][off] - brute[off])) < 5e-5
        assert np.array_equal(inter[r], inter[r].T)
        np.testing.assert_allclose(inter[r].sum(axis=1), shap[r], atol=1e-4)


def test_saabas_rows_sum_to_margin_and_leaves_follow_traversal(oracle):
    m, X = _model(oracle, 3, F=6, depth=5, rounds=8)
    rows = X[:400]
    margin = m.predict_margin(rows)
    approx = m.approx_contribs(rows)
    np.testing.assert_allclose(approx.sum(axis=1), margin, atol=1e-5)
    trees = _trees(m.json())
    leaves = m.pred_leaf(rows)
    assert leaves.shape == (400, len(trees))
    for r in range(0, 400, 37):
        for t, tree in enumerate(trees):
            i = 0
            while tree["left"][i] >= 0:
                i = tree["left"][i] if _goes_left(tree, i, rows[r, tree["feat"][i]]) else tree["right"][i]
            assert leaves[r, t] == i


def _categorical_model(oracle, seed):
    rng = np.random.default_rng(seed)
    n = 3000
    X = rng.standard_normal((n, 4)).astype(np.float32)
    X[:, 1] = rng.integers(0, 12, n)
    X[:, 3] = rng.integers(0, 3, n)
    X[rng.random(X.shape) < 0.05] = np.nan
    z = np.nan_to_num(X[:, 0]) + np.where(np.isin(X[:, 1], [1, 4, 7, 9]), 1.5, -1.0) + 0.5 * np.nan_to_num(X[:, 3])
    y = (rng.random(n) < 1 / (1 + np.exp(-z))).astype(np.float32)
    cat = np.array([0, 1, 0, 1], np.uint8)
    m = oracle.train(X, y, objective="binary:logistic", max_depth=4, eta=0.5, max_bin=32, n_rounds=6,
                     min_child_weight=0.0, categorical=cat, max_cat_to_onehot=4)
    return m, X


def test_categorical_splits_follow_the_set_in_every_explanation(oracle):
    """explain.rs:241-286: partition splits (12 categories) and one-hot
    splits (3) in SHAP, interactions, Saabas values and leaf indices, with
    unseen, negative, fractional and huge codes among the rows."""
    m, X = _categorical_model(oracle, 5)
    trees = _trees(m.json())
    assert any(t["cats"] for t in trees)
    rows = X[:10].copy()
    rows[0, 1], rows[1, 1], rows[2, 1], rows[3, 1] = 40.0, -2.0, 4.5, 3e7
    shap, inter = m.shap(rows), m.interactions(rows)
    for r in range(len(rows)):
        phi, brute = _brute(trees, rows[r], 4)
        assert np.max(np.abs(shap[r, :4] - phi)) < 2e-5, r
        off = ~np.eye(4, dtype=bool)
        assert np.max(np.abs(inter[r, :4, :4][off] - brute[off])) < 5e-5, r
    np.testing.assert_allclose(m.approx_contribs(rows).sum(axis=1), m.predict_margin(rows), atol=1e-5)
    leaves = m.pred_leaf(rows)
    for r in range(len(rows)):
        for t, tree in enumerate(trees):
            i = 0
            while tree["left"][i] >= 0:
                i = tree["left"][i] if _goes_left(tree, i, rows[r, tree["feat"][i]]) else tree["right"][i]
            assert leaves[r, t] == i


def test_worker_count_does_not_change_results(oracle):
    """explain.rs:333-350: every explanation kind is bit-identical for any
    thread count."""
    m, X = _model(oracle, 7)
    rows = X[:300]
    for kind in ("shap", "interactions", "approx_contribs", "pred_leaf", "predict_margin"):
        one = getattr(m, kind)(rows, nthread=1)
        for nt in (2, 5):
            assert np.array_equal(getattr(m, kind)(rows, nthread=nt).view(np.uint32), one.view(np.uint32)), kind


def test_root_only_trees_contribute_to_the_bias(oracle):
    """explain.rs:390-407: trees without a split add their leaf to the bias
    column and nothing to any feature."""
    rng = np.random.default_rng(2)
    X = rng.standard_normal((500, 3)).astype(np.float32)
    y = rng.standard_normal(500).astype(np.float32)
    m = oracle.train(X, y, objective="reg:squarederror", max_depth=0, n_rounds=3, eta=0.5)
    shap = m.shap(X[:20])
    assert np.all(shap[:, :3] == 0.0)
    np.testing.assert_allclose(shap[:, 3], m.predict_margin(X[:20]), atol=1e-6)
    inter = m.interactions(X[:20])
    assert np.all(inter[:, :3, :] == 0.0) and np.all(inter[:, :, :3] == 0.0)


def test_multiclass_groups_match_brute_force(oracle):
    """explain.rs:704-727: class k's explanation uses the trees of class k
    (tree t belongs to class t % K) and the class's own margin."""
    rng = np.random.default_rng(11)
    n, F, K = 2000, 4, 3
    X = rng.standard_normal((n, F)).astype(np.float32)
    y = np.digitize(X[:, 0] + 0.5 * X[:, 1], [-0.5, 0.5]).astype(np.float32)
    m = oracle.train(X, y, objective="multi:softprob", num_class=K, max_depth=3, n_rounds=3, max_bin=32)
    trees = _trees(m.json())
    rows = X[:6]
    shap = m.shap(rows)
    assert shap.shape == (6, K, F + 1)
    margins = m.predict_margin(rows)
    for r in range(len(rows)):
        for k in range(K):
            phi, _ = _brute(trees[k::K], rows[r], F)
            assert np.max(np.abs(shap[r, k, :F] - phi)) < 2e-5, (r, k)
        np.testing.assert_allclose(shap[r].sum(axis=1), margins[r], atol=1e-5)

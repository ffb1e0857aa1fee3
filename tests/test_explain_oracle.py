"""The oracle's explanation kinds beyond SHAP values (leaf indices, Saabas
contributions, SHAP interaction values) against the reference's own checks
(src/model/explain.rs tests): brute-force Shapley values and interaction
values on small models (2e-5 / 5e-5), interaction rows summing to the SHAP
values (1e-4), symmetric interaction matrices, Saabas rows summing to the
margin, and leaf indices that the model's own traversal lands on."""
import json
import math

import numpy as np
import pytest


def _trees(js):
    out = []
    for t in json.loads(js)["learner"]["gradient_booster"]["model"]["trees"]:
        out.append(dict(left=t["left_children"], right=t["right_children"], feat=t["split_indices"],
                        cond=np.array(t["split_conditions"], np.float32), dleft=t["default_left"],
                        val=np.array(t["base_weights"], np.float32), hess=np.array(t["sum_hessian"], np.float32)))
    return out


def _tree_value(t, i, x, known):
    """explain.rs tests tree_value: conditional expectation with the features
    in `known` fixed to x and the others averaged by cover."""
    if t["left"][i] < 0:
        return float(t["val"][i])
    f = t["feat"][i]
    l, r = t["left"][i], t["right"][i]
    if known >> f & 1:
        v = x[f]
        left = bool(t["dleft"][i]) if math.isnan(v) else v < t["cond"][i]
        return _tree_value(t, l if left else r, x, known)
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
                v = rows[r, tree["feat"][i]]
                left = bool(tree["dleft"][i]) if math.isnan(v) else v < tree["cond"][i]
                i = tree["left"][i] if left else tree["right"][i]
            assert leaves[r, t] == i

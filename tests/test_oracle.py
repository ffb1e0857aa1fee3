"""The CPU oracle against the reference's XGBoost 3.4.1 golden margins.

Mirrors tests/bit_exact_vs_xgboost.rs of the reference: every case must match
bit for bit (no tolerance), for every thread count.
"""
import numpy as np
import pytest

from conftest import golden_cases

ALL = golden_cases("index.json") + golden_cases("weighted_index.json") + golden_cases("monotone_index.json")


@pytest.mark.parametrize("case", ALL, ids=[c[0] for c in ALL])
def test_oracle_matches_xgboost_bit_for_bit(oracle, case):
    name, X, y, w, want, params = case
    m = oracle.train(X, y, w, **params)
    got = m.predict_margin(X)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), name


@pytest.mark.parametrize("nthread", [1, 2, 4, 8])
def test_oracle_thread_count_invariant(oracle, nthread):
    # reference tests/bit_exact_vs_xgboost.rs:430-449
    for name, X, y, w, want, params in golden_cases("index.json")[:16]:
        m = oracle.train(X, y, w, nthread=nthread, **params)
        assert np.array_equal(m.predict_margin(X).view(np.uint32), want.view(np.uint32)), (name, nthread)


def test_json_is_deterministic_and_well_formed(oracle):
    import json
    name, X, y, w, want, params = golden_cases("index.json")[2]
    a = oracle.train(X, y, w, **params).json()
    b = oracle.train(X, y, w, nthread=3, **params).json()
    assert a == b
    doc = json.loads(a)
    trees = doc["learner"]["gradient_booster"]["model"]["trees"]
    assert len(trees) == params["num_boost_round"]
    assert doc["learner"]["learner_model_param"]["base_score"] == "0.5"


def test_sketch_low_cardinality_is_exact(oracle):
    # reference src/data/sketch.rs:468-485
    X = np.tile(np.array([1.0, 2.0, 3.0, 5.0], dtype=np.float32), 1000)[:, None]
    cuts, off = oracle.sketch(X, 256)
    assert list(off) == [0, 3]
    assert list(cuts) == [1.5, 2.5, 4.0]


def test_sketch_constant_and_nan(oracle):
    X = np.full((1000, 1), 42.0, dtype=np.float32)
    cuts, off = oracle.sketch(X, 256)
    assert off[-1] == 0
    X = np.arange(100, dtype=np.float32)[:, None]
    X = np.concatenate([X, np.full((100, 1), np.nan, np.float32)])
    cuts, off = oracle.sketch(X, 8)
    assert off[-1] == 7 and np.all(np.diff(cuts) > 0)


def test_shap_rows_sum_to_margin(oracle):
    # reference src/model/explain.rs:1096-1110 (sum-to-margin <= 1e-4 for 10 trees)
    name, X, y, w, want, params = golden_cases("index.json")[2]
    m = oracle.train(X, y, w, **params)
    phi = m.shap(X)
    np.testing.assert_allclose(phi.sum(axis=1), m.predict_margin(X), atol=1e-4)


def test_shap_brute_force_small_tree(oracle):
    # exact Shapley values by subset enumeration (reference src/model/explain.rs:1002-1025, <= 2e-5)
    import itertools
    import math
    rng = np.random.default_rng(3)
    X = rng.integers(0, 4, size=(300, 3)).astype(np.float32)
    y = (X[:, 0] + 0.5 * X[:, 1] * X[:, 2] + rng.normal(0, 0.1, 300)).astype(np.float32)
    m = oracle.train(X, y, objective="reg:squarederror", max_depth=3, num_boost_round=1, base_score=0.0)
    import json
    t = json.loads(m.json())["learner"]["gradient_booster"]["model"]["trees"][0]

    def expect(x, S):
        def rec(i):
            if t["left_children"][i] == -1:
                return t["split_conditions"][i]
            f = t["split_indices"][i]
            l, r = t["left_children"][i], t["right_children"][i]
            if f in S:
                return rec(l) if x[f] < t["split_conditions"][i] else rec(r)
            hl, hr = t["sum_hessian"][l], t["sum_hessian"][r]
            return (hl * rec(l) + hr * rec(r)) / (hl + hr)
        return rec(0)

    for x in X[:20]:
        phi = m.shap(x[None, :])[0]
        F = 3
        for f in range(F):
            others = [g for g in range(F) if g != f]
            v = 0.0
            for k in range(F):
                for S in itertools.combinations(others, k):
                    wgt = math.factorial(k) * math.factorial(F - k - 1) / math.factorial(F)
                    v += wgt * (expect(x, set(S) | {f}) - expect(x, set(S)))
            assert abs(v - phi[f]) <= 2e-5

"""Leaf indices, Saabas contributions and SHAP interaction values on the
device against the CPU oracle (src/model/explain.rs Kind::Leaf,
Contribs { approx: true }, Interactions): leaf indices and Saabas values bit
for bit (the kernels keep the reference's f32 order), interaction values
within the SHAP bar of 1e-5, symmetric, with rows summing to the SHAP
values."""
import numpy as np
import pytest

import ferrisboost_b200 as fb

pytestmark = pytest.mark.gpu


def _data(seed, n, F, missing=0.02):
    rng = np.random.default_rng(seed)
    X = rng.standard_normal((n, F)).astype(np.float32)
    X[rng.random(X.shape) < missing] = np.nan
    z = np.nan_to_num(X[:, 0]) + 0.5 * np.nan_to_num(X[:, 1]) * np.nan_to_num(X[:, 2]) - 0.3 * np.nan_to_num(X[:, 3]) ** 2
    y = (rng.random(n) < 1 / (1 + np.exp(-z))).astype(np.float32)
    return X, y


MODELS = {
    "depth8": (dict(objective="binary:logistic", max_depth=8, eta=0.3, max_bin=256), 20, 28, None),
    "depth6_many_trees": (dict(objective="binary:logistic", max_depth=6, eta=0.1, max_bin=64), 60, 12, None),
    "categorical": (dict(objective="reg:squarederror", max_depth=7, eta=0.3, max_bin=128), 12, 8, [5, 6]),
    "deep_paths": (dict(objective="binary:logistic", max_depth=14, eta=0.3, max_bin=64, min_child_weight=0.0), 4,
                   30, None),
}


def _model(oracle, name):
    p, rounds, F, cat_cols = MODELS[name]
    X, y = _data(sum(map(ord, name)), 20000, F)
    ft = None
    cat = None
    if cat_cols:
        rng = np.random.default_rng(5)
        for c in cat_cols:
            X[:, c] = rng.integers(0, 20, len(X))
        y = (np.nan_to_num(X[:, 0]) + (X[:, cat_cols[0]] % 3) - 0.1 * X[:, cat_cols[1]]).astype(np.float32)
        ft = ["c" if c in cat_cols else "q" for c in range(F)]
        cat = np.array([c in cat_cols for c in range(F)], np.uint8)
    m = fb.train(p, X, label=y, num_boost_round=rounds, feature_types=ft)
    ref = oracle.train(X, y, n_rounds=rounds, **(dict(p, categorical=cat) if cat is not None else p))
    assert m.to_json() == ref.json()
    Xt, _ = _data(77, 600, F, missing=0.05)
    if cat_cols:
        rng = np.random.default_rng(6)
        for c in cat_cols:
            Xt[:, c] = rng.integers(-1, 24, len(Xt))
        Xt[::11, cat_cols[0]] = np.nan
    Xt[::13, 1] = np.inf
    return m, ref, Xt


@pytest.mark.parametrize("name", sorted(MODELS))
def test_leaf_indices_and_saabas_bit_equal(oracle, name):
    m, ref, Xt = _model(oracle, name)
    leaves = m.predict(Xt, pred_leaf=True)
    assert leaves.shape == (len(Xt), m.num_trees)
    assert np.array_equal(leaves, ref.pred_leaf(Xt))
    approx = m.predict(Xt, pred_contribs=True, approx_contribs=True)
    assert np.array_equal(approx.view(np.uint32), ref.approx_contribs(Xt).view(np.uint32))
    np.testing.assert_allclose(approx.sum(axis=1), m.predict(Xt, output_margin=True), atol=1e-4)


@pytest.mark.parametrize("name", sorted(MODELS))
def test_interactions_match_oracle(oracle, name):
    m, ref, Xt = _model(oracle, name)
    Xt = Xt[:200]
    got = m.predict(Xt, pred_interactions=True)
    want = ref.interactions(Xt)
    assert got.shape == want.shape
    assert np.max(np.abs(got - want)) <= 1e-5
    assert np.max(np.abs(got - np.transpose(got, (0, 2, 1)))) <= 1e-6
    np.testing.assert_allclose(got.sum(axis=2), m.predict(Xt, pred_contribs=True), atol=1e-4)


def test_device_explain_entry_point_matches_host():
    import ctypes as C
    import torch
    from ferrisboost_b200 import _lib
    X, y = _data(3, 20000, 10)
    m = fb.train({"objective": "binary:logistic", "max_depth": 6}, X, label=y, num_boost_round=10)
    Xt = X[:500]
    h = m.device_handle(0)
    xd = torch.from_numpy(np.ascontiguousarray(Xt)).cuda()
    s = torch.cuda.current_stream()
    lib = _lib.load()
    for kind, shape, host in ((0, (500, m.num_trees), dict(pred_leaf=True)),
                              (1, (500, 11), dict(pred_contribs=True, approx_contribs=True)),
                              (2, (500, 11, 11), dict(pred_interactions=True))):
        od = torch.empty(shape, dtype=torch.float32, device="cuda")
        assert lib.fbgpu_explain_device(h, kind, xd.data_ptr(), 500, od.data_ptr(), s.cuda_stream) == 0
        torch.cuda.synchronize()
        assert np.array_equal(od.cpu().numpy(), m.predict(Xt, **host))
    bad = np.zeros(1, np.float32)
    assert lib.fbgpu_explain(h, 7, _lib.ptr(np.zeros((1, 10), np.float32), C.c_float), 1,
                             _lib.ptr(bad, C.c_float)) != 0


def test_wide_models_explain_like_the_oracle(oracle):
    # configs[2]-shaped (2000 features, colsample_bytree 0.5): interaction
    # matrices of 2001 x 2001 per row are accumulated in global memory, and
    # Saabas values of rows wider than shared memory in the output rows
    rng = np.random.default_rng(11)
    n, F = 20000, 2000
    X = rng.uniform(-1.0, 1.0, (n, F)).astype(np.float32)
    idx = rng.choice(F, 50, replace=False)
    y = ((X[:, idx] @ rng.standard_normal(50) + rng.normal(0.0, 0.1, n)) > 0).astype(np.float32)
    p = dict(objective="binary:logistic", max_depth=6, eta=0.3, max_bin=64, colsample_bytree=0.5)
    m = fb.train(p, X, label=y, num_boost_round=8)
    ref = oracle.train(X, y, n_rounds=8, **p)
    assert m.to_json() == ref.json()
    Xt = rng.uniform(-1.0, 1.0, (6, F)).astype(np.float32)
    Xt[0, idx[:5]] = np.nan
    got = m.predict(Xt, pred_interactions=True)
    want = ref.interactions(Xt)
    assert got.shape == (6, F + 1, F + 1)
    assert np.max(np.abs(got - want)) <= 1e-5
    np.testing.assert_allclose(got.sum(axis=2), m.predict(Xt, pred_contribs=True), atol=1e-4)
    Xa = rng.uniform(-1.0, 1.0, (300, F)).astype(np.float32)
    approx = m.predict(Xa, pred_contribs=True, approx_contribs=True)
    assert np.array_equal(approx.view(np.uint32), ref.approx_contribs(Xa).view(np.uint32))


def test_interactions_with_wide_category_sets(oracle):
    from test_gpu_wide_categorical import wide_data
    X, y, ft = wide_data(30000, [1200], seed=12)
    p = dict(objective="reg:squarederror", max_depth=5, eta=0.3, max_bin=64)
    m = fb.train(p, X, label=y, num_boost_round=4, feature_types=ft)
    ref = oracle.train(X, y, n_rounds=4, categorical=np.array([t == "c" for t in ft], np.uint8), **p)
    assert m.to_json() == ref.json()
    Xt, _, _ = wide_data(300, [1200], seed=13)
    Xt[:4, -1] = [5000.0, -1.0, 0.5, np.nan]
    got = m.predict(Xt, pred_interactions=True)
    assert np.max(np.abs(got - ref.interactions(Xt))) <= 1e-5
    assert np.max(np.abs(m.predict(Xt, pred_contribs=True) - ref.shap(Xt))) <= 1e-5

"""End-to-end training on the device against the oracle and the reference's
XGBoost 3.4.1 golden margins.  Exact mode must be byte-identical: same JSON
bytes as the oracle, margins bit for bit."""
import json

import numpy as np
import pytest

import ferrisboost_b200 as fb
from conftest import golden_cases

pytestmark = pytest.mark.gpu

GOLDEN = golden_cases("index.json") + golden_cases("weighted_index.json") + golden_cases("monotone_index.json")


def _fb_params(params):
    p = dict(params)
    p.pop("num_boost_round", None)
    return p


@pytest.mark.parametrize("case", GOLDEN, ids=[c[0] for c in GOLDEN])
def test_golden_margins_bit_exact(oracle, case):
    name, X, y, w, want, params = case
    m = fb.train(_fb_params(params), X, label=y, num_boost_round=params["num_boost_round"], weight=w)
    got = m.predict(X, output_margin=True)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), name
    ref = oracle.train(X, y, w, **params)
    assert m.to_json() == ref.json(), name


def _synthetic(n, F, seed, missing=0.0):
    # configs[0] generator shape: N(0,1) features, logistic labels
    rng = np.random.default_rng(seed)
    X = rng.standard_normal((n, F), dtype=np.float32)
    w = rng.standard_normal(F)
    z = X @ w + 0.5 * X[:, 0] * X[:, 1] - 0.3 * X[:, 2] ** 2
    y = (rng.random(n) < 1.0 / (1.0 + np.exp(-z))).astype(np.float32)
    if missing:
        X[rng.random(X.shape) < missing] = np.nan
    return X, y


CONFIGS = [
    dict(objective="binary:logistic", max_depth=6, eta=0.1, max_bin=256),
    dict(objective="reg:squarederror", max_depth=8, eta=0.3, max_bin=256),
    dict(objective="binary:logistic", max_depth=5, eta=0.3, max_bin=64, subsample=0.7, colsample_bytree=0.5,
         seed=3),
    dict(objective="binary:logistic", max_depth=7, eta=0.2, max_bin=1024, max_leaves=40, min_child_weight=5.0,
         gamma=0.2, reg_lambda=2.0),
    dict(objective="reg:squarederror", max_depth=4, eta=0.5, max_bin=255, alpha=0.5, max_delta_step=0.3),
    # scale_pos_weight: positives' gradients weighted, and the default base
    # score one Newton step from margin 0 (objective.rs:403-493)
    dict(objective="binary:logistic", max_depth=6, eta=0.3, max_bin=256, scale_pos_weight=0.3),
    dict(objective="binary:logistic", max_depth=5, eta=0.3, max_bin=128, scale_pos_weight=4.0, subsample=0.8, seed=5),
]


@pytest.mark.parametrize("k", range(len(CONFIGS)))
def test_synthetic_models_byte_identical(oracle, k):
    p = CONFIGS[k]
    X, y = _synthetic(30000, 28, seed=k, missing=0.03 if k % 2 else 0.0)
    if p["objective"] == "reg:squarederror":
        y = (np.nan_to_num(X[:, 0]) * 2 + np.nan_to_num(X[:, 3]) ** 2).astype(np.float32)
    w = np.random.default_rng(k).uniform(0.2, 2.0, len(y)).astype(np.float32) if k in (3, 6) else None
    m = fb.train(p, X, label=y, num_boost_round=12, weight=w)
    ref = oracle.train(X, y, w, n_rounds=12, **p)
    a, b = m.to_json(), ref.json()
    assert a == b
    got = m.predict(X, output_margin=True)
    assert np.array_equal(got.view(np.uint32), ref.predict_margin(X).view(np.uint32))


def test_mixed_bin_counts_byte_identical(oracle):
    # two-byte bins of every histogram tile kind in one block: features up to
    # 440 bins (lane per feature), 441..1024 bins (8 lanes per row, tiles cut
    # at 8 features or 4 record chunks) and beyond max_bin's 1024 when a
    # feature has fewer distinct values than bins; colsample leaves holes
    rng = np.random.default_rng(31)
    n = 30000
    levels = [300, 2000, 700, 50, 1024, 441, 5000, 440, 900, 3000, 600, 128, 1500, 800, 999, 2500, 460]
    X = np.stack([rng.integers(0, k, n).astype(np.float32) / k for k in levels], axis=1)
    X[rng.random(X.shape) < 0.03] = np.nan
    y = (np.nan_to_num(X[:, 1]) + np.nan_to_num(X[:, 4]) ** 2 - np.nan_to_num(X[:, 9]) + rng.normal(0, 0.1, n)).astype(
        np.float32)
    for p in (dict(objective="reg:squarederror", max_depth=7, eta=0.3, max_bin=1024),
              dict(objective="reg:squarederror", max_depth=6, eta=0.3, max_bin=1024, colsample_bytree=0.6, seed=2),
              dict(objective="reg:squarederror", max_depth=6, eta=0.3, max_bin=512)):
        m = fb.train(p, X, label=y, num_boost_round=6)
        assert m.to_json() == oracle.train(X, y, n_rounds=6, **p).json(), p


def test_root_only_and_depth_one(oracle):
    X, y = _synthetic(5000, 5, seed=9)
    for depth in (0, 1):
        p = dict(objective="binary:logistic", max_depth=depth)
        m = fb.train(p, X, label=y, num_boost_round=3)
        assert m.to_json() == oracle.train(X, y, n_rounds=3, **p).json()


def test_categorical_depthwise_byte_identical(oracle):
    rng = np.random.default_rng(4)
    n = 20000
    Xn = rng.standard_normal((n, 6)).astype(np.float32)
    Xn[rng.random(Xn.shape) < 0.05] = np.nan
    Xc = rng.integers(0, 64, (n, 3)).astype(np.float32)
    Xc[:, 2] = rng.integers(0, 3, n)  # few categories: one-hot
    X = np.concatenate([Xn, Xc], axis=1)
    eff = rng.standard_normal(64)
    y = (eff[Xc[:, 0].astype(int)] + np.nan_to_num(Xn[:, 0]) + rng.normal(0, 0.5, n)).astype(np.float32)
    ft = ["q"] * 6 + ["c"] * 3
    cat = np.array([0] * 6 + [1] * 3, np.uint8)
    p = dict(objective="reg:squarederror", max_depth=6, eta=0.3, max_bin=256)
    m = fb.train(p, X, label=y, num_boost_round=8, feature_types=ft)
    ref = oracle.train(X, y, n_rounds=8, categorical=cat, **p)
    assert m.to_json() == ref.json()
    assert np.array_equal(m.predict(X, output_margin=True).view(np.uint32), ref.predict_margin(X).view(np.uint32))


def test_fast_mode_within_tolerance(oracle):
    X, y = _synthetic(40000, 28, seed=21)
    p = dict(objective="binary:logistic", max_depth=6, eta=0.1, max_bin=256)
    fast = fb.train(dict(p, gpu_math="fast"), X, label=y, num_boost_round=20)
    exact = oracle.train(X, y, n_rounds=20, **p)
    a = fast.predict(X, output_margin=True).astype(np.float64)
    b = exact.predict_margin(X).astype(np.float64)

    def logloss(m):
        pr = np.clip(1 / (1 + np.exp(-m)), 1e-15, 1 - 1e-15)
        return -np.mean(y * np.log(pr) + (1 - y) * np.log(1 - pr))

    assert abs(logloss(a) - logloss(b)) < 1e-4
    pa, pb = 1 / (1 + np.exp(-a)), 1 / (1 + np.exp(-b))
    rel = np.abs(pa - pb) / np.abs(pb)
    # north_star: fast-mode predictions within 1e-5 relative of exact mode, every row
    assert rel.max() <= 1e-5, (f"max {rel.max():.3e}, p99 {np.quantile(rel, 0.99):.3e}, "
                               f"median {np.median(rel):.3e}, rows over {np.count_nonzero(rel > 1e-5)}")


def test_predict_and_shap_match_oracle(oracle):
    X, y = _synthetic(20000, 28, seed=5, missing=0.02)
    p = dict(objective="binary:logistic", max_depth=8, eta=0.1, max_bin=256)
    m = fb.train(p, X, label=y, num_boost_round=15)
    ref = oracle.train(X, y, n_rounds=15, **p)
    Xt, _ = _synthetic(3000, 28, seed=77, missing=0.02)
    assert np.array_equal(m.predict(Xt, output_margin=True).view(np.uint32),
                          ref.predict_margin(Xt).view(np.uint32))
    phi = m.predict(Xt, pred_contribs=True)
    want = ref.shap(Xt)
    assert np.max(np.abs(phi - want)) <= 1e-5
    np.testing.assert_allclose(phi.sum(axis=1), ref.predict_margin(Xt), atol=2e-4)


def test_shap_bit_equal_to_oracle(oracle, monkeypatch):
    # the node-by-node kernel keeps the CPU engine's f32 operation order
    X, y = _synthetic(8000, 12, seed=6, missing=0.03)
    p = dict(objective="binary:logistic", max_depth=6, eta=0.3, max_bin=64)
    ref = oracle.train(X, y, n_rounds=8, **p)
    Xt, _ = _synthetic(1000, 12, seed=78, missing=0.03)
    m = fb.train(p, X, label=y, num_boost_round=8)
    monkeypatch.setenv("FBGPU_SHAP", "dfs")
    assert np.array_equal(m.predict(Xt, pred_contribs=True).view(np.uint32), ref.shap(Xt).view(np.uint32))


def test_path_shap_matches_node_kernel_and_oracle(oracle, monkeypatch):
    # the path kernel (default) against the node-by-node kernel on a
    # 200-tree depth-8 model, and against the oracle; rows sum to margins
    X, y = _synthetic(40000, 28, seed=15, missing=0.02)
    p = dict(objective="binary:logistic", max_depth=8, eta=0.1, max_bin=256)
    m = fb.train(p, X, label=y, num_boost_round=200)
    Xt, _ = _synthetic(5000, 28, seed=79, missing=0.02)
    Xt[::37, 3] = np.inf
    Xt[::41, 5] = -np.inf
    phi = m.predict(Xt, pred_contribs=True)
    monkeypatch.setenv("FBGPU_SHAP", "dfs")
    dfs = m.predict(Xt, pred_contribs=True)
    assert np.max(np.abs(phi - dfs)) <= 1e-5
    np.testing.assert_allclose(phi.sum(axis=1), m.predict(Xt, output_margin=True), atol=2e-4)
    ref = oracle.train(X, y, n_rounds=20, **p)
    m20 = fb.train(p, X, label=y, num_boost_round=20)
    monkeypatch.delenv("FBGPU_SHAP")
    assert np.max(np.abs(m20.predict(Xt[:1000], pred_contribs=True) - ref.shap(Xt[:1000]))) <= 1e-5


def test_path_shap_deep_paths_use_the_reference_rule(oracle):
    # depth-14 trees over 40 features: paths with more than 8 features, where
    # the reference's 8-point rule is not exact and the path kernel uses it too
    rng = np.random.default_rng(33)
    X = rng.standard_normal((6000, 40)).astype(np.float32)
    z = X[:, :12].sum(1) + X[:, 12] * X[:, 13]
    y = (rng.random(6000) < 1 / (1 + np.exp(-z))).astype(np.float32)
    p = dict(objective="binary:logistic", max_depth=14, eta=0.3, max_bin=64, min_child_weight=0.0)
    m = fb.train(p, X, label=y, num_boost_round=4)
    ref = oracle.train(X, y, n_rounds=4, **p)
    Xt = rng.standard_normal((800, 40)).astype(np.float32)
    assert np.max(np.abs(m.predict(Xt, pred_contribs=True) - ref.shap(Xt))) <= 1e-5


def test_shap_deep_trees_and_categorical(oracle):
    # depth-14 lossguide trees (deepest DFS stacks) and categorical splits
    rng = np.random.default_rng(12)
    n = 20000
    Xn = rng.standard_normal((n, 5)).astype(np.float32)
    Xc = rng.integers(0, 20, (n, 2)).astype(np.float32)
    X = np.concatenate([Xn, Xc], axis=1)
    y = (Xn[:, 0] + np.sin(3 * Xn[:, 1]) + (Xc[:, 0] % 3) - 0.5 * Xc[:, 1] / 10).astype(np.float32)
    p = dict(objective="reg:squarederror", grow_policy="lossguide", max_depth=14, max_leaves=200, eta=0.3)
    cat = np.array([0] * 5 + [1] * 2, np.uint8)
    m = fb.train(p, X, label=y, num_boost_round=6, feature_types=["q"] * 5 + ["c"] * 2)
    ref = oracle.train(X, y, n_rounds=6, categorical=cat, **p)
    Xt = X[:2000]
    phi = m.predict(Xt, pred_contribs=True)
    assert np.max(np.abs(phi - ref.shap(Xt))) <= 1e-5
    np.testing.assert_allclose(phi.sum(axis=1), ref.predict_margin(Xt), atol=2e-4)
    # unseen, negative, fractional, very large and missing category codes,
    # and missing numeric values (every branch of the category test)
    Xo = X[2000:2600].copy()
    Xo[0::7, 5] = np.nan
    Xo[1::7, 5] = -1.0
    Xo[2::7, 6] = 25.0
    Xo[3::7, 6] = 300.0
    Xo[4::7, 5] = 2.5
    Xo[5::7, 6] = 3.0e7
    Xo[6::7, 0] = np.nan
    assert np.max(np.abs(m.predict(Xo, pred_contribs=True) - ref.shap(Xo))) <= 1e-5


def test_json_is_valid_xgboost_schema():
    X, y = _synthetic(3000, 4, seed=1)
    m = fb.train({"max_depth": 3}, X, label=y, num_boost_round=2)
    doc = json.loads(m.to_json())
    t = doc["learner"]["gradient_booster"]["model"]["trees"][0]
    n = int(t["tree_param"]["num_nodes"])
    assert len(t["left_children"]) == n == len(t["split_conditions"])
    assert doc["learner"]["objective"]["name"] == "binary:logistic"


def test_lossguide_known_answers_on_device(oracle):
    from test_lossguide_oracle import BASE, known_answers

    def train(x, y, **kw):
        p = dict(BASE, **kw)
        rounds = p.pop("n_rounds")
        got = fb.train(p, x, label=y, num_boost_round=rounds).to_json()
        assert got == oracle.train(x, y, **dict(BASE, **kw)).json()
        return got

    known_answers(train)


LOSSGUIDE = [
    # max_leaves cannot bind: the depthwise tree renumbered in pop order
    dict(objective="reg:squarederror", grow_policy="lossguide", max_depth=6, max_leaves=255, eta=0.3, max_bin=256),
    dict(objective="binary:logistic", grow_policy="lossguide", max_depth=5, max_leaves=0, eta=0.3, max_bin=64),
    # binding leaf caps: best-first waves
    dict(objective="binary:logistic", grow_policy="lossguide", max_depth=8, max_leaves=20, eta=0.2, max_bin=128),
    dict(objective="reg:squarederror", grow_policy="lossguide", max_depth=14, max_leaves=63, eta=0.1, max_bin=1024,
         min_child_weight=3.0, subsample=0.8, colsample_bytree=0.6, seed=5),
    dict(objective="reg:squarederror", grow_policy="lossguide", max_depth=10, max_leaves=7, eta=0.5, max_bin=256,
         gamma=0.5, reg_lambda=3.0),
]


@pytest.mark.parametrize("k", range(len(LOSSGUIDE)))
def test_lossguide_models_byte_identical(oracle, k):
    p = LOSSGUIDE[k]
    X, y = _synthetic(30000, 20, seed=40 + k, missing=0.05)
    if p["objective"] == "reg:squarederror":
        y = (np.nan_to_num(X[:, 0]) * 2 + np.nan_to_num(X[:, 3]) ** 2 + np.nan_to_num(X[:, 5])).astype(np.float32)
    m = fb.train(p, X, label=y, num_boost_round=10)
    ref = oracle.train(X, y, n_rounds=10, **p)
    assert m.to_json() == ref.json()
    assert np.array_equal(m.predict(X, output_margin=True).view(np.uint32), ref.predict_margin(X).view(np.uint32))


def test_lossguide_categorical_and_monotone_byte_identical(oracle):
    # configs[3] shape at a small size: numeric features with NaN, 64-code
    # categorical features (partition splits), a leaf cap that binds
    rng = np.random.default_rng(8)
    n = 40000
    Xn = rng.standard_normal((n, 8)).astype(np.float32)
    Xn[rng.random(Xn.shape) < 0.05] = np.nan
    Xc = rng.integers(0, 64, (n, 4)).astype(np.float32)
    X = np.concatenate([Xn, Xc], axis=1)
    eff = rng.standard_normal((4, 64))
    y = (sum(eff[j][Xc[:, j].astype(int)] for j in range(4)) + np.nan_to_num(Xn) @ rng.standard_normal(8)
         + rng.normal(0, 0.5, n)).astype(np.float32)
    ft = ["q"] * 8 + ["c"] * 4
    cat = np.array([0] * 8 + [1] * 4, np.uint8)
    p = dict(objective="reg:squarederror", grow_policy="lossguide", max_depth=12, max_leaves=31, eta=0.05,
             max_bin=1024, monotone_constraints=[1, 0, -1, 0, 0, 0, 0, 0, 0, 0, 0, 0])
    m = fb.train(p, X, label=y, num_boost_round=6, feature_types=ft)
    ref = oracle.train(X, y, n_rounds=6, categorical=cat, **p)
    assert m.to_json() == ref.json()
    assert np.array_equal(m.predict(X, output_margin=True).view(np.uint32), ref.predict_margin(X).view(np.uint32))


def test_lossguide_fast_mode_within_tolerance(oracle):
    X, y = _synthetic(40000, 28, seed=23)
    p = dict(objective="binary:logistic", grow_policy="lossguide", max_depth=10, max_leaves=40, eta=0.1)
    fast = fb.train(dict(p, gpu_math="fast"), X, label=y, num_boost_round=15)
    exact = oracle.train(X, y, n_rounds=15, **p)
    a = fast.predict(X, output_margin=True).astype(np.float64)
    b = exact.predict_margin(X).astype(np.float64)

    def logloss(m):
        pr = np.clip(1 / (1 + np.exp(-m)), 1e-15, 1 - 1e-15)
        return -np.mean(y * np.log(pr) + (1 - y) * np.log(1 - pr))

    assert abs(logloss(a) - logloss(b)) < 1e-4


@pytest.mark.parametrize("case", ["numeric", "categorical"])
def test_partition_leaf_path_byte_identical(oracle, tmp_path, case):
    # the leaf values reach the margins through the partition chunks and the
    # final-level pass (FBGPU_WALK=0) instead of the tree walk: the same
    # models and bit-identical training margins; "numeric" trees take the
    # walk's fast form, "categorical" ones its general form
    import os
    import subprocess
    import sys
    X, y = _synthetic(30000, 12, seed=77, missing=0.03)
    ft = None
    if case == "categorical":
        X[:, 5] = np.random.default_rng(5).integers(0, 20, len(X))
        ft = ["q"] * 12
        ft[5] = "c"
    np.save(tmp_path / "X.npy", X)
    np.save(tmp_path / "y.npy", y)
    p = dict(objective="binary:logistic", max_depth=6, eta=0.3, max_bin=256)
    code = (
        "import sys, numpy as np, ferrisboost_b200 as fb\n"
        f"X = np.load({str(tmp_path / 'X.npy')!r}); y = np.load({str(tmp_path / 'y.npy')!r})\n"
        f"b = fb.Booster({p!r}, fb.Dataset(X, max_bin=256, feature_types={ft!r}), y)\n"
        "b.update(6)\n"
        f"open({str(tmp_path / 'm.json')!r}, 'wb').write(b.model().to_json())\n"
        f"np.save({str(tmp_path / 'margin.npy')!r}, b.margins())\n")
    env = dict(os.environ, FBGPU_WALK="0")
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    subprocess.run([sys.executable, "-c", code], check=True, env=env, cwd=root)
    cat = {} if ft is None else {"categorical": np.array([c == "c" for c in ft], np.uint8)}
    ref = oracle.train(X, y, n_rounds=6, **cat, **p)
    assert (tmp_path / "m.json").read_bytes() == ref.json()
    walked = fb.Booster(p, fb.Dataset(X, max_bin=256, feature_types=ft), y)
    walked.update(6)
    assert walked.model().to_json() == ref.json()
    assert np.array_equal(walked.margins().view(np.uint32), np.load(tmp_path / "margin.npy").view(np.uint32))


def test_non_finite_gradient_stops_the_booster():
    # w * scale_pos_weight overflows to +inf on the positive rows: the
    # gradient bounds are not finite, the round raises (the scales are
    # computed on the device and the error is read back with the tree), and
    # the booster takes no further rounds
    X, y = _synthetic(5000, 6, seed=4)
    w = np.full(len(y), 1e37, np.float32)
    b = fb.Booster(dict(objective="binary:logistic", max_depth=3, scale_pos_weight=100.0, base_score=0.5),
                   fb.Dataset(X, max_bin=64, weight=w), y, w)
    with pytest.raises(Exception, match="non-finite gradient or Hessian"):
        b.update(3)
    with pytest.raises(Exception, match="non-finite|stopped after an error"):
        b.update(1)

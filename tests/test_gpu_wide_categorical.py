"""Categorical features of more than 256 codes on the device (the reference
accepts codes up to 65533, src/data/categorical.rs:19-28, and its GPU path
scans them with tiled scans and a select, backend/cuda/histogram.cu:
3978-4040).  Exact mode must equal the oracle byte for byte: the sorted
partition scans (split.rs:484-617) over a stable weight order of thousands of
codes, their right-going sets, one-hot mode for wide features, scans longer
than one tile (a large max_cat_threshold), histograms wider than shared
memory, and lossguide growth."""
import numpy as np
import pytest

import ferrisboost_b200 as fb

pytestmark = pytest.mark.gpu


def wide_data(n, codes, seed, numeric=3, missing=0.02, objective="reg:squarederror"):
    """Numeric N(0,1) columns plus one categorical column per entry of
    `codes` (uniform codes with some missing); the target sums per-code
    effects (a few large, most small) and a linear term."""
    rng = np.random.default_rng(seed)
    X = np.empty((n, numeric + len(codes)), np.float32)
    X[:, :numeric] = rng.standard_normal((n, numeric), dtype=np.float32)
    z = X[:, 0].astype(np.float64) * 0.5
    for j, c in enumerate(codes):
        col = rng.integers(0, c, n)
        eff = rng.standard_normal(c) * (1.0 + 2.0 * (rng.random(c) < 0.05))
        z += eff[col]
        v = col.astype(np.float32)
        v[rng.random(n) < missing] = np.nan
        X[:, numeric + j] = v
    z += rng.normal(0.0, 0.3, n)
    if objective == "binary:logistic":
        y = (rng.random(n) < 1.0 / (1.0 + np.exp(-z))).astype(np.float32)
    else:
        y = z.astype(np.float32)
    ft = ["q"] * numeric + ["c"] * len(codes)
    return X, y, ft


def _check(oracle, X, y, ft, rounds, **p):
    m = fb.train(p, X, label=y, num_boost_round=rounds, feature_types=ft)
    ref = oracle.train(X, y, n_rounds=rounds, categorical=np.array([t == "c" for t in ft], np.uint8), **p)
    assert m.to_json() == ref.json(), p
    assert np.array_equal(m.predict(X, output_margin=True).view(np.uint32), ref.predict_margin(X).view(np.uint32))
    return m, ref


def test_thousand_and_five_thousand_codes_byte_identical(oracle):
    X, y, ft = wide_data(60000, [1000, 5000], seed=1)
    m, _ = _check(oracle, X, y, ft, 6, objective="reg:squarederror", max_depth=6, eta=0.3, max_bin=256)
    import json
    trees = json.loads(m.to_json())["learner"]["gradient_booster"]["model"]["trees"]
    sizes = [s for t in trees for s in t["categories_sizes"]]
    cats = [c for t in trees for c in t["categories"]]
    assert sizes and max(cats) >= 256, "the wide features take part in the model"


def test_wide_logistic_with_weights_of_both_signs(oracle):
    X, y, ft = wide_data(40000, [700], seed=2, objective="binary:logistic")
    _check(oracle, X, y, ft, 5, objective="binary:logistic", max_depth=5, eta=0.3, max_bin=64)


def test_long_scans_span_several_tiles(oracle):
    # max_cat_threshold 1500: 1499 codes per scan direction, three sorted tiles each
    X, y, ft = wide_data(50000, [3000], seed=3)
    _check(oracle, X, y, ft, 3, objective="reg:squarederror", max_depth=4, eta=0.3, max_bin=64,
           max_cat_threshold=1500)


def test_wide_one_hot_mode(oracle):
    X, y, ft = wide_data(30000, [400], seed=4)
    _check(oracle, X, y, ft, 3, objective="reg:squarederror", max_depth=4, eta=0.3, max_bin=64,
           max_cat_to_onehot=1000)


def test_histograms_wider_than_shared_memory(oracle):
    # 20000 codes: more bins than a shared-memory tile holds, so the histogram
    # adds straight to global memory
    X, y, ft = wide_data(80000, [20000, 300], seed=5, numeric=2)
    _check(oracle, X, y, ft, 3, objective="reg:squarederror", max_depth=5, eta=0.3, max_bin=128)


def test_wide_lossguide_binding_cap(oracle):
    X, y, ft = wide_data(40000, [2000], seed=6)
    _check(oracle, X, y, ft, 3, objective="reg:squarederror", grow_policy="lossguide", max_leaves=12,
           max_depth=8, eta=0.3, max_bin=64)


def test_wide_sets_predict_and_explain(oracle):
    X, y, ft = wide_data(30000, [1500], seed=7)
    m, ref = _check(oracle, X, y, ft, 4, objective="reg:squarederror", max_depth=5, eta=0.3, max_bin=64)
    Xt, _, _ = wide_data(2000, [1500], seed=8)
    Xt[:5, -1] = [70000.0, -3.0, 2.5, np.inf, np.nan]  # unseen, negative, fractional, infinite, missing
    assert np.array_equal(m.predict(Xt, output_margin=True).view(np.uint32), ref.predict_margin(Xt).view(np.uint32))
    assert np.max(np.abs(m.predict(Xt, pred_contribs=True) - ref.shap(Xt))) <= 1e-5


def test_partition_by_a_wide_set():
    from gpu_util import Ctx, random_bins
    rng = np.random.default_rng(9)
    n = 100000
    nbins = [4000, 64]
    bins, widths = random_bins(rng, n, nbins)
    ctx = Ctx(bins, nbins, widths, categorical=[1, 0])
    assert ctx.cat_words() == 125
    rows = np.sort(rng.choice(n, 77777, replace=False)).astype(np.uint32)
    words = np.zeros(125, np.uint32)
    members = rng.choice(4000, 1300, replace=False)
    for c in members:
        words[c // 32] |= np.uint32(1 << (c % 32))
    got, nl = ctx.partition_set(rows, 0, True, words)
    b = bins[0][rows].astype(np.int64)
    missing = b == 65535
    right = np.isin(b, members) & ~missing
    left = ~right  # missing rows go left with missing_left
    assert nl == int(left.sum())
    assert np.array_equal(got, np.concatenate([rows[left], rows[right]]))

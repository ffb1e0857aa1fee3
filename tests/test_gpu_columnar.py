"""Training and prediction from Parquet files and pyarrow tables on the device
(python/ferrisboost/__init__.py:1090 ``train`` with a path or a table;
src/source/parquet_source.rs): the column-major ingest gives the same cuts,
bins and model as the row-major array path, and the model JSON equals the
CPU oracle's on the decoded matrix, with the file's column names as the
feature names."""
import json

import numpy as np
import pyarrow as pa
import pyarrow.parquet as pq
import pytest

import ferrisboost_b200 as fb
from ferrisboost_b200 import columnar

pytestmark = pytest.mark.gpu


def _frame(n, seed):
    rng = np.random.default_rng(seed)
    a = rng.standard_normal(n).astype(np.float32)
    b = rng.standard_normal(n) * 10.0
    c = rng.integers(-50, 50, n).astype(np.int64)
    d = rng.integers(0, 1000, n).astype(np.int32)
    codes = rng.integers(0, 12, n)
    nulls_a = rng.random(n) < 0.05
    nulls_c = rng.random(n) < 0.03
    z = np.where(nulls_a, 0, a) + 0.05 * b - 0.02 * np.where(nulls_c, 0, c) + (codes % 3) - 1
    y = (rng.random(n) < 1 / (1 + np.exp(-z))).astype(np.float32)
    w = rng.uniform(0.5, 2.0, n).astype(np.float32)
    cat = pa.DictionaryArray.from_arrays(pa.array(codes, pa.int32()), pa.array(np.arange(12) * 2, pa.int64()))
    t = pa.table({"a": pa.array(a, mask=nulls_a), "b": pa.array(b), "y": pa.array(y), "c": pa.array(c, mask=nulls_c),
                  "d": pa.array(d), "k": cat, "w": pa.array(w)})
    X = np.stack([np.where(nulls_a, np.nan, a).astype(np.float32), b.astype(np.float32),
                  np.where(nulls_c, np.nan, c.astype(np.float32)).astype(np.float32), d.astype(np.float32),
                  (codes * 2).astype(np.float32)], axis=1)
    return t, X, y, w


def _named(js: bytes, names) -> bytes:
    return js.replace(b'"feature_names":[]', b'"feature_names":' + json.dumps(names, separators=(",", ":")).encode(), 1)


@pytest.mark.parametrize("weighted", [False, True])
def test_parquet_training_matches_array_and_oracle(oracle, tmp_path, weighted):
    t, X, y, w = _frame(40000, 1)
    path = tmp_path / "train.parquet"
    pq.write_table(t, path, row_group_size=7000)
    p = dict(objective="binary:logistic", max_depth=6, eta=0.3, max_bin=128)
    m = fb.train(p, str(path), label="y", weight="w" if weighted else None, num_boost_round=8)
    names = ["a", "b", "c", "d", "k"] + ([] if weighted else ["w"])
    assert m.feature_names == names
    Xa = X if weighted else np.concatenate([X, w[:, None]], axis=1)
    ft = ["q", "q", "q", "q", "c"] + ([] if weighted else ["q"])
    cat = np.array([f == "c" for f in ft], np.uint8)
    ref = oracle.train(Xa, y, w if weighted else None, n_rounds=8, categorical=cat, **p)
    assert m.to_json() == _named(ref.json(), names)
    arr = fb.train(p, Xa, label=y, weight=w if weighted else None, num_boost_round=8, feature_types=ft)
    assert m.to_json() == _named(arr.to_json(), names)
    # prediction binds the file's columns by name (the label column is not read)
    got = m.predict(str(path), output_margin=True)
    assert np.array_equal(got.view(np.uint32), arr.predict(Xa, output_margin=True).view(np.uint32))
    shuffled = t.select(["k", "w", "d", "c", "b", "a"] if not weighted else ["k", "d", "c", "b", "a"])
    got_t = m.predict(shuffled, output_margin=True)
    assert np.array_equal(got_t.view(np.uint32), got.view(np.uint32))


def test_column_major_cuts_and_bins_equal_row_major():
    rng = np.random.default_rng(2)
    X = rng.standard_normal((30000, 9)).astype(np.float32)
    X[rng.random(X.shape) < 0.1] = np.nan
    X[:, 4] = rng.integers(0, 40, len(X))
    ft = ["q"] * 4 + ["c"] + ["q"] * 4
    cols = columnar.Columns(np.ascontiguousarray(X.T), [f"f{i}" for i in range(9)], None, None, None)
    for mb in (16, 256, 1024, 3000):  # 3000: host sketch of the column-major copy
        a = fb.Dataset(X, max_bin=mb, feature_types=ft, device=0)
        b = fb.Dataset(cols, max_bin=mb, feature_types=ft, device=0)
        ca, cb = a.cuts(), b.cuts()
        assert np.array_equal(ca[0], cb[0]) and np.array_equal(ca[1], cb[1])
        for f in range(9):
            assert np.array_equal(a.column(f), b.column(f))


def test_arrow_table_training_and_multi_file(oracle, tmp_path):
    t, X, y, w = _frame(30000, 4)
    feats = t.drop_columns(["y", "w"])
    p = dict(objective="binary:logistic", max_depth=5, eta=0.3, max_bin=64, enable_categorical=True)
    m = fb.train(p, feats, label=y, num_boost_round=6)
    # a table's dictionary column trains on its indices
    Xi = X.copy()
    Xi[:, 4] = Xi[:, 4] / 2
    pr = {k: v for k, v in p.items() if k != "enable_categorical"}
    ref = oracle.train(Xi, y, n_rounds=6, categorical=np.array([0, 0, 0, 0, 1], np.uint8), **pr)
    assert m.to_json() == _named(ref.json(), ["a", "b", "c", "d", "k"])
    # the same rows in three files, as a directory
    d = tmp_path / "parts"
    d.mkdir()
    for i, (lo, hi) in enumerate(((0, 10000), (10000, 25000), (25000, 30000))):
        pq.write_table(t.slice(lo, hi - lo), d / f"p{i}.parquet")
    m2 = fb.train(pr, str(d), label="y", weight="w", num_boost_round=6)
    ref2 = oracle.train(X, y, w, n_rounds=6, categorical=np.array([0, 0, 0, 0, 1], np.uint8), **pr)
    assert m2.to_json() == _named(ref2.json(), ["a", "b", "c", "d", "k"])


def test_csv_training_matches_array(oracle, tmp_path):
    rng = np.random.default_rng(9)
    X = rng.standard_normal((20000, 5)).astype(np.float32)
    X[rng.random(X.shape) < 0.03] = np.nan
    y = (np.nan_to_num(X[:, 0]) - np.nan_to_num(X[:, 3]) > 0).astype(np.float32)
    rows = [",".join("" if np.isnan(v) else repr(float(v)) for v in X[r]) + f",{int(y[r])}" for r in range(len(X))]
    path = tmp_path / "t.csv"
    path.write_text("a,b,c,d,e,y\n" + "\n".join(rows) + "\n")
    p = dict(objective="binary:logistic", max_depth=5, eta=0.3, max_bin=64)
    m = fb.train(p, str(path), label="y", num_boost_round=5)
    ref = oracle.train(X, y, n_rounds=5, **p)
    assert m.to_json() == _named(ref.json(), ["a", "b", "c", "d", "e"])
    hp = tmp_path / "h.csv"
    hp.write_text("\n".join(rows) + "\n")
    mh = fb.train(p, str(hp), label=5, num_boost_round=5, header=False)
    assert mh.to_json() == ref.json() and mh.feature_names is None

"""Columnar ingest on the host: the Parquet decode rules of the reference's
Rust reader (src/source/arrow_source.rs:121-200 visit_column_f32,
src/source/parquet_source.rs:447-500 feature columns and categorical flags)
and the pyarrow-table rules of its Python layer
(python/ferrisboost/__init__.py:798-880 ``_table_matrix``), checked value for
value against an independent numpy statement of each rule."""
import numpy as np
import pyarrow as pa
import pyarrow.parquet as pq
import pytest

from ferrisboost_b200 import columnar


def _table(n=500, seed=0):
    rng = np.random.default_rng(seed)
    f32 = rng.standard_normal(n).astype(np.float32)
    f64 = rng.standard_normal(n) * 1e3 + 1e-7            # needs rounding to f32
    i32 = rng.integers(-2**31, 2**31 - 1, n, dtype=np.int64).astype(np.int32)
    i64 = rng.integers(-2**62, 2**62, n, dtype=np.int64)  # single rounding i64 -> f32
    i64[:4] = [2**53 + 1, -(2**53 + 3), 2**60 + 2**36 + 1, 16777217]
    nulls = rng.random(n) < 0.1
    codes = rng.integers(0, 6, n)
    dict_vals = pa.array([3, 10, 11, 40, 7, 2], pa.int64())
    dcol = pa.DictionaryArray.from_arrays(pa.array(codes, pa.int32(), mask=nulls), dict_vals)
    y = rng.random(n).astype(np.float32)
    w = rng.uniform(0.5, 2, n).astype(np.float32)
    t = pa.table({
        "a32": pa.array(f32, mask=nulls),
        "label": pa.array(y),
        "b64": pa.array(f64),
        "c_i32": pa.array(i32),
        "d_i64": pa.array(i64, mask=nulls),
        "cat": dcol,
        "wt": pa.array(w),
    })
    exp = np.stack([
        np.where(nulls, np.nan, f32).astype(np.float32),
        f64.astype(np.float32),
        i32.astype(np.float32),
        np.where(nulls, np.nan, i64.astype(np.float32)).astype(np.float32),
        np.where(nulls, np.nan, np.array([3, 10, 11, 40, 7, 2], np.float64)[codes]).astype(np.float32),
    ])
    return t, exp, y, w


def test_parquet_decode_rules(tmp_path):
    t, exp, y, w = _table()
    path = tmp_path / "d.parquet"
    pq.write_table(t, path, row_group_size=128)
    c = columnar.read_files([str(path)], "label", "wt")
    assert c.names == ["a32", "b64", "c_i32", "d_i64", "cat"]
    assert c.X.shape == exp.shape and c.X.flags.c_contiguous and c.X.dtype == np.float32
    assert np.array_equal(c.X.view(np.uint32), exp.view(np.uint32))
    assert np.array_equal(c.label, y) and np.array_equal(c.weight, w)
    # dictionary columns are categorical unless feature_types decides
    assert list(c.categorical) == [0, 0, 0, 0, 1]
    c2 = columnar.read_files([str(path)], "label", None, feature_types=["c", "q", "q", "q", "q", "q"])
    assert list(c2.categorical) == [1, 0, 0, 0, 0, 0] and "wt" in c2.names and c2.weight is None
    assert columnar.read_files([str(path)], "label", None, feature_types=["q"] * 6).categorical is None


def test_parquet_single_rounding_of_int64():
    # Rust `i64 as f32` rounds once; a detour through f64 would round twice
    v = np.array([2**53 + 1, 2**60 + 2**36 + 1, -(2**61 + 2**37 + 1)], np.int64)
    out = np.empty(3, np.float32)
    columnar._file_column_f32(pa.chunked_array([pa.array(v)]), "x", float("nan"), out)
    assert np.array_equal(out, v.astype(np.float32))


def test_parquet_missing_sentinel_inf_and_types(tmp_path):
    p = tmp_path / "m.parquet"
    pq.write_table(pa.table({"x": pa.array([1.0, -999.0, 2.0], pa.float64()), "y": pa.array([0.0, 1.0, 0.0])}), p)
    c = columnar.read_files([str(p)], "y", None, missing=-999.0)
    assert np.isnan(c.X[0, 1]) and c.X[0, 0] == 1.0
    bad = tmp_path / "inf.parquet"
    pq.write_table(pa.table({"x": pa.array([1.0, 1e300]), "y": pa.array([0.0, 1.0])}), bad)
    with pytest.raises(ValueError, match="outside the f32 range"):
        columnar.read_files([str(bad)], "y", None)
    inf_label = tmp_path / "infl.parquet"
    pq.write_table(pa.table({"x": pa.array([1.0, 2.0]), "y": pa.array([0.0, np.inf])}), inf_label)
    with pytest.raises(ValueError, match="'y'"):
        columnar.read_files([str(inf_label)], "y", None)
    b = tmp_path / "b.parquet"
    pq.write_table(pa.table({"x": pa.array([True, False]), "y": pa.array([0.0, 1.0])}), b)
    with pytest.raises(ValueError, match="only numeric columns"):
        columnar.read_files([str(b)], "y", None)
    s = tmp_path / "s.parquet"
    pq.write_table(pa.table({"x": pa.array(["a", "b"]).dictionary_encode(), "y": pa.array([0.0, 1.0])}), s)
    with pytest.raises(ValueError, match="category names"):
        columnar.read_files([str(s)], "y", None)
    with pytest.raises(ValueError, match="label column 'nope'"):
        columnar.read_files([str(p)], "nope", None)
    with pytest.raises(ValueError, match="format"):
        columnar.expand_paths([str(tmp_path / "x.txt")])


def test_parquet_prediction_keeps_inf(tmp_path):
    p = tmp_path / "p.parquet"
    pq.write_table(pa.table({"b": pa.array([np.inf, 2.0]), "a": pa.array([1, None], pa.int64())}), p)
    X = columnar.read_file_features([str(p)], ["a", "b"])
    assert X[0, 0] == 1.0 and np.isnan(X[0, 1]) and np.isinf(X[1, 0]) and X[1, 1] == 2.0


def test_several_files_directory_and_glob(tmp_path):
    t, exp, y, w = _table(900, seed=3)
    d = tmp_path / "parts"
    d.mkdir()
    for i, (a, b) in enumerate(((0, 300), (300, 700), (700, 900))):
        part = t.slice(a, b - a)
        if i == 1:  # another column order in one file: bound by name
            part = part.select(["cat", "d_i64", "label", "wt", "c_i32", "b64", "a32"])
        pq.write_table(part, d / f"part-{i}.parquet")
    for spec in ([str(d)], [str(d / "part-*.parquet")], [str(d / f"part-{i}.parquet") for i in range(3)]):
        c = columnar.read_files(spec, "label", "wt")
        assert np.array_equal(c.X.view(np.uint32), exp.view(np.uint32))
        assert np.array_equal(c.label, y)


def test_arrow_table_rules():
    t, exp, y, w = _table(300, seed=5)
    feats = t.drop_columns(["label", "wt"])
    with pytest.raises(ValueError, match="enable_categorical"):
        columnar.read_table(feats)
    c = columnar.read_table(feats, enable_categorical=True)
    assert c.names == ["a32", "b64", "c_i32", "d_i64", "cat"]
    # a table's dictionary column contributes its indices
    idx = np.asarray(feats.column("cat").chunks[0].indices.to_numpy(zero_copy_only=False), np.float64)
    assert np.array_equal(np.isnan(c.X[4]), np.isnan(exp[4]))
    ok = ~np.isnan(exp[4])
    assert np.array_equal(c.X[4][ok], idx[ok].astype(np.float32))
    assert np.array_equal(c.X[:2], exp[:2], equal_nan=True)
    assert list(c.categorical) == [0, 0, 0, 0, 1]
    # scoring: an integer dictionary contributes its values, bound by name
    s = columnar.read_table(feats.select(["cat", "d_i64", "a32", "c_i32", "b64"]), scoring=True,
                            order=["a32", "b64", "c_i32", "d_i64", "cat"])
    assert np.array_equal(s.X[4], exp[4], equal_nan=True)
    with pytest.raises(ValueError, match="bound by name"):
        columnar.read_table(feats, scoring=True, order=["a32", "b64"])
    rb = feats.to_batches()[0]
    assert columnar.arrow_table(rb).num_rows == rb.num_rows
    assert columnar.arrow_table(np.zeros((2, 2))) is None
    assert columnar.path_specs("x.parquet") == ["x.parquet"] and columnar.path_specs(np.zeros(2)) is None


def test_csv_decode_rules(tmp_path):
    # csv_source.rs: Arrow's inference (integers -> Int64, decimals -> Float64)
    # and only an empty field is null; then the Parquet decode rules
    rng = np.random.default_rng(7)
    n = 300
    ints = rng.integers(-2**40, 2**40, n)
    dec = rng.standard_normal(n) * 100
    y = rng.integers(0, 2, n)
    lines = ["a,b,label,c"]
    for i in range(n):
        b = "" if i % 17 == 0 else repr(float(dec[i]))
        c = "NaN" if i % 23 == 0 else "0.1"
        lines.append(f"{ints[i]},{b},{y[i]},{c}")
    path = tmp_path / "d.csv"
    path.write_text("\n".join(lines) + "\n")
    c = columnar.read_files([str(path)], "label", None)
    assert c.names == ["a", "b", "c"]
    assert np.array_equal(c.X[0], ints.astype(np.float32))  # one rounding, int64 -> f32
    want_b = np.where(np.arange(n) % 17 == 0, np.nan, dec).astype(np.float32)
    assert np.array_equal(c.X[1], want_b, equal_nan=True)
    want_c = np.where(np.arange(n) % 23 == 0, np.nan, 0.1).astype(np.float32)
    assert np.array_equal(c.X[2], want_c, equal_nan=True)
    assert np.array_equal(c.label, y.astype(np.float32))
    # headerless: label and weight by column index, no feature names
    hp = tmp_path / "h.csv"
    hp.write_text("\n".join(lines[1:]) + "\n")
    h = columnar.read_files([str(hp)], 2, None, header=False)
    assert h.names == [] and np.array_equal(h.X, c.X, equal_nan=True) and np.array_equal(h.label, c.label)
    with pytest.raises(ValueError, match="column index 9"):
        columnar.read_files([str(hp)], 9, None, header=False)
    bad = tmp_path / "s.csv"
    bad.write_text("a,label\nx,1\ny,0\n")
    with pytest.raises(ValueError, match="only numeric columns"):
        columnar.read_files([str(bad)], "label", None)


def test_csv_columns_bin_like_the_array():
    import ferrisboost_b200 as fb
    import tempfile, os
    rng = np.random.default_rng(8)
    X = rng.standard_normal((2000, 4)).astype(np.float32)
    X[rng.random(X.shape) < 0.05] = np.nan
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "t.csv")
        with open(path, "w") as f:
            f.write("f0,f1,f2,f3,y\n")
            for r in range(len(X)):
                f.write(",".join("" if np.isnan(v) else repr(float(v)) for v in X[r]) + ",0\n")
        c = columnar.read_files([path], "y", None)
    a = fb.Dataset(X, max_bin=64)
    b = fb.Dataset(c, max_bin=64)
    assert all(np.array_equal(u, v) for u, v in zip(a.cuts(), b.cuts()))
    assert all(np.array_equal(a.column(f), b.column(f)) for f in range(4))
    assert b.feature_names == ["f0", "f1", "f2", "f3"]


def test_parquet_decode_property(tmp_path):
    # random numeric columns (every accepted type, nulls, a missing sentinel)
    # decode like an independent numpy statement of the rules
    from hypothesis import given, settings, strategies as st

    types = [pa.float32(), pa.float64(), pa.int32(), pa.int64()]

    @settings(max_examples=25, deadline=None)
    @given(st.integers(1, 200), st.lists(st.integers(0, 3), min_size=1, max_size=5), st.integers(0, 2**31 - 1),
           st.booleans())
    def check(n, kinds, seed, sentinel):
        rng = np.random.default_rng(seed)
        cols, want = {}, []
        miss = -7.0 if sentinel else float("nan")
        for j, k in enumerate(kinds):
            t = types[k]
            nulls = rng.random(n) < 0.2
            if pa.types.is_integer(t):
                lim = 2**31 - 1 if t == pa.int32() else 2**62
                v = rng.integers(-lim, lim, n).astype(np.int64)
                v[rng.random(n) < 0.1] = -7
                cols[f"c{j}"] = pa.array(v.astype(np.int32) if t == pa.int32() else v, t, mask=nulls)
                exp = v.astype(np.float32)
            else:
                v = rng.standard_normal(n) * 1e3
                v[rng.random(n) < 0.1] = -7.0
                cols[f"c{j}"] = pa.array(v.astype(np.float32) if t == pa.float32() else v, t, mask=nulls)
                exp = v.astype(np.float32)
            exp = np.where(nulls, np.nan, exp).astype(np.float32)
            if sentinel:
                exp[exp == np.float32(-7.0)] = np.nan
            want.append(exp)
        cols["y"] = pa.array(np.zeros(n, np.float32))
        path = tmp_path / f"p{seed}.parquet"
        pq.write_table(pa.table(cols), path)
        c = columnar.read_files([str(path)], "y", None, missing=miss)
        assert np.array_equal(c.X, np.stack(want), equal_nan=True)

    check()

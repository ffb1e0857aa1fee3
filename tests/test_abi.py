"""The C-ABI library builds, loads and exports every symbol include/*.h declares
(no device needed); the host-side dataset preparation matches the oracle."""
import ctypes
import pathlib
import re

import numpy as np
import pytest

ROOT = pathlib.Path(__file__).resolve().parents[1]


def declared_functions():
    names = set()
    for h in (ROOT / "include").glob("*.h"):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        for m in re.finditer(r"\b(fbgpu_\w+|fb_\w+)\s*\(", text):
            names.add(m.group(1))
    return sorted(names)


def test_headers_declare_entry_points():
    names = declared_functions()
    assert "fbgpu_build_tree" in names and "fbgpu_histogram" in names and "fb_train" in names
    assert len(names) >= 40


def test_library_exports_every_declared_symbol():
    import ferrisboost_b200
    lib = ferrisboost_b200.lib()
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing
    raw = ctypes.CDLL(str(ROOT / "ferrisboost_b200" / "libfbgpu.so"))
    for n in declared_functions():
        getattr(raw, n)


def test_python_binding_covers_the_headers():
    from ferrisboost_b200 import _lib
    assert set(declared_functions()) == set(_lib.SIGNATURES)


def test_struct_layouts_match_headers():
    from ferrisboost_b200 import _lib
    assert ctypes.sizeof(_lib.FbgpuSplit) == 4 * 6 + 8 * 4 + 32
    assert ctypes.sizeof(_lib.FbgpuConfig) == 48


def test_unknown_and_cpu_parameters_raise():
    import ferrisboost_b200 as fb
    with pytest.raises(ValueError, match="unknown parameter"):
        fb._normalize_params({"max_dept": 3}, 10)
    with pytest.raises(ValueError, match="CUDA devices only"):
        fb._normalize_params({"device": "cpu"}, 10)
    with pytest.raises(ValueError, match="max_depth"):
        fb._normalize_params({"max_depth": 15}, 10)
    p = fb._normalize_params({"learning_rate": 0.1, "reg_lambda": 2.0}, 5)
    assert p["eta"] == 0.1 and p["lambda"] == 2.0
    # objective.rs:144 / :1346 names_round_trip: reg:linear is squared error
    assert fb._normalize_params({"objective": "reg:linear"}, 1)["objective"] == "reg:squarederror"
    with pytest.raises(ValueError, match="not supported"):
        fb._normalize_params({"objective": "rank:bogus"}, 1)


def test_missing_sentinel_rules():
    """src/source/mod.rs:449-475: NaN and finite float32 sentinels are taken
    (f32::MIN too); +-inf, f32::MAX and values that overflow float32 are
    refused, in training parameters and in host data."""
    import ferrisboost_b200 as fb
    assert np.isnan(fb._normalize_params({}, 1)["missing"])
    for ok in (-999.0, 0.0, float(np.finfo(np.float32).min)):
        assert fb._normalize_params({"missing": ok}, 1)["missing"] == np.float32(ok)
    for bad in (float("inf"), float("-inf"), float(np.finfo(np.float32).max), 1e39, -1e39):
        with pytest.raises(ValueError, match="missing"):
            fb._normalize_params({"missing": bad}, 1)
        with pytest.raises(ValueError, match="missing"):
            fb._as_matrix(np.zeros((2, 2)), bad)
    got = fb._as_matrix(np.array([[1.0, -999.0], [np.nan, 2.0]]), -999.0)
    assert np.isnan(got[0, 1]) and np.isnan(got[1, 0]) and got[0, 0] == 1.0 and got[1, 1] == 2.0


@pytest.mark.parametrize("max_bin", [16, 255, 256, 1024])
def test_dataset_cuts_and_bins_match_oracle(oracle, max_bin):
    import ferrisboost_b200 as fb
    rng = np.random.default_rng(max_bin)
    X = rng.standard_normal((20000, 6)).astype(np.float32)
    X[rng.random(X.shape) < 0.05] = np.nan
    X[:, 3] = np.round(X[:, 3] * 2)  # low cardinality
    w = rng.uniform(0.5, 2.0, 20000).astype(np.float32)
    for weight in (None, w):
        ds = fb.Dataset(X, max_bin=max_bin, weight=weight)
        cuts, off = ds.cuts()
        rc, ro = oracle.sketch(X, max_bin, w=weight)
        assert np.array_equal(off, ro)
        assert np.array_equal(cuts.view(np.uint32), rc.view(np.uint32))
        bins = oracle.quantize(X, rc, ro)
        for f in range(X.shape[1]):
            assert np.array_equal(ds.column(f), bins[f]), f


def test_dataset_categorical_codes_match_oracle(oracle):
    import ferrisboost_b200 as fb
    rng = np.random.default_rng(7)
    X = np.concatenate([rng.standard_normal((5000, 2)), rng.integers(0, 64, (5000, 2))], axis=1).astype(np.float32)
    X[rng.random(X.shape) < 0.03] = np.nan
    cat = np.array([0, 0, 1, 1], np.uint8)
    ds = fb.Dataset(X, max_bin=256, feature_types=["q", "q", "c", "c"])
    cuts, off = ds.cuts()
    rc, ro = oracle.sketch(X, 256, categorical=cat)
    assert np.array_equal(off, ro) and np.array_equal(cuts, rc)
    bins = oracle.quantize(X, rc, ro, categorical=cat)
    for f in range(4):
        assert np.array_equal(ds.column(f), bins[f])


def test_invalid_category_is_rejected():
    import ferrisboost_b200 as fb
    X = np.array([[0.0], [1.5]], dtype=np.float32)
    with pytest.raises(ValueError, match="invalid category"):
        fb.Dataset(X, feature_types=["c"])


def test_host_expf_table_is_verified_on_this_host():
    import ctypes as C
    from ferrisboost_b200 import _lib
    why = C.c_char_p()
    assert _lib.load().fbgpu_exact_exp_available(C.byref(why)) == 1, why.value


@pytest.mark.parametrize("form", [
    (1, -1, 0, 0), [1, -1, 0, 0], "(1,-1,0,0)", "(1, -1, 0, 0)", np.array([1, -1, 0, 0]), (1, -1), (5, -2, 0, 0),
])
def test_monotone_forms_are_equivalent(form):
    """python/tests/test_monotone.py:61-72: tuple, list, string, numpy,
    shorter than the feature count (zeros after), sign only (5 == 1)."""
    import ferrisboost_b200 as fb
    mc = fb._normalize_params({"monotone_constraints": form}, 1)["monotone_constraints"]
    assert fb._positional_monotone(mc, None, 4).tolist() == [1, -1, 0, 0]


@pytest.mark.parametrize("bad,match", [
    ((1, 0, 0, 0, 1), "only 4 features"), ((1.5, 0), "integer"), ((True, 0), "integer"),
    ("1,0,-1", "string must look like"), ("(1,x)", "non-integer"), (3.0, "tuple"),
])
def test_invalid_monotone_constraints_are_rejected(bad, match):
    """python/tests/test_monotone.py:86-99."""
    import ferrisboost_b200 as fb
    with pytest.raises(ValueError, match=match):
        mc = fb._normalize_params({"monotone_constraints": bad}, 1)["monotone_constraints"]
        fb._positional_monotone(mc, None, 4)


def test_named_monotone_constraints():
    """python/ferrisboost/__init__.py:422-426, 1344-1350: by column name when
    the data has names; unknown names and nameless data are refused; all
    zeros and empty mean no constraint."""
    import ferrisboost_b200 as fb
    mc = fb._normalize_params({"monotone_constraints": {"b": -1, "d": 3}}, 1)["monotone_constraints"]
    assert fb._positional_monotone(mc, ["a", "b", "c", "d"], 4).tolist() == [0, -1, 0, 1]
    with pytest.raises(ValueError, match="column names"):
        fb._positional_monotone(mc, None, 4)
    with pytest.raises(ValueError, match="not feature columns"):
        fb._positional_monotone({"z": 1}, ["a", "b"], 2)
    with pytest.raises(ValueError, match="keys must be column name strings"):
        fb._normalize_params({"monotone_constraints": {0: 1}}, 1)
    for zeros in [(0, 0, 0, 0), (0,), "(0,0)", []]:
        mc = fb._normalize_params({"monotone_constraints": zeros}, 1)["monotone_constraints"]
        assert not fb._positional_monotone(mc, None, 4).any()


@pytest.mark.parametrize("bad", [{"alpha": -1.0}, {"max_delta_step": -0.1}, {"scale_pos_weight": -2.0},
                                 {"alpha": float("inf")}, {"max_delta_step": float("nan")}])
def test_invalid_regularization_values_are_rejected(bad):
    """python/tests/test_regularization.py:118-124."""
    import ferrisboost_b200 as fb
    with pytest.raises(ValueError, match=next(iter(bad))):
        fb._normalize_params(bad, 1)
    # reg_alpha is alpha; neutral values equal the defaults (test_regularization.py:64-78)
    assert fb._normalize_params({"reg_alpha": 2.0}, 1)["alpha"] == 2.0
    d = fb._normalize_params({}, 1)
    n = fb._normalize_params({"alpha": 0.0, "max_delta_step": 0.0, "scale_pos_weight": 1.0}, 1)
    assert all(d[k] == n[k] for k in ("alpha", "max_delta_step", "scale_pos_weight"))

"""Device dataset preparation against the CPU oracle, bit for bit: the
weighted quantile sketch run on the device (src/data/sketch.rs restated) must
give the same cuts, and device binning the same bins, as the oracle's
sequential sketch and quantize_dense (src/source/dense.rs:99-308)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _cases():
    """(name, X, max_bin, categorical flags) covering the sketch's branches."""
    rng = np.random.default_rng(3)
    out = []
    # many chunks and levels: limit = max_bin x 16 values per chunk
    X = rng.standard_normal((200_000, 3)).astype(np.float32)
    out.append(("normal_mb256", X, 256, None))
    out.append(("normal_mb255_nonpow2_limit", X, 255, None))
    out.append(("normal_mb16_deep_tree", X[:100_000], 16, None))   # 391 chunks, 9 levels
    out.append(("normal_mb2", X[:30_000], 2, None))                # limit 32: 938 chunks
    out.append(("normal_mb1024", X[:150_000], 1024, None))         # limit 16384
    # exact multiples of the chunk size and one past them
    for n in (4096, 4097, 8192, 3 * 4096, 3 * 4096 + 1, 1):
        out.append((f"n{n}", rng.standard_normal((n, 2)).astype(np.float32), 256, None))
    # NaNs, all-NaN and constant columns, extreme magnitudes, heavy ties
    X = rng.standard_normal((60_000, 7)).astype(np.float32)
    X[rng.random(60_000) < 0.3, 0] = np.nan
    X[:, 1] = np.nan
    X[:, 2] = 1.5
    X[:, 3] = np.round(X[:, 3] * 4) / 4                             # low cardinality: midpoints
    X[rng.random(60_000) < 0.5, 4] = 0.0                            # half the values tie
    X[::97, 5] = 1e30                                               # extreme finite magnitudes
    X[::89, 5] = -1e30
    X[:, 6] = np.where(X[:, 6] > 0, -0.0, X[:, 6])                  # one signed zero, many times
    out.append(("edges", X, 64, None))
    out.append(("edges_mb256", X, 256, None))
    # categorical codes next to numeric features, u8 and u16 blocks
    Xc = np.concatenate([rng.standard_normal((40_000, 2)), rng.integers(0, 64, (40_000, 2)),
                         rng.integers(0, 300, (40_000, 1))], axis=1).astype(np.float32)
    Xc[rng.random(Xc.shape) < 0.03] = np.nan
    out.append(("categorical", Xc, 256, np.array([0, 0, 1, 1, 1], np.uint8)))
    # configs[3]-like widths: 1024-bin numerics (u16) beside 64-code categoricals (u8)
    Xm = np.concatenate([rng.standard_normal((50_000, 3)), rng.integers(0, 64, (50_000, 2))], axis=1)
    Xm = Xm.astype(np.float32)
    Xm[:, :3][rng.random((50_000, 3)) < 0.05] = np.nan
    out.append(("mixed_mb1024", Xm, 1024, np.array([0, 0, 0, 1, 1], np.uint8)))
    # many features (several column blocks of 64 u16 / 128 u8 features)
    out.append(("wide", rng.uniform(-1, 1, (3000, 150)).astype(np.float32), 256, None))
    out.append(("wide_u8", rng.uniform(-1, 1, (3000, 150)).astype(np.float32), 64, None))
    return out


CASES = _cases()


@pytest.mark.parametrize("name,X,max_bin,cat", CASES, ids=[c[0] for c in CASES])
def test_device_cuts_and_bins_match_oracle(oracle, name, X, max_bin, cat):
    import ferrisboost_b200 as fb
    ft = None if cat is None else ["c" if c else "q" for c in cat]
    ds = fb.Dataset(X, max_bin=max_bin, feature_types=ft, device=0)
    cuts, off = ds.cuts()
    rc, ro = oracle.sketch(X, max_bin, categorical=cat)
    assert np.array_equal(off, ro)
    assert np.array_equal(cuts.view(np.uint32), rc.view(np.uint32))
    bins = oracle.quantize(X, rc, ro, categorical=cat)
    for f in range(X.shape[1]):
        assert np.array_equal(ds.column(f), bins[f]), f


def test_device_binning_with_given_cuts(oracle):
    import ferrisboost_b200 as fb
    rng = np.random.default_rng(5)
    X = rng.standard_normal((30_000, 5)).astype(np.float32)
    X[rng.random(X.shape) < 0.02] = np.nan
    cuts, off = oracle.sketch(X[:10_000], 128)
    ds = fb.Dataset(X, max_bin=128, cuts=(cuts, off), device=0)
    got_c, got_o = ds.cuts()
    assert np.array_equal(got_o, off) and np.array_equal(got_c, cuts)
    bins = oracle.quantize(X, cuts, off)
    for f in range(5):
        assert np.array_equal(ds.column(f), bins[f])


def test_device_sketch_features_matches_host():
    from ferrisboost_b200 import distributed as fbd
    rng = np.random.default_rng(9)
    X = rng.standard_normal((50_000, 6)).astype(np.float32)
    X[rng.random(X.shape) < 0.1] = np.nan
    feats = [4, 1, 5]
    host = fbd.sketch_features(X, feats, 256)
    dev = fbd.sketch_features(X, feats, 256, device=0)
    for a, b in zip(host, dev):
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


def test_device_dataset_rejects_reserved_and_invalid_values():
    import ferrisboost_b200 as fb
    X = np.zeros((100, 2), np.float32)
    X[7, 1] = np.finfo(np.float32).max
    with pytest.raises(ValueError, match="f32::MAX"):
        fb.Dataset(X, device=0)
    for v in (np.inf, -np.inf):  # python/mod.rs:4063-4073 reject_inf
        Xi = np.zeros((100, 2), np.float32)
        Xi[9, 0] = v
        with pytest.raises(ValueError, match="inf"):
            fb.Dataset(Xi, device=0)
    Xc = np.array([[0.0], [1.5]], dtype=np.float32)
    with pytest.raises(ValueError, match="invalid category"):
        fb.Dataset(Xc, feature_types=["c"], device=0)


def test_device_dataset_trains_the_host_dataset_model():
    import ferrisboost_b200 as fb
    rng = np.random.default_rng(21)
    X = rng.standard_normal((50_000, 8)).astype(np.float32)
    X[rng.random(X.shape) < 0.02] = np.nan
    y = (X[:, 0] + 0.5 * np.nan_to_num(X[:, 1]) > 0).astype(np.float32)
    p = {"objective": "binary:logistic", "max_depth": 6, "max_bin": 256, "eta": 0.3}
    models = []
    for dev in (None, 0):
        b = fb.Booster(p, fb.Dataset(X, max_bin=256, device=dev), y)
        b.update(5)
        models.append(b.model().to_json())
    assert models[0] == models[1]


def test_full_size_device_cuts_match_host():
    """configs[1]-shaped column at 2M rows (489 chunks, 9 merge levels): the
    device cuts equal the host engine's bit for bit."""
    import ferrisboost_b200 as fb
    rng = np.random.default_rng(0)
    X = rng.standard_normal((2_000_000, 2), dtype=np.float32)
    a = fb.Dataset(X, max_bin=256).cuts()
    b = fb.Dataset(X, max_bin=256, device=0).cuts()
    assert np.array_equal(a[1], b[1]) and np.array_equal(a[0].view(np.uint32), b[0].view(np.uint32))

"""Model.load_model (the reference's XGBoost-JSON loading, src/model/tree.rs:
760-960): a model written by the CPU oracle loads into the engine and is
written back byte for byte (objectives, base scores, class margins, feature
types, categorical splits, feature names), so the loaded trees are the
written ones; malformed models are rejected.  CPU only: loading and writing
run on the host."""
import json

import numpy as np
import pytest

import ferrisboost_b200 as fb


def _data(seed, n=3000, F=6):
    rng = np.random.default_rng(seed)
    X = rng.standard_normal((n, F)).astype(np.float32)
    X[rng.random(X.shape) < 0.05] = np.nan
    y = (np.nan_to_num(X[:, 0]) + 0.5 * np.nan_to_num(X[:, 1]) > 0).astype(np.float32)
    return X, y


@pytest.mark.parametrize("kind", ["logistic", "sqerr_categorical", "multiclass", "softmax_base_score"])
def test_oracle_model_round_trips(oracle, kind):
    X, y = _data(3)
    kw = dict(n_rounds=4, max_depth=4, max_bin=32)
    if kind == "logistic":
        ref = oracle.train(X, y, objective="binary:logistic", **kw)
    elif kind == "sqerr_categorical":
        X[:, 2] = np.random.default_rng(1).integers(0, 20, len(X))
        y = (X[:, 2] % 3 + np.nan_to_num(X[:, 0])).astype(np.float32)
        ref = oracle.train(X, y, objective="reg:squarederror", categorical=np.array([0, 0, 1, 0, 0, 0], np.uint8),
                           max_cat_to_onehot=1, **kw)
        trees = json.loads(ref.json())["learner"]["gradient_booster"]["model"]["trees"]
        assert any(1 in t["split_type"] for t in trees)  # categorical splits take part
    elif kind == "multiclass":
        yk = np.digitize(np.nan_to_num(X[:, 0]), [-0.5, 0.5]).astype(np.float32)
        ref = oracle.train(X, yk, objective="multi:softprob", num_class=3, **kw)
    else:
        yk = np.digitize(np.nan_to_num(X[:, 1]), [0.0]).astype(np.float32)
        ref = oracle.train(X, yk, objective="multi:softmax", num_class=2, base_score=0.3, **kw)
    js = ref.json()
    m = fb.Model.load_model(js)
    assert m.to_json() == js
    assert m.num_trees == ref.num_trees
    assert m.num_outputs == ref.num_outputs


def test_feature_names_and_file_round_trip(oracle, tmp_path):
    X, y = _data(4)
    ref = oracle.train(X, y, objective="binary:logistic", n_rounds=3, max_depth=3)
    names = [f"col_{i}" for i in range(X.shape[1])]
    doc = json.loads(ref.json())
    doc["learner"]["feature_names"] = names
    js = json.dumps(doc, separators=(",", ":")).encode()
    path = tmp_path / "m.json"
    path.write_bytes(js)
    m = fb.Model.load_model(str(path))
    assert m.feature_names == names
    out = tmp_path / "again.json"
    m.save_model(out)
    assert json.loads(out.read_bytes()) == doc
    assert out.read_bytes() == ref.json().replace(b'"feature_names":[]', b'"feature_names":' + json.dumps(
        names, separators=(",", ":")).encode(), 1)


def test_malformed_models_are_rejected(oracle):
    X, y = _data(5)
    doc = json.loads(oracle.train(X, y, objective="binary:logistic", n_rounds=2, max_depth=3).json())
    bad = json.loads(json.dumps(doc))
    bad["learner"]["objective"]["name"] = "rank:ndcg"
    with pytest.raises(ValueError, match="not supported"):
        fb.Model.load_model(json.dumps(bad).encode())
    bad = json.loads(json.dumps(doc))
    bad["learner"]["gradient_booster"]["model"]["trees"][0]["left_children"][0] = 999
    with pytest.raises(ValueError, match="outside the tree"):
        fb.Model.load_model(json.dumps(bad).encode())
    bad = json.loads(json.dumps(doc))
    bad["learner"]["gradient_booster"]["model"]["trees"][1]["split_indices"][0] = 77
    with pytest.raises(ValueError, match="feature 77"):
        fb.Model.load_model(json.dumps(bad).encode())


@pytest.mark.gpu
def test_loaded_models_predict_like_the_oracle(oracle):
    X, y = _data(6, n=5000)
    ref = oracle.train(X, y, objective="binary:logistic", n_rounds=5, max_depth=5)
    m = fb.Model.load_model(ref.json())
    got = m.predict(X, output_margin=True)
    assert np.array_equal(got.view(np.uint32), ref.predict_margin(X).view(np.uint32))
    yk = np.digitize(np.nan_to_num(X[:, 0]), [-0.5, 0.5]).astype(np.float32)
    refk = oracle.train(X, yk, objective="multi:softprob", num_class=3, n_rounds=3, max_depth=4)
    mk = fb.Model.load_model(refk.json())
    assert np.array_equal(mk.predict(X, output_margin=True), refk.predict_margin(X))

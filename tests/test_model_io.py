"""Model.load_model (the reference's XGBoost-JSON loading, src/model/tree.rs:
760-960): a model written by the CPU oracle loads into the engine and is
written back byte for byte (objectives, base scores, class margins, feature
types, categorical splits, feature names), so the loaded trees are the
written ones; an XGBoost-written dump loads; what the reference's loader
rejects is rejected (src/model/tree.rs:765-1447 and its tests :287-629).
Loading and writing run on the host; one test predicts on the device.""" 
import json
import re

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
    # the oracle's own loader (used to explain device-trained models on the
    # CPU) reads the document back to the same trees
    back = oracle.load_json(js)
    assert back.json() == js
    assert np.array_equal(back.predict_margin(X).view(np.uint32), ref.predict_margin(X).view(np.uint32))
    assert np.array_equal(back.shap(X[:200]).view(np.uint32), ref.shap(X[:200]).view(np.uint32))


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
    with pytest.raises(ValueError, match="invalid child indices"):
        fb.Model.load_model(json.dumps(bad).encode())
    bad = json.loads(json.dumps(doc))
    bad["learner"]["gradient_booster"]["model"]["trees"][1]["split_indices"][0] = 77
    with pytest.raises(ValueError, match="feature 77"):
        fb.Model.load_model(json.dumps(bad).encode())


def _xgb_dump() -> dict:
    """A small model laid out the way XGBoost itself writes one (tree.rs:
    480-546 test fixture): every parameter a string, floats in scientific
    notation, fields this engine does not use (version 2.0.3, attributes,
    base_weights, id, boost_from_average).  One split on feature 1 at 2.5,
    missing left; leaves -0.3 and 0.15; base score 0.5 (margin 0)."""
    tree = {
        "base_weights": [0.0, -1.0, 0.5], "categories": [], "categories_nodes": [], "categories_segments": [],
        "categories_sizes": [], "default_left": [1, 0, 0], "id": 0, "left_children": [1, -1, -1],
        "loss_changes": [12.5, 0.0, 0.0], "parents": [2147483647, 0, 0], "right_children": [2, -1, -1],
        "split_conditions": [2.5, -0.3, 0.15], "split_indices": [1, 0, 0], "split_type": [0, 0, 0],
        "sum_hessian": [8.0, 5.0, 3.0],
        "tree_param": {"num_deleted": "0", "num_feature": "3", "num_nodes": "3", "size_leaf_vector": "1"},
    }
    return {
        "version": [2, 0, 3],
        "learner": {
            "attributes": {"best_iteration": "3"}, "feature_names": [], "feature_types": [],
            "gradient_booster": {"model": {"gbtree_model_param": {"num_parallel_tree": "1", "num_trees": "1"},
                                           "iteration_indptr": [0, 1], "tree_info": [0], "trees": [tree]},
                                 "name": "gbtree"},
            "learner_model_param": {"base_score": "5E-1", "boost_from_average": "1", "num_class": "0",
                                    "num_feature": "3", "num_target": "1"},
            "objective": {"name": "binary:logistic", "reg_loss_param": {"scale_pos_weight": "1"}},
        },
    }


def _xgb_text(doc: dict) -> bytes:
    """XGBoost's float text: 5E-1, 2.5E0, -3E-1 (the loader must read it)."""
    def sci(v):
        if v == 0:
            return "0E0"
        m, e = f"{v:.8E}".split("E")
        return f"{m.rstrip('0').rstrip('.')}E{int(e)}"

    def mark(o):
        if isinstance(o, float):
            return "@@" + sci(o) + "@@"
        if isinstance(o, dict):
            return {k: mark(v) for k, v in o.items()}
        if isinstance(o, list):
            return [mark(v) for v in o]
        return o
    return re.sub(r'"@@([^@]*)@@"', r"\1", json.dumps(mark(doc))).encode()


def test_reads_an_xgboost_written_dump():
    """tree.rs:520-546 reads_a_real_looking_xgboost_dump."""
    js = _xgb_text(_xgb_dump())
    assert b"2.5E0" in js and b"-3E-1" in js and b"1.5E-1" in js
    m = fb.Model.load_model(js)
    assert m.num_trees == 1 and m.num_outputs == 1
    t = m.tree(0)
    assert not t["is_leaf"][0] and t["feat"][0] == 1 and t["cond"][0] == np.float32(2.5)
    assert t["default_left"][0] == 1 and t["hess"][0] == 8.0 and t["gain"][0] == 12.5
    assert t["is_leaf"][1] and t["leaf"][1] == np.float32(-0.3) and t["leaf"][2] == np.float32(0.15)
    assert json.loads(m.to_json())["learner"]["learner_model_param"]["base_score"] == "0.5"
    # the written model reads back to the same bytes
    again = fb.Model.load_model(m.to_json())
    assert again.to_json() == m.to_json()


def _edit(doc, path, value):
    d = json.loads(json.dumps(doc))
    node = d
    for k in path[:-1]:
        node = node[k]
    node[path[-1]] = value
    return json.dumps(d).encode()


_TREE = ("learner", "gradient_booster", "model", "trees", 0)


@pytest.mark.parametrize("path,value,what", [
    (("learner", "learner_model_param", "num_class"), "3", "num_class"),
    (("learner", "objective", "name"), "survival:bogus", "not supported"),
    (("learner", "gradient_booster", "model", "gbtree_model_param", "num_parallel_tree"), "4", "num_parallel_tree"),
    (_TREE + ("split_type",), [1, 0, 0], "no category segment"),
    (_TREE + ("left_children",), [0, -1, -1], "root"),
    (_TREE + ("right_children",), [-1, -1, -1], "only one child"),
    (_TREE + ("split_indices",), [3, 0, 0], "feature 3"),
    (("learner", "learner_model_param", "num_target"), "2", "num_target"),
    (("learner", "gradient_booster", "model", "tree_info"), [1], "tree_info"),
    (_TREE + ("tree_param", "size_leaf_vector"), "2", "size_leaf_vector"),
    (("learner", "gradient_booster", "name"), "gblinear", "gbtree"),
    (_TREE + ("split_type",), [2, 0, 0], "split_type"),
    (_TREE + ("default_left",), [1, 0], "default_left length"),
    (("learner", "learner_model_param", "base_score"), "[0.1, 0.2]", "multi-target"),
])
def test_rejects_what_it_cannot_represent(path, value, what):
    """tree.rs:548-617 rejects_what_it_cannot_represent and
    multi_output_models_are_rejected: each edit of a loadable dump is refused
    with a message that names the problem."""
    with pytest.raises(ValueError, match=what):
        fb.Model.load_model(_edit(_xgb_dump(), path, value))


def test_tree_shape_is_checked():
    """tree.rs:1375-1447: a node with two parents, a cycle below the root, an
    unreachable node."""
    def tree(left, right):
        d = _xgb_dump()
        t = d["learner"]["gradient_booster"]["model"]["trees"][0]
        n = len(left)
        t.update(left_children=left, right_children=right, split_indices=[0] * n, default_left=[0] * n,
                 split_conditions=[0.0] * n, split_type=[0] * n, loss_changes=[0.0] * n, sum_hessian=[1.0] * n)
        return json.dumps(d).encode()
    with pytest.raises(ValueError, match="invalid child indices"):
        fb.Model.load_model(tree([1, 3, -1, -1], [2, 3, -1, -1]))
    with pytest.raises(ValueError, match="node 3 has more than one parent"):
        fb.Model.load_model(tree([1, 3, 3, -1, -1], [2, 4, 4, -1, -1]))
    with pytest.raises(ValueError, match="node 1 has more than one parent"):  # 1 -> 3 -> 1
        fb.Model.load_model(tree([1, 3, -1, 1, -1], [2, 4, -1, 2, -1]))
    with pytest.raises(ValueError, match="node 3 is unreachable"):
        fb.Model.load_model(tree([1, -1, -1, -1], [2, -1, -1, -1]))
    with pytest.raises(ValueError, match="node 3 is unreachable"):  # 3 -> 4 -> 3, apart from the root
        fb.Model.load_model(tree([1, -1, -1, 4, 3, -1, -1], [2, -1, -1, 5, 6, -1, -1]))
    with pytest.raises(ValueError, match="root"):  # 0 -> 1 -> 0
        fb.Model.load_model(tree([1, 0, -1, -1], [2, 3, -1, -1]))
    fb.Model.load_model(tree([2, -1, 3, -1, -1], [1, -1, 4, -1, -1]))  # children before parent ids is a tree


def test_old_dumps_and_base_score_spellings():
    """tree.rs:610-629: size_leaf_vector "0" and no num_target load; base_score
    as "5E-1", "[5E-1]" or " [ -1.5 ] "; an empty or non-numeric one is refused;
    a multiclass model with one stored base score uses it for every class."""
    d = _xgb_dump()
    d["learner"]["gradient_booster"]["model"]["trees"][0]["tree_param"]["size_leaf_vector"] = "0"
    del d["learner"]["learner_model_param"]["num_target"]
    fb.Model.load_model(json.dumps(d).encode())
    for raw, want in (("5E-1", "0.5"), ("[5E-1]", "0.5"), (" [ 0.25 ] ", "0.25")):
        m = fb.Model.load_model(_edit(_xgb_dump(), ("learner", "learner_model_param", "base_score"), raw))
        assert json.loads(m.to_json())["learner"]["learner_model_param"]["base_score"] == want
    sq = json.loads(_edit(_xgb_dump(), ("learner", "objective", "name"), "reg:squarederror"))
    m = fb.Model.load_model(_edit(sq, ("learner", "learner_model_param", "base_score"), " [ -1.5 ] "))
    assert json.loads(m.to_json())["learner"]["learner_model_param"]["base_score"] == "-1.5"
    for raw in ("[]", "abc"):
        with pytest.raises(ValueError, match="base_score"):
            fb.Model.load_model(_edit(_xgb_dump(), ("learner", "learner_model_param", "base_score"), raw))
    mc = _xgb_dump()
    lrn = mc["learner"]
    lrn["objective"] = {"name": "multi:softprob", "softmax_multiclass_param": {"num_class": "2"}}
    lrn["learner_model_param"].update(num_class="2", base_score="2.5E-1")
    t0 = lrn["gradient_booster"]["model"]["trees"][0]
    lrn["gradient_booster"]["model"].update(trees=[t0, dict(t0, id=1)], tree_info=[0, 1])
    m = fb.Model.load_model(json.dumps(mc).encode())
    assert m.num_outputs == 2
    assert json.loads(m.to_json())["learner"]["learner_model_param"]["base_score"] == "[0.25,0.25]"


def test_scale_pos_weight_text():
    """tree.rs:300-330 scale_pos_weight_is_saved_and_loaded: written as the
    shortest decimal (3 -> "3", 0.3 -> "0.3", 2.5 -> "2.5") and read back."""
    for spw, text in ((3.0, "3"), (0.3, "0.3"), (2.5, "2.5")):
        js = _edit(_xgb_dump(), ("learner", "objective", "reg_loss_param", "scale_pos_weight"), text)
        m = fb.Model.load_model(js)
        out = json.loads(m.to_json())
        assert out["learner"]["objective"]["reg_loss_param"]["scale_pos_weight"] == text
        assert fb.Model.load_model(m.to_json()).to_json() == m.to_json()
    d = _xgb_dump()
    del d["learner"]["objective"]["reg_loss_param"]
    m = fb.Model.load_model(json.dumps(d).encode())
    assert json.loads(m.to_json())["learner"]["objective"]["reg_loss_param"]["scale_pos_weight"] == "1"


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
    # tree.rs:538-545: the XGBoost-written dump predicts by strict less-than,
    # missing values following the default direction
    xm = fb.Model.load_model(_xgb_text(_xgb_dump()))
    rows = np.array([[0.0, 2.0, 0.0], [0.0, np.nan, 0.0], [0.0, 9.0, 0.0], [0.0, 2.5, 0.0]], np.float32)
    got = xm.predict(rows, output_margin=True)
    assert np.array_equal(got, np.array([-0.3, -0.3, 0.15, 0.15], np.float32))


@pytest.mark.parametrize("objective", ["binary:logistic", "reg:squarederror"])
def test_transform_inverts_base_margin(objective):
    """objective.rs:1348-1358 transform_inverts_base_margin: the engine's
    base margin (logit for logistic, identity for squared error) maps back to
    base_score within 1e-6."""
    for bs in (0.1, 0.5, 0.9):
        d = _xgb_dump()
        d["learner"]["objective"]["name"] = objective
        d["learner"]["learner_model_param"]["base_score"] = repr(bs)
        m = fb.Model.load_model(json.dumps(d).encode())
        margin = fb.lib().fb_model_base_margin(m._h)
        back = 1.0 / (1.0 + np.exp(-np.float64(margin))) if objective == "binary:logistic" else margin
        assert abs(back - bs) < 1e-6, (objective, bs, back)

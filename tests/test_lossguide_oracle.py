"""Lossguide (best-first) growth of the oracle against the reference's own
known-answer tests (tests/lossguide.rs:52-150, python/tests/test_lossguide.py):
one feature 0..7, max_bin 16, eta 0.3, lambda 0, min_child_weight 0,
base_score 0, squared error, one round.  These pin the pop order (highest
gain first, lower node id on ties, candidates of different depths compared)
and the leaf cap."""
import json

import numpy as np
import pytest

BASE = dict(objective="reg:squarederror", max_bin=16, eta=0.3, reg_lambda=0.0, min_child_weight=0.0,
            base_score=0.0, grow_policy="lossguide", n_rounds=1, nthread=1)


def _tree(model_json):
    return json.loads(model_json)["learner"]["gradient_booster"]["model"]["trees"][0]


def _fit(train, labels, max_depth=8, max_leaves=0):
    y = np.asarray(labels, dtype=np.float32)
    x = np.arange(y.size, dtype=np.float32).reshape(-1, 1)
    return _tree(train(x, y, max_depth=max_depth, max_leaves=max_leaves))


def _leaves(t):
    return sum(c == -1 for c in t["left_children"])


def known_answers(train):
    """The reference's assertions; `train(x, y, **params)` returns model JSON."""
    t = _fit(train, [0, 0, 1, 1, 10, 10, 14, 20], max_leaves=3)  # highest gain under the cap
    assert _leaves(t) == 3 and t["left_children"][0] != -1
    assert t["left_children"][1] == -1 and t["left_children"][2] != -1
    t = _fit(train, [0, 0, 1, 1, 3, 3, 4, 4], max_leaves=3)  # equal gains: lower node id
    assert _leaves(t) == 3 and t["left_children"][1] != -1 and t["left_children"][2] == -1
    for depth, cap in ((0, 0), (8, 1)):  # root-only trees
        t = _fit(train, [0, 0, 1, 1, 3, 3, 4, 4], max_depth=depth, max_leaves=cap)
        assert len(t["left_children"]) == 1
    ys = [float((v // 4) ** 2) for v in range(32)]  # max_leaves = 0 is unlimited
    assert _leaves(_fit(train, ys, max_leaves=0)) > 3
    assert _leaves(_fit(train, ys, max_leaves=3)) == 3
    t = _fit(train, [0, 0, 1, 1, 10, 10, 14, 20], max_leaves=4)  # candidates at different depths
    assert _leaves(t) == 4 and t["left_children"][1] == -1 and t["left_children"][3] != -1


def test_oracle_lossguide_known_answers(oracle):
    known_answers(lambda x, y, **kw: oracle.train(x, y, **dict(BASE, **kw)).json())

"""The reference's depthwise leaf-cap tests (tests/max_leaves.rs:74-206) on
the CPU oracle: under ``max_leaves`` a depthwise tree expands nodes in node
order while the cap allows, 0 and a cap that cannot bind give the same bytes,
the depth limit and a root-only depth take precedence, every round keeps the
cap, and a branch that ends early still counts toward the cap.  The device
grows the same trees byte for byte (the GPU training tests with max_leaves)."""
import json

import numpy as np

SEPARABLE = np.array([0.0, 0.0, 1.0, 1.0, 3.0, 3.0, 4.0, 4.0], np.float32)
LABELS = np.array([0.0, 0.0, 1.0, 1.0, 3.0, 3.0, 4.0, 4.0], np.float32)


def _fit(oracle, values, labels, max_leaves, max_depth, n_rounds=1, reg_lambda=1.0):
    """max_leaves.rs:16-51: one feature, squared error, base_score 1.5, eta
    0.3, min_child_weight 0."""
    X = np.asarray(values, np.float32)[:, None]
    return oracle.train(X, np.asarray(labels, np.float32), objective="reg:squarederror", n_rounds=n_rounds,
                        max_depth=max_depth, max_leaves=max_leaves, max_bin=16, eta=0.3, reg_lambda=reg_lambda,
                        min_child_weight=0.0, base_score=1.5, nthread=1)


def _trees(ref):
    return json.loads(ref.json())["learner"]["gradient_booster"]["model"]["trees"]


def _is_leaf(t, i):
    return t["left_children"][i] == -1


def _leaves(t):
    return sum(c == -1 for c in t["left_children"])


def test_leaf_caps_select_depthwise_in_node_order(oracle):
    one = _trees(_fit(oracle, SEPARABLE, LABELS, 1, 6))[0]
    assert _leaves(one) == 1 and _is_leaf(one, 0)
    two = _trees(_fit(oracle, SEPARABLE, LABELS, 2, 6))[0]
    assert _leaves(two) == 2 and not _is_leaf(two, 0) and _is_leaf(two, 1) and _is_leaf(two, 2)
    # both depth-one nodes can split; room for one more leaf goes to the left node
    three = _trees(_fit(oracle, SEPARABLE, LABELS, 3, 6))[0]
    assert _leaves(three) == 3 and not _is_leaf(three, 0) and not _is_leaf(three, 1) and _is_leaf(three, 2)


def test_zero_and_nonbinding_leaf_limits_match_bit_for_bit(oracle):
    unlimited = _fit(oracle, SEPARABLE, LABELS, 0, 6, n_rounds=3)
    nonbinding = _fit(oracle, SEPARABLE, LABELS, 64, 6, n_rounds=3)
    assert unlimited.json() == nonbinding.json()
    X = SEPARABLE[:, None]
    assert np.array_equal(unlimited.predict_margin(X).view(np.uint32), nonbinding.predict_margin(X).view(np.uint32))


def test_depth_limit_and_root_only_depth_take_precedence(oracle):
    d1 = _trees(_fit(oracle, SEPARABLE, LABELS, 3, 1))[0]
    assert _leaves(d1) == 2 and _is_leaf(d1, 1) and _is_leaf(d1, 2)
    root = _trees(_fit(oracle, SEPARABLE, LABELS, 8, 0))[0]
    assert len(root["left_children"]) == 1 and _leaves(root) == 1


def test_every_round_respects_the_cap(oracle):
    ref = _fit(oracle, SEPARABLE, LABELS, 3, 6, n_rounds=4)
    trees = _trees(ref)
    assert len(trees) == 4 and all(_leaves(t) <= 3 for t in trees)


def test_an_early_terminal_branch_still_counts_toward_the_cap(oracle):
    """lambda 0, base margin 1.5: the root isolates the four zeros (gain
    231.125), the right child splits [10, 10] from [11, 12] (gain 2.25) and
    [11, 12] could split again (gain 0.5); the left branch is terminal."""
    values = np.arange(8, dtype=np.float32)
    labels = np.array([0, 0, 0, 0, 10, 10, 11, 12], np.float32)
    t = _trees(_fit(oracle, values, labels, 3, 8, reg_lambda=0.0))[0]
    assert _leaves(t) <= 3
    assert _is_leaf(t, 1) and not _is_leaf(t, 2)
    assert abs(t["loss_changes"][0] - 231.125) < 1e-3 and abs(t["loss_changes"][2] - 2.25) < 1e-4

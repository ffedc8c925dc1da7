"""The oracle's host-driven grower (the reference's fallback driver,
src/tree.cpp:291-349, 1031-1120): a queue of evaluated leaves, popped in
depth-wise batches of at most 256 leaves or one leaf at a time by largest
gain. Checked on the CPU against the level-synchronous grower the GPU path
is pinned to: identical trees where both apply, the same splits in another
numbering for loss-guided trees, and the leaf and depth limits."""
import numpy as np
import pytest

import checkers as C

BASE = dict(eta=0.3, reg_lambda=1.0, reg_alpha=0.0, min_child_weight=1.0, max_delta_step=0.0,
            min_split_loss=0.0)


def _inputs(seed, rows=3000, cols=6, max_bin=32, nan=0.1):
    o = C.oracle()
    rng = np.random.default_rng(seed)
    X = rng.normal(size=(rows, cols)).astype(np.float32)
    X[rng.random(X.shape) < nan] = np.nan
    cuts, counts, minima = o.sketch_cuts(X, max_bin)
    bins = o.quantize(X, cuts, counts)
    y = np.nan_to_num(X[:, 0]) * 2 - np.nan_to_num(X[:, 2]) + np.sin(np.nan_to_num(X[:, 1]) * 3)
    pairs = np.stack([(0.5 - y + 0.3 * rng.normal(size=rows)), np.ones(rows)], 1).astype(np.float32)[:, None, :]
    scale = o.gradient_scales(pairs)[0]
    q = o.quantize_gradients(pairs, scale[None])[:, 0, :]
    return o, bins, q, scale, cuts, counts, minima


def _canonical(nodes, i=0):
    n = nodes[i]
    if n["left"] < 0:
        return ("leaf", float(n["leaf"]), float(n["cover"]))
    return (int(n["feature"]), float(n["threshold"]), int(n["default_left"]), float(n["gain"]),
            float(n["cover"]), _canonical(nodes, n["left"]), _canonical(nodes, n["right"]))


def _depths(nodes):
    depth = np.zeros(len(nodes), int)
    for i, n in enumerate(nodes):
        if n["left"] >= 0:
            depth[n["left"]] = depth[n["right"]] = depth[i] + 1
    return depth


@pytest.mark.parametrize("seed,max_depth", [(1, 1), (2, 4), (3, 6), (4, 8)])
def test_depthwise_queue_equals_level_synchronous_growth(seed, max_depth):
    o, bins, q, scale, cuts, counts, minima = _inputs(seed)
    params = dict(BASE, max_depth=max_depth)
    want_nodes, want_leaf = o.grow_tree(bins, q, scale, cuts, counts, minima, params)
    got_nodes, got_leaf = C.grow_tree_queue(bins, q, scale, cuts, counts, minima, params)
    assert got_nodes.tobytes() == want_nodes.tobytes()
    assert got_leaf.tobytes() == want_leaf.tobytes()


def test_deep_depthwise_tree_beyond_ten_levels():
    o, bins, q, scale, cuts, counts, minima = _inputs(5, rows=1500, cols=4, max_bin=64, nan=0.0)
    params = dict(BASE, max_depth=14, min_child_weight=0.0)
    want_nodes, want_leaf = o.grow_tree(bins, q, scale, cuts, counts, minima, params)
    # No level of this tree has more than 256 expanding nodes, so the 256-leaf
    # batches of the queue reproduce the level-synchronous tree exactly.
    d = _depths(want_nodes)
    assert max(np.sum((d == k) & (want_nodes["left"] >= 0)) for k in range(15)) <= 256
    assert d.max() > 10
    got_nodes, got_leaf = C.grow_tree_queue(bins, q, scale, cuts, counts, minima, params)
    assert got_nodes.tobytes() == want_nodes.tobytes()
    assert got_leaf.tobytes() == want_leaf.tobytes()


@pytest.mark.parametrize("max_depth", [3, 6, 0])
def test_lossguide_without_limits_finds_the_same_splits(max_depth):
    o, bins, q, scale, cuts, counts, minima = _inputs(7, rows=2000)
    params = dict(BASE, max_depth=max_depth or 20)
    want_nodes, want_leaf = o.grow_tree(bins, q, scale, cuts, counts, minima, params)
    if not max_depth:
        assert _depths(want_nodes).max() < 20  # the depth limit never bound
    got_nodes, got_leaf = C.grow_tree_queue(bins, q, scale, cuts, counts, minima, dict(params, max_depth=max_depth),
                                            lossguide=True)
    # Another node numbering, the same tree.
    assert _canonical(got_nodes) == _canonical(want_nodes)
    assert got_leaf.tobytes() == want_leaf.tobytes()


@pytest.mark.parametrize("lossguide", [False, True])
def test_max_leaves_caps_the_tree(lossguide):
    o, bins, q, scale, cuts, counts, minima = _inputs(9)
    for max_leaves in (2, 5, 17, 64):
        nodes, _ = C.grow_tree_queue(bins, q, scale, cuts, counts, minima, dict(BASE, max_depth=0 if lossguide else 8),
                                     lossguide=lossguide, max_leaves=max_leaves)
        leaves = int(np.sum(nodes["left"] < 0))
        assert leaves <= max_leaves and len(nodes) == 2 * leaves - 1
    if lossguide:
        # One leaf at a time, largest gain first: the splits taken under a
        # budget are a prefix of those taken with a larger one.
        small, _ = C.grow_tree_queue(bins, q, scale, cuts, counts, minima, dict(BASE, max_depth=0),
                                     lossguide=True, max_leaves=6)
        large, _ = C.grow_tree_queue(bins, q, scale, cuts, counts, minima, dict(BASE, max_depth=0),
                                     lossguide=True, max_leaves=20)
        split = small["left"] >= 0
        assert np.array_equal(small["feature"][split], large["feature"][: len(small)][split])
        assert np.array_equal(small["gain"][split], large["gain"][: len(small)][split])


def test_whole_run_training_with_the_host_driven_grower():
    rng = np.random.default_rng(11)
    X = rng.normal(size=(2500, 5)).astype(np.float32)
    X[rng.random(X.shape) < 0.05] = np.nan
    y = (np.nan_to_num(X[:, 0]) + np.nan_to_num(X[:, 1]) ** 2 > 0.5).astype(np.float32)
    base = {"objective": "binary:logistic", "max_depth": 5, "max_bin": 64}
    depthwise, m_d, _ = C.oracle_train(X, y, base, 4)
    lossguide, m_l, _ = C.oracle_train(X, y, dict(base, grow_policy="lossguide"), 4)
    # Without a leaf budget the loss-guided trees are the depth-wise trees
    # numbered in another order, so the margins agree bit for bit.
    assert [_canonical(t) for t in lossguide] == [_canonical(t) for t in depthwise]
    assert m_l.tobytes() == m_d.tobytes()
    capped, _, _ = C.oracle_train(X, y, dict(base, grow_policy="lossguide", max_depth=0, max_leaves=7), 4)
    assert all(np.sum(t["left"] < 0) <= 7 for t in capped)
    deep, _, _ = C.oracle_train(X, y, dict(base, max_depth=12, min_child_weight=0.0), 2)
    assert max(_depths(t).max() for t in deep) > 10

"""Built histograms, word for word.

The product's exact int64 (g, h) sums of one tree level (the smaller child of
every node pair, or the root) are compared with the oracle's `orc_histogram`
over the same rows: the reference's histogram semantics
(kernels/boost.metal:700-733, kernels/histogram_missing.metal.h:13-60; the
smaller-child choice of kernels/boost.metal:661-698). A bin that no split
ever lands on is checked too, which tree and margin comparisons cannot do.

The c4-width case has BASELINE's c4 row format: 128 features, 256 bins plus a
missing bin (uint16 codes), 5 % NaN, binary:logistic, and enough rows (2^22)
that every gradient fits the staged two-limb accumulation. Its values are the
integers 0..255, whose cuts are the integer grid for any row count (the
sketch keeps every distinct value when there are at most max_bin of them), so
the oracle's bins are the values themselves; a 100k-row sample pins that
against the oracle's own sketch and binning.
"""
import json

import numpy as np
import pytest

import checkers as C
import product as P

pytestmark = pytest.mark.gpu

MISSING = 0xFFFFFFFF


def _int_grid(rows, cols, nan, seed):
    rng = np.random.default_rng(seed)
    codes = rng.integers(0, 256, size=(rows, cols), dtype=np.uint8)
    X = codes.astype(np.float32)
    bins = codes.astype(np.uint32)
    step = 1 << 19
    for i in range(0, rows, step):
        m = rng.random((min(step, rows - i), cols), dtype=np.float32) < nan
        X[i:i + step][m] = np.nan
        bins[i:i + step][m] = MISSING
    return X, bins


def _tree_arrays(bst):
    t = json.loads(bst.save_raw("json"))["learner"]["gradient_booster"]["model"]["trees"][0]
    return (np.array(t["left_children"], np.int64), np.array(t["right_children"], np.int64),
            np.array(t["split_indices"], np.int64),
            np.array(t["split_conditions"], np.float64).astype(np.float32),
            np.array(t["default_left"], np.int64).astype(bool))


def _node_of_rows(X, tree, depth):
    """Node id each row occupies after `depth` levels (x < threshold goes
    left, NaN by the default direction)."""
    left, right, feat, cond, dleft = tree
    node = np.zeros(X.shape[0], np.int64)
    idx = np.arange(X.shape[0])
    for _ in range(depth):
        internal = left[node] >= 0
        x = X[idx, np.where(internal, feat[node], 0)]
        go_left = np.where(np.isnan(x), dleft[node], x < cond[node])
        node = np.where(internal, np.where(go_left, left[node], right[node]), node)
    return node


def _oracle_q(objective, y, weights, groups=1):
    base = C.oracle_base_margin(objective, y, weights, groups)
    margins = np.repeat(base[None, :], len(y), axis=0)
    pairs = C.oracle_gradients(objective, margins, y, weights)
    o = C.oracle()
    scales = o.gradient_scales(pairs)
    return o.quantize_gradients(pairs, scales)[:, 0, :]


def _check_level(xgb, dtrain, params, X, bins, q, stride, depth):
    bst = xgb.Booster(params, [dtrain])
    P.capture_level_histograms(bst, depth)
    bst.update(dtrain, 0)
    meta, hist, node_ids = P.level_histograms(bst)
    assert meta["depth"] == depth and meta["bins1"] == stride + 1
    assert (meta["f_lo"], meta["f_hi"]) == (0, X.shape[1])
    assert meta["pairs"] == len(node_ids) >= 1
    tree = _tree_arrays(bst)
    node = _node_of_rows(X, tree, depth)
    counts = np.bincount(node, minlength=len(tree[0]))
    parent = {int(c): p for p, (l, r) in enumerate(zip(tree[0], tree[1])) if l >= 0 for c in (l, r)}
    for p, nid in enumerate(node_ids):
        nid = int(nid)
        if depth:
            # The smaller child of the pair is built; a tie builds the left one.
            pl = int(tree[0][parent[nid]])
            sib = pl + 1 if nid == pl else pl
            assert counts[nid] < counts[sib] or (counts[nid] == counts[sib] and nid == pl), (p, nid)
        rows = np.flatnonzero(node == nid).astype(np.uint32)
        want = C.oracle_histogram(bins, q, rows, stride)
        np.testing.assert_array_equal(hist[p], want, err_msg="depth %d pair %d node %d" % (depth, p, nid))
    return meta


def test_c4_width_histogram_words_match_oracle():
    import xgboost as xgb
    rows, cols = 1 << 22, 128
    X, bins = _int_grid(rows, cols, 0.05, seed=41)
    # The oracle's own sketch and binning of a sample: the integer grid.
    o = C.oracle()
    cuts, counts, minima = o.sketch_cuts(X[:100_000], 256)
    assert (counts == 256).all()
    np.testing.assert_array_equal(o.quantize(X[:100_000], cuts, counts), bins[:100_000])
    rng = np.random.default_rng(42)
    y = (rng.random(rows) < 0.4).astype(np.float32)
    q = _oracle_q("binary:logistic", y, None)
    # Every |q| fits 42 bits: the staged two-limb kernel builds these levels.
    assert int(np.abs(q).max()).bit_length() <= 42
    dtrain = xgb.DMatrix(X, label=y)
    params = {"objective": "binary:logistic", "max_depth": 10, "eta": 0.1, "max_bin": 256,
              "tree_method": "hist", "device": "cuda"}
    for depth in (0, 1, 4, 9):
        _check_level(xgb, dtrain, params, X, bins, q, 256, depth)


@pytest.mark.parametrize("case", ["unit_hessian_13_features", "weighted_u8_40_features",
                                  "weighted_u8_40_features_unstaged", "three_limb_small",
                                  "three_limb_small_unstaged"])
def test_level_histogram_words_match_oracle(case):
    """The weighted uint8 and three_limb_small cases have values wider than
    42 bits, which the staged three-limb kernel builds; their `_unstaged`
    forms (cuda_hist_staged3=0) build the same levels with the unstaged
    three-limb kernel."""
    import xgboost as xgb
    unstaged = case.endswith("_unstaged")
    case = case.replace("_unstaged", "")
    rng = np.random.default_rng({"unit_hessian_13_features": 1, "weighted_u8_40_features": 2,
                                 "three_limb_small": 3}[case])
    if case == "unit_hessian_13_features":
        rows, cols, nan, objective, weighted, depths, max_bin = 60_000, 13, 0.1, "reg:squarederror", False, \
            range(0, 7), 256
    elif case == "weighted_u8_40_features":
        rows, cols, nan, objective, weighted, depths, max_bin = 300_000, 40, 0.0, "reg:squarederror", True, \
            (0, 2, 7), 64
    else:
        rows, cols, nan, objective, weighted, depths, max_bin = 3_000, 33, 0.2, "binary:logistic", False, \
            range(0, 6), 32
    X = rng.normal(size=(rows, cols)).astype(np.float32)
    X[rng.random(X.shape) < nan] = np.nan
    w = rng.uniform(0.2, 3.0, rows).astype(np.float32) if weighted else None
    if objective == "binary:logistic":
        y = (rng.random(rows) < 0.3).astype(np.float32)
    else:
        y = (np.nan_to_num(X) @ rng.normal(size=cols)).astype(np.float32)
    o = C.oracle()
    cuts, counts, minima = o.sketch_cuts(X, max_bin, w)
    bins = o.quantize(X, cuts, counts)
    q = _oracle_q(objective, y, w)
    dtrain = xgb.DMatrix(X, label=y, weight=w)
    params = {"objective": objective, "max_depth": 8, "eta": 0.3, "max_bin": max_bin,
              "tree_method": "hist", "device": "cuda"}
    if objective != "reg:squarederror" or weighted:
        assert int(np.abs(q).max()).bit_length() > 42  # three-limb values
    if unstaged:
        params["cuda_hist_staged3"] = 0
    for depth in depths:
        _check_level(xgb, dtrain, params, X, bins, q, cuts.shape[1], depth)

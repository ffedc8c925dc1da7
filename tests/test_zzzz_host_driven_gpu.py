"""Host-driven trees on the GPU (csrc/grower.cpp + csrc/queue.cu: the
reference's fallback driver, src/tree.cpp:291-349, 1031-1120) against the
oracle's host-driven grower, bit for bit: loss-guided trees, leaf budgets,
depths beyond ten levels and levels wider than one 256-leaf batch, with every
node of every tree and the training margins compared."""
import numpy as np
import pytest

import checkers as C
import product as P
from test_gpu_parity import assert_same_trees, bits

pytestmark = pytest.mark.gpu


def _run(X, y, params, rounds, weights=None):
    full = C.train_params(params)
    trees_o, margins_o, _ = C.oracle_train(X, y, full, rounds, weights=weights)
    prod = {k: v for k, v in full.items() if k != "num_class" or full["objective"].startswith("multi")}
    trees_p, margins_p = P.train(X, y, prod, rounds, weights=weights)
    assert_same_trees(trees_p, trees_o)
    np.testing.assert_array_equal(bits(margins_p), bits(margins_o))
    return trees_p


def _data(rows, cols, nan, seed):
    rng = np.random.default_rng(seed)
    X = rng.normal(size=(rows, cols)).astype(np.float32)
    y = (np.sin(3 * X[:, 0]) + X[:, 1] * X[:, 2] + 0.5 * X[:, 3 % cols] + 0.1 * rng.normal(size=rows))
    X[rng.random(X.shape) < nan] = np.nan
    return X, y.astype(np.float32)


def _depths(nodes):
    d = np.zeros(len(nodes), int)
    for i, n in enumerate(nodes):
        if n["left"] >= 0:
            d[n["left"]] = d[n["right"]] = d[i] + 1
    return d


def test_depthwise_beyond_ten_levels():
    X, y = _data(20000, 6, 0.05, 31)
    trees = _run(X, y, dict(max_depth=13, min_child_weight=0.0, max_bin=64), 3)
    assert max(_depths(t).max() for t in trees) > 10


def test_levels_wider_than_one_batch():
    X, y = _data(40000, 5, 0.02, 32)
    trees = _run(X, y, dict(max_depth=12, min_child_weight=0.0, max_bin=128), 2)
    widest = max(np.sum((_depths(t) == d) & (t["left"] >= 0)) for t in trees for d in range(12))
    assert widest > 256


def test_lossguide_with_leaf_budget_weights_and_logistic():
    X, y = _data(15000, 8, 0.1, 33)
    w = np.random.default_rng(3).random(15000).astype(np.float32) + 0.1
    trees = _run(X, (y > 0).astype(np.float32),
                 dict(objective="binary:logistic", grow_policy="lossguide", max_depth=0, max_leaves=31), 4,
                 weights=w)
    assert all(np.sum(t["left"] < 0) <= 31 for t in trees)


def test_lossguide_depth_limit_and_regularisation():
    X, y = _data(12000, 7, 0.05, 34)
    _run(X, y, dict(grow_policy="lossguide", max_depth=6, reg_alpha=0.5, reg_lambda=2.0, max_delta_step=0.4,
                    min_split_loss=0.01, min_child_weight=2.0), 3)


def test_depthwise_leaf_budget_multiclass():
    rng = np.random.default_rng(35)
    X = rng.normal(size=(9000, 8)).astype(np.float32)
    y = np.argmax(X[:, :4] @ rng.normal(size=(4, 3)), axis=1).astype(np.float32)
    _run(X, y, dict(objective="multi:softprob", num_class=3, max_depth=8, max_leaves=20), 2)


def test_two_byte_codes():
    # 256 bins with missing values: the codes are uint16.
    X, y = _data(30000, 4, 0.15, 36)
    _run(X, y, dict(grow_policy="lossguide", max_depth=0, max_leaves=64, max_bin=256), 2)


def test_python_api_predictions_follow_the_training_margins():
    import xgboost as xgb
    X, y = _data(10000, 6, 0.05, 37)
    d = xgb.DMatrix(X, label=y)
    for params in (dict(grow_policy="lossguide", max_leaves=48, max_depth=0), dict(max_depth=14)):
        bst = xgb.train(dict(params, tree_method="hist", device="cuda"), d, 5)
        # Raw-feature prediction (thresholds) and the training margins (bins)
        # walk the same trees.
        np.testing.assert_array_equal(bits(bst.predict(d, output_margin=True)),
                                      bits(bst.predict(xgb.DMatrix(X), output_margin=True)))
        raw = bst.save_raw("json")
        again = xgb.Booster(model_file=bytearray(raw))
        np.testing.assert_array_equal(bits(again.predict(xgb.DMatrix(X))), bits(bst.predict(xgb.DMatrix(X))))


def test_sparse_row_histograms():
    # cuda_sparse_hist=1: node histograms from each row's present values,
    # missing bins from the node totals; the trees are the oracle's.
    X, y = _data(20000, 30, 0.9, 38)
    _run(X, y, dict(max_depth=6, cuda_sparse_hist=1, max_bin=64), 3)
    _run(X, y, dict(grow_policy="lossguide", max_depth=0, max_leaves=40, cuda_sparse_hist=1), 2)
    rng = np.random.default_rng(6)
    Xc = rng.normal(size=(8000, 5)).astype(np.float32)  # no missing values
    _run(Xc, Xc[:, 0] * 2 + Xc[:, 1], dict(max_depth=5, cuda_sparse_hist=1), 2)

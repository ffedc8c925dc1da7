"""More device-against-oracle training cases, bit for bit: feature counts
that leave a partial 32-feature group, two-bin cuts, a given base_score,
zero sample weights, many classes and a large min_child_weight."""
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


def _data(rows, cols, nan, seed):
    rng = np.random.default_rng(seed)
    X = rng.normal(size=(rows, cols)).astype(np.float32)
    y = (X[:, : min(cols, 8)].astype(np.float64).sum(1) + 0.2 * rng.normal(size=rows)).astype(np.float32)
    X[rng.random(X.shape) < nan] = np.nan
    return X, y


@pytest.mark.parametrize("cols", [33, 65, 200])
def test_partial_feature_groups(cols):
    X, y = _data(6000, cols, 0.05, cols)
    _run(X, y, dict(max_depth=6, eta=0.3), 3)


def test_two_bins_and_given_base_score():
    X, y = _data(5000, 6, 0.1, 21)
    _run(X, y, dict(max_depth=5, max_bin=2, base_score=0.25), 3)
    yb = (y > 0).astype(np.float32)
    _run(X, yb, dict(objective="binary:logistic", max_depth=5, base_score=0.7), 3)


def test_zero_sample_weights_and_large_min_child_weight():
    X, y = _data(8000, 7, 0.0, 22)
    w = np.random.default_rng(5).random(8000).astype(np.float32) * 2
    w[::3] = 0.0
    _run(X, y, dict(max_depth=7, min_child_weight=40.0), 4, weights=w)


def test_many_classes():
    rng = np.random.default_rng(23)
    X = rng.normal(size=(6000, 10)).astype(np.float32)
    y = (np.argmax(X[:, :6] @ rng.normal(size=(6, 12)), axis=1)).astype(np.float32)
    _run(X, y, dict(objective="multi:softprob", num_class=12, max_depth=4, eta=0.3), 2)

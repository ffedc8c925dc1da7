"""CUDA product vs the oracle (and the reference's golden vectors), bit for
bit: cuts and bins, gradients and their fixed-point scales, whole training
runs (every node of every tree, and the training margins)."""
import os

import numpy as np
import pytest

import checkers as C
import product as P

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "reference_vectors.npz")


def bits(a):
    a = np.ascontiguousarray(a)
    return a.view(np.uint32) if a.dtype == np.float32 else a


def assert_same_trees(got, want):
    assert len(got) == len(want)
    for t, (g, w) in enumerate(zip(got, want)):
        assert len(g) == len(w), "tree %d: %d vs %d nodes" % (t, len(g), len(w))
        for f in ("left", "right", "parent", "feature"):
            np.testing.assert_array_equal(g[f], w[f], err_msg="tree %d %s" % (t, f))
        for f in ("leaf", "cover"):
            np.testing.assert_array_equal(bits(g[f]), bits(w[f]), err_msg="tree %d %s" % (t, f))
        internal = w["left"] >= 0
        for f in ("threshold", "gain"):
            np.testing.assert_array_equal(bits(g[f][internal]), bits(w[f][internal]),
                                          err_msg="tree %d %s" % (t, f))
        np.testing.assert_array_equal(g["default_left"][internal], w["default_left"][internal])
        np.testing.assert_array_equal(g["split_bin"][internal], w["split_bin"][internal])


def test_quantize_matches_reference_golden_vectors():
    g = np.load(GOLDEN)
    names = sorted({k[2:-2] for k in g.files if k.startswith("q_") and k.endswith("_X")})
    for name in names:
        X, mb = g["q_%s_X" % name], int(g["q_%s_maxbin" % name][0])
        cuts, counts, minima, bins = P.quantize(X, mb)
        np.testing.assert_array_equal(counts, g["q_%s_counts" % name], err_msg=name)
        np.testing.assert_array_equal(bits(cuts), bits(g["q_%s_cuts" % name]), err_msg=name)
        np.testing.assert_array_equal(bins, g["q_%s_bins" % name], err_msg=name)


@pytest.mark.parametrize("shape,nan,mb", [((100000, 32), 0.0, 256), ((100000, 32), 0.15, 256),
                                          ((5000, 7), 0.5, 16), ((3, 2), 0.0, 256)])
def test_quantize_matches_oracle(shape, nan, mb):
    rng = np.random.default_rng(1337)
    X = rng.normal(size=shape).astype(np.float32)
    X[rng.random(shape) < nan] = np.nan
    o = C.oracle()
    cuts, counts, minima = o.sketch_cuts(X, mb)
    want = o.quantize(X, cuts, counts)
    pc, pn, pm, pb = P.quantize(X, mb)
    np.testing.assert_array_equal(pn, counts)
    np.testing.assert_array_equal(bits(pc), bits(cuts))
    np.testing.assert_array_equal(pb, want)


@pytest.mark.parametrize("objective,groups,weighted", [
    ("reg:squarederror", 1, False), ("reg:squarederror", 1, True), ("binary:logistic", 1, False),
    ("binary:logistic", 1, True), ("multi:softprob", 4, False), ("multi:softprob", 10, True)])
def test_gradients_and_scales_match_oracle(objective, groups, weighted):
    rng = np.random.default_rng(7)
    n = 50000
    margins = (rng.normal(size=(n, groups)) * 3).astype(np.float32)
    if objective == "multi:softprob":
        labels = rng.integers(0, groups, n).astype(np.float32)
    elif objective == "binary:logistic":
        labels = (rng.random(n) < 0.3).astype(np.float32)
    else:
        labels = rng.normal(size=n).astype(np.float32)
    w = rng.random(n).astype(np.float32) * 3 if weighted else None
    want = C.oracle_gradients(objective, margins, labels, w, 1.5 if weighted else 1.0)
    pairs, scales = P.gradients(objective, margins, labels, w, 1.5 if weighted else 1.0)
    np.testing.assert_array_equal(bits(pairs), bits(want))
    want_scales = C.oracle().gradient_scales(want)
    np.testing.assert_array_equal(bits(scales), bits(want_scales))


def _data(rows, cols, nan, seed=1337):
    rng = np.random.default_rng(seed)
    X = rng.normal(size=(rows, cols)).astype(np.float32)
    w = np.random.default_rng(seed + 1).normal(size=cols)
    y = (X.astype(np.float64) @ w + 0.1 * rng.normal(size=rows)).astype(np.float32)
    X[rng.random(X.shape) < nan] = np.nan
    return X, y


TRAIN_CASES = {
    "c0_like": (dict(max_depth=6, eta=0.3), 20000, 32, 0.0, 10),
    "c1_like_nan15": (dict(max_depth=6, eta=0.3), 20000, 32, 0.15, 10),
    "depth8": (dict(max_depth=8, eta=0.3), 30000, 16, 0.0, 4),
    "depth10_nan": (dict(max_depth=10, eta=0.1), 20000, 8, 0.05, 3),
    "regularised": (dict(max_depth=5, eta=0.5, reg_lambda=0.0, reg_alpha=0.8, min_split_loss=3.0,
                         min_child_weight=5.0, max_delta_step=0.7), 8000, 6, 0.1, 5),
    "depth1": (dict(max_depth=1), 1000, 3, 0.0, 3),
    "u16_bins_with_missing": (dict(max_depth=4, max_bin=256), 3000, 4, 0.3, 3),
    "few_bins": (dict(max_depth=6, max_bin=4), 5000, 5, 0.1, 4),
}


@pytest.mark.parametrize("name", sorted(TRAIN_CASES))
def test_train_matches_oracle(name):
    params, rows, cols, nan, rounds = TRAIN_CASES[name]
    X, y = _data(rows, cols, nan)
    full = C.train_params(params)
    trees_o, margins_o, _ = C.oracle_train(X, y, full, rounds)
    trees_p, margins_p = P.train(X, y, {k: v for k, v in full.items() if k != "num_class"}, rounds)
    assert_same_trees(trees_p, trees_o)
    np.testing.assert_array_equal(bits(margins_p), bits(margins_o))


@pytest.mark.parametrize("weighted", [False, True])
def test_train_logistic_matches_oracle(weighted):
    X, y = _data(20000, 12, 0.05, seed=4)
    y = (y > 0).astype(np.float32)
    w = np.random.default_rng(9).random(len(y)).astype(np.float32) * 2 if weighted else None
    params = C.train_params(dict(objective="binary:logistic", max_depth=7, eta=0.1,
                                 scale_pos_weight=2.0 if weighted else 1.0))
    trees_o, margins_o, _ = C.oracle_train(X, y, params, 6, weights=w)
    trees_p, margins_p = P.train(X, y, {k: v for k, v in params.items() if k != "num_class"}, 6, weights=w)
    assert_same_trees(trees_p, trees_o)
    np.testing.assert_array_equal(bits(margins_p), bits(margins_o))


def test_train_softprob_matches_oracle():
    rng = np.random.default_rng(11)
    n, k = 12000, 4
    X = rng.integers(0, 256, size=(n, 20)).astype(np.float32)
    X[rng.random(X.shape) < 0.7] = 0
    y = rng.integers(0, k, n).astype(np.float32)
    params = C.train_params(dict(objective="multi:softprob", num_class=k, max_depth=6, eta=0.3))
    trees_o, margins_o, _ = C.oracle_train(X, y, params, 3)
    trees_p, margins_p = P.train(X, y, params, 3)
    assert_same_trees(trees_p, trees_o)
    np.testing.assert_array_equal(bits(margins_p), bits(margins_o))


@pytest.mark.parametrize("rows", [1, 2, 31, 33, 257])
def test_train_tiny_inputs(rows):
    X, y = _data(rows, 3, 0.2, seed=rows)
    params = C.train_params(dict(max_depth=4, min_child_weight=0.0))
    trees_o, margins_o, _ = C.oracle_train(X, y, params, 2)
    trees_p, margins_p = P.train(X, y, {k: v for k, v in params.items() if k != "num_class"}, 2)
    assert_same_trees(trees_p, trees_o)
    np.testing.assert_array_equal(bits(margins_p), bits(margins_o))


def test_constant_label_and_all_missing_column():
    X, _ = _data(3000, 4, 0.0)
    X[:, 1] = np.nan
    y = np.full(3000, 2.5, np.float32)
    params = C.train_params(dict(max_depth=6))
    trees_o, margins_o, _ = C.oracle_train(X, y, params, 2)
    trees_p, margins_p = P.train(X, y, {k: v for k, v in params.items() if k != "num_class"}, 2)
    assert_same_trees(trees_p, trees_o)
    np.testing.assert_array_equal(bits(margins_p), bits(margins_o))


def test_python_api_matches_oracle_margins():
    import xgboost as xgb
    X, y = _data(100000, 32, 0.0)
    params = {"tree_method": "hist", "device": "cuda", "max_depth": 6, "eta": 0.3,
              "max_bin": 256, "seed": 42, "objective": "reg:squarederror"}
    d = xgb.DMatrix(X, label=y)
    bst = xgb.train(params, d, 5)
    _, margins_o, _ = C.oracle_train(X, y, C.train_params(dict(max_depth=6, eta=0.3)), 5)
    np.testing.assert_array_equal(bits(bst.predict(d, output_margin=True)), bits(margins_o[:, 0]))
    # A fresh matrix with the same values goes through the raw-threshold path.
    d2 = xgb.DMatrix(X)
    np.testing.assert_array_equal(bits(bst.predict(d2)), bits(margins_o[:, 0]))
    assert bst.num_boosted_rounds() == 5


def test_c2_full_size_matches_oracle():
    X, y = _data(262144, 64, 0.0)
    params = C.train_params(dict(max_depth=8, eta=0.3))
    trees_o, margins_o, _ = C.oracle_train(X, y, params, 3)
    trees_p, margins_p = P.train(X, y, {k: v for k, v in params.items() if k != "num_class"}, 3)
    assert_same_trees(trees_p, trees_o)
    np.testing.assert_array_equal(bits(margins_p), bits(margins_o))


def test_zero_copy_infinity_is_reported_on_first_use():
    import xgboost as xgb
    X = np.ones((64, 3), np.float32)
    X[5, 1] = np.inf
    d = xgb.DMatrix(X, label=np.zeros(64, np.float32))
    with pytest.raises(xgb.XGBoostError, match="infinity"):
        xgb.train({"device": "cuda"}, d, 1)


# Millions of rows with gradients of similar magnitude keep every |q| of a
# round within 42 bits (scale = 2^62 / 2^bitlen(sum |v|)), which selects the
# staged two-limb histogram path; smaller cases run the three-limb path.
def test_two_limb_logistic_u16_partial_group_matches_oracle():
    rows, cols = 3_000_000, 40
    rng = np.random.default_rng(5)
    X = rng.normal(size=(rows, cols)).astype(np.float32)
    X[rng.random(X.shape) < 0.05] = np.nan
    y = (np.nan_to_num(X[:, 0]) + 0.5 * rng.normal(size=rows) > 0).astype(np.float32)
    params = C.train_params(dict(objective="binary:logistic", max_depth=6, eta=0.3))
    trees_o, margins_o, _ = C.oracle_train(X, y, params, 3)
    trees_p, margins_p = P.train(X, y, {k: v for k, v in params.items() if k != "num_class"}, 3)
    assert_same_trees(trees_p, trees_o)
    np.testing.assert_array_equal(bits(margins_p), bits(margins_o))


def test_two_limb_unit_hessian_u8_matches_oracle():
    rows, cols = 3_000_000, 20
    rng = np.random.default_rng(6)
    X = rng.normal(size=(rows, cols)).astype(np.float32)
    y = np.where(X[:, 1] + 0.3 * rng.normal(size=rows) > 0, 1.0, -1.0).astype(np.float32)
    params = C.train_params(dict(max_depth=5, eta=0.3, max_bin=64))
    trees_o, margins_o, _ = C.oracle_train(X, y, params, 3)
    trees_p, margins_p = P.train(X, y, {k: v for k, v in params.items() if k != "num_class"}, 3)
    assert_same_trees(trees_p, trees_o)
    np.testing.assert_array_equal(bits(margins_p), bits(margins_o))


def _c3_like(rows, cols, classes, seed):
    """Integer-valued images in the manner of BASELINE's c3: per class a
    pattern P[k] of uniform(0, 255) intensities; a cell is zero where its
    class pattern plus per-row noise falls below the class's 80th percentile
    (so classes overlap and trees grow), else clip(Poisson(P[k]), 0, 255);
    balanced shuffled classes."""
    rng = np.random.default_rng(seed)
    P = rng.uniform(0, 255, size=(classes, cols)).astype(np.float32)
    thr = np.quantile(P, 0.8, axis=1, keepdims=True)
    y = rng.permutation(np.arange(rows) % classes)
    X = np.clip(rng.poisson(P[y]), 0, 255).astype(np.float32)
    X[P[y] + rng.normal(0, 60, size=X.shape) < thr[y]] = 0.0
    return X, y.astype(np.float32)


def test_c3_shape_softprob_784_features_10_classes_matches_oracle():
    """BASELINE's c3 shape: 784 features (25 feature groups of 32, the last
    partial), 10 classes (10 trees per round), ~80 % exact zeros, integer
    values with at most 256 distinct values per feature (exact cuts, uint8
    codes, no missing bin)."""
    X, y = _c3_like(24000, 784, 10, seed=31)
    assert (X == 0).mean() > 0.75
    params = C.train_params(dict(objective="multi:softprob", num_class=10, max_depth=6, eta=0.3))
    trees_o, margins_o, _ = C.oracle_train(X, y, params, 2)
    trees_p, margins_p = P.train(X, y, params, 2)
    assert len(trees_p) == 20
    assert_same_trees(trees_p, trees_o)
    np.testing.assert_array_equal(bits(margins_p), bits(margins_o))


def test_c4_width_logistic_128_features_matches_oracle():
    """BASELINE's c4 row format at 128 features: 256 bins plus missing
    (uint16 codes), 5 % NaN, binary:logistic, depth 10, 2 rounds."""
    X, _ = _data(60000, 128, 0.05, seed=33)
    rng = np.random.default_rng(34)
    y = (rng.random(60000) < 0.35).astype(np.float32)
    params = C.train_params(dict(objective="binary:logistic", max_depth=10, eta=0.1))
    trees_o, margins_o, _ = C.oracle_train(X, y, params, 2)
    trees_p, margins_p = P.train(X, y, {k: v for k, v in params.items() if k != "num_class"}, 2)
    assert_same_trees(trees_p, trees_o)
    np.testing.assert_array_equal(bits(margins_p), bits(margins_o))

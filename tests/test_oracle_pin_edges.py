"""Pins the oracle against the reference's own serial kernel functions
(oracle/_ref) on the missing-value edge families the reference's own tests
exercise (tests/test_histogram_missing.py:11-20, 63-80 of the reference):
mostly-missing rows with explicit zeros, rows that are entirely missing, a
column that is entirely missing and a partial last feature group; row
counts around the SIMD width and the histogram tile (1, 31-33, 255-257,
2049); a matrix with no value at all; and dense data with no missing value.
Each case runs three squared-error rounds at depth 4 (base margin 0) and
compares cuts, bins, gradient scales, quantised gradients, node tables and
per-row leaf values bit for bit."""
import numpy as np
import pytest

import checkers as C

pytestmark = pytest.mark.skipif(not C.have_reference(),
                                reason="reference harness not built (no reference checkout)")

TREE = dict(max_depth=4, eta=0.3, reg_lambda=1.0, reg_alpha=0.0, min_child_weight=1.0,
            max_delta_step=0.0, min_split_loss=0.0)


def _bits(a):
    return np.ascontiguousarray(a).view(np.uint32 if a.dtype == np.float32 else a.dtype)


def _sparse_rows(rows, density=0.05, seed=7315):
    """7 features, about `density` of the cells present; a label from a few
    of the features before masking; explicit zeros in feature 0 every 17th
    row; every 29th row entirely missing; the last feature never present."""
    rng = np.random.default_rng(seed)
    X = rng.normal(size=(rows, 7)).astype(np.float32)
    y = (X[:, 0] - X[:, 1] * X[:, 2] + X[:, 3] ** 2).astype(np.float32)
    X[rng.random(X.shape) >= density] = np.nan
    X[1::17, 0] = 0.0
    X[::29] = np.nan
    X[:, -1] = np.nan
    return X, y


def _pin(X, y, max_bin, rounds=3):
    o, r = C.oracle(), C.reference()
    co, cr = o.sketch_cuts(X, max_bin), r.sketch_cuts(X, max_bin)
    for a, b in zip(co, cr):
        np.testing.assert_array_equal(_bits(a), _bits(b))
    bins = o.quantize(X, co[0], co[1])
    np.testing.assert_array_equal(bins, r.quantize(X, cr[0], cr[1]))
    margins = np.zeros((len(y), 1), np.float32)
    nodes = 0
    for _ in range(rounds):
        pairs = C.oracle_gradients("reg:squarederror", margins, y)
        np.testing.assert_array_equal(_bits(pairs), _bits(C.reference_gradients("reg:squarederror", margins, y)))
        scale = o.gradient_scales(pairs)
        np.testing.assert_array_equal(_bits(scale), _bits(r.gradient_scales(pairs)))
        q = o.quantize_gradients(pairs, scale)
        np.testing.assert_array_equal(q, r.quantize_gradients(pairs, scale))
        no, lo = o.grow_tree(bins, q[:, 0, :], scale[0], co[0], co[1], co[2], TREE)
        nr, lr = r.grow_tree(bins, q[:, 0, :], scale[0], co[0], co[1], co[2], TREE)
        assert no.tobytes() == nr.tobytes()
        # The harness reports a row's leaf as 0 + leaf (the reference's
        # predict kernel), which reads a -0.0 leaf as +0.0.
        np.testing.assert_array_equal(_bits(np.float32(0) + lo), _bits(lr))
        margins[:, 0] += lo
        nodes += len(no)
    return nodes, bins


@pytest.mark.parametrize("max_bin", [16, 256])
def test_mostly_missing_rows_with_explicit_zeros(max_bin):
    X, y = _sparse_rows(769)
    nodes, bins = _pin(X, y, max_bin)
    assert (bins == C.MISSING).mean() > 0.9
    assert (bins[:, -1] == C.MISSING).all() and (bins[::29] == C.MISSING).all()
    assert nodes > 3


@pytest.mark.parametrize("rows", [1, 31, 32, 33, 255, 256, 257, 2049])
def test_partial_simd_groups_and_tiles(rows):
    X, y = _sparse_rows(rows)
    if rows == 1:
        X.fill(np.nan)
    _pin(X, y, 16, rounds=1)


def test_matrix_without_any_value():
    X = np.full((529, 7), np.nan, np.float32)
    y = np.linspace(-1, 1, len(X), dtype=np.float32)
    nodes, bins = _pin(X, y, 16, rounds=2)
    assert (bins == C.MISSING).all()
    assert nodes == 2  # one leaf per round


def test_dense_ramp_without_missing_values():
    X = np.arange(257 * 7, dtype=np.float32).reshape(-1, 7) / 100
    y = (X[:, 0] > 3).astype(np.float32)
    nodes, bins = _pin(X, y, 256, rounds=2)
    assert not (bins == C.MISSING).any()
    assert nodes > 2


def _tree_family(case, rows=513):
    """The depth-wise tree families of the reference's own tests
    (tests/test_gpu_tree.py:36-80 of the reference), restated: 7 N(0, 1)
    features and a label from four of them, then one change per case."""
    rng = np.random.default_rng(82171)
    X = rng.normal(size=(rows, 7)).astype(np.float32)
    y = (X[:, 0] - X[:, 1] * X[:, 2] + X[:, 3] ** 2).astype(np.float32)
    w = None
    objective, groups = "reg:squarederror", 1
    if case == "missing":
        X[::7, 0] = np.nan
        X[::11, 3] = np.nan
        X[:, 6] = np.nan
    elif case == "ties":   # four values, every feature a copy of the first
        X[:, 0] = np.arange(rows) % 4
        X[:, 1:] = X[:, :1]
        y = (X[:, 0] >= 2).astype(np.float32)
    elif case == "constant":
        y.fill(0)
    elif case == "weighted":   # weights in (0.01, 3), every 13th row weight 0
        w = rng.uniform(0.01, 3, rows).astype(np.float32)
        w[::13] = 0
    elif case == "multiclass":
        y = np.argmax(X[:, :3], axis=1).astype(np.float32)
        objective, groups = "multi:softprob", 3
    elif case == "subnormal_features":
        tiny = np.nextafter(np.float32(0), np.float32(1))
        X[:, 0] = np.resize(np.asarray([-4 * tiny, -tiny, -0.0, 0.0, tiny, 4 * tiny], np.float32), rows)
        y = (np.arange(rows) % 6 >= 3).astype(np.float32)
    return X, y, w, objective, groups


def _zeros_as_positive(a):
    return np.where(a == 0, np.float32(0), a).astype(a.dtype)


def _thresholds_as_positive(nodes):
    out = nodes.copy()
    out["threshold"] = _zeros_as_positive(out["threshold"])
    return out


@pytest.mark.parametrize("case", ["regression", "missing", "ties", "constant", "weighted", "multiclass",
                                  "subnormal_features"])
def test_reference_tree_families(case):
    """max_bin 32, depth 4, three rounds (one tree per class), base margin 0:
    weighted cuts and gradients where the case has weights; the oracle's
    gradient pairs feed both growers (softmax probabilities may round
    differently through the host libm's exp). Each side grows from its own
    cuts. The one deliberate difference: the oracle (and the library) reads
    -0.0 as +0.0 in the sketch, while the reference keeps the sign of the
    first zero of a run, so where a column holds signed zeros a cut, and a
    threshold at that cut, may be -0.0 in the reference and +0.0 here. The
    two compare equal, so the bins, the splits and the leaf values are the
    same; every other bit is compared as is."""
    o, r = C.oracle(), C.reference()
    X, y, w, objective, groups = _tree_family(case)
    co, cr = o.sketch_cuts(X, 32, w), r.sketch_cuts(X, 32, w)
    np.testing.assert_array_equal(co[1], cr[1])
    np.testing.assert_array_equal(_bits(co[2]), _bits(cr[2]))
    signed_zero = (co[0] == 0) & (_bits(co[0]) != _bits(cr[0]))
    assert (case == "subnormal_features") or not signed_zero.any()
    assert not (_bits(co[0]) != _bits(cr[0]))[~signed_zero].any()
    assert (_bits(co[0])[signed_zero] == 0).all()
    bins = o.quantize(X, co[0], co[1])
    np.testing.assert_array_equal(bins, r.quantize(X, cr[0], cr[1]))
    margins = np.zeros((len(y), groups), np.float32)
    nodes = 0
    for _ in range(3):
        pairs = C.oracle_gradients(objective, margins, y, w)
        if objective == "reg:squarederror":
            np.testing.assert_array_equal(_bits(pairs), _bits(C.reference_gradients(objective, margins, y, w)))
        scales = o.gradient_scales(pairs)
        np.testing.assert_array_equal(_bits(scales), _bits(r.gradient_scales(pairs)))
        q = o.quantize_gradients(pairs, scales)
        np.testing.assert_array_equal(q, r.quantize_gradients(pairs, scales))
        for g in range(groups):
            no, lo = o.grow_tree(bins, q[:, g, :], scales[g], co[0], co[1], co[2], TREE)
            nr, lr = r.grow_tree(bins, q[:, g, :], scales[g], cr[0], cr[1], cr[2], TREE)
            assert len(no) == len(nr), (case, g)
            if signed_zero.any():
                assert _thresholds_as_positive(no).tobytes() == _thresholds_as_positive(nr).tobytes(), (case, g)
            else:
                assert no.tobytes() == nr.tobytes(), (case, g)
            np.testing.assert_array_equal(_bits(np.float32(0) + lo), _bits(lr))
            margins[:, g] += lo
            nodes += len(no)
    if case == "constant":
        assert nodes == 3
    else:
        assert nodes > 3 * groups


@pytest.mark.parametrize("bins", [2, 31, 32, 33, 127, 256])
@pytest.mark.parametrize("custom", [False, True])
def test_regularised_split_scan_families(bins, custom):
    """The split-scan family of the reference's tests
    (tests/test_split_scan.py:8-31 of the reference), restated for the
    depth-wise path: values on a 1/64 grid (many ties), feature 1 a copy of
    feature 0, missing values in three features, alpha 0.17, lambda 0.4,
    max_delta_step 1, min_child_weight 0.5, eta 0.2; and with `custom` the
    caller's fixed gradients in quarters and hessians of 1.25 or -0.5."""
    o, r = C.oracle(), C.reference()
    rng = np.random.default_rng(833)
    X = rng.integers(-200, 201, (1025, 7)).astype(np.float32) / 64
    X[:, 1] = X[:, 0]
    y = (1.2 * X[:, 0] - X[:, 3] ** 2 + X[:, 5]).astype(np.float32)
    X[::11, 2] = np.nan
    X[::13, 4] = np.nan
    X[::17, 6] = np.nan
    tp = dict(max_depth=4, eta=0.2, reg_lambda=0.4, reg_alpha=0.17, min_child_weight=0.5,
              max_delta_step=1.0, min_split_loss=0.0)
    co, cr = o.sketch_cuts(X, bins), r.sketch_cuts(X, bins)
    for a, b in zip(co, cr):
        np.testing.assert_array_equal(_bits(a), _bits(b))
    bins_ = o.quantize(X, co[0], co[1])
    np.testing.assert_array_equal(bins_, r.quantize(X, cr[0], cr[1]))
    row = np.arange(len(X))
    margins = np.zeros((len(X), 1), np.float32)
    nodes = 0
    for _ in range(3):
        if custom:
            pairs = np.stack([((row % 7 - 3) / 4), np.where(row % 5, 1.25, -0.5)], 1).astype(np.float32)[:, None, :]
        else:
            pairs = C.oracle_gradients("reg:squarederror", margins, y)
        scale = o.gradient_scales(pairs)
        np.testing.assert_array_equal(_bits(scale), _bits(r.gradient_scales(pairs)))
        q = o.quantize_gradients(pairs, scale)
        np.testing.assert_array_equal(q, r.quantize_gradients(pairs, scale))
        no, lo = o.grow_tree(bins_, q[:, 0, :], scale[0], co[0], co[1], co[2], tp)
        nr, lr = r.grow_tree(bins_, q[:, 0, :], scale[0], cr[0], cr[1], cr[2], tp)
        assert no.tobytes() == nr.tobytes()
        np.testing.assert_array_equal(_bits(np.float32(0) + lo), _bits(lr))
        margins[:, 0] += lo
        nodes += len(no)
    assert nodes >= 3

"""Quantile cuts on the GPU (csrc/sketch_gpu.cu running the data-parallel
sketch of csrc/sketch_par.h) against the host sketch, bit for bit: missing
values, ties and long runs, signed zeros, empty and constant features, float
and integer weights, many batches and levels, and features processed in
groups; then quantisation with the GPU cuts trains the same model."""
import os

import numpy as np
import pytest

import product as P

pytestmark = pytest.mark.gpu


def _same(X, max_bin, weights=None):
    want = P.sketch(X, max_bin, weights)
    got = P.sketch_device(X, max_bin, weights)
    np.testing.assert_array_equal(got[1], want[1])
    np.testing.assert_array_equal(got[0].view(np.uint32), want[0].view(np.uint32))
    np.testing.assert_array_equal(got[2].view(np.uint32), want[2].view(np.uint32))


@pytest.mark.parametrize("max_bin", [2, 16, 256])
def test_continuous_values_with_missing(max_bin):
    rng = np.random.default_rng(max_bin)
    X = rng.normal(size=(20000, 9)).astype(np.float32)
    X[rng.random(X.shape) < 0.1] = np.nan
    _same(X, max_bin)


def test_runs_ties_constants_and_signed_zeros():
    rng = np.random.default_rng(2)
    n = 30000
    X = np.zeros((n, 6), np.float32)
    X[:, 0] = np.sort(rng.integers(0, 30, n))
    X[:, 1] = 3.0
    X[:, 2] = rng.integers(0, 3, n)
    X[:, 3] = np.where(rng.random(n) < 0.5, 0.0, -0.0)
    X[:, 4] = np.nan
    X[:, 5] = rng.normal(size=n)
    X[rng.random(n) < 0.3, 5] = np.nan
    for max_bin in (32, 256):
        _same(X, max_bin)


def test_weights():
    rng = np.random.default_rng(3)
    n = 25000
    X = rng.normal(size=(n, 3)).astype(np.float32)
    X[:, 1] = np.sort(rng.integers(0, 100, n)).astype(np.float32)
    X[rng.random(X.shape) < 0.05] = np.nan
    w = rng.random(n).astype(np.float32) * 3
    w[::7] = 0.0
    for max_bin in (8, 256):
        _same(X, max_bin, w)
    _same(X, 64, rng.integers(0, 4, n).astype(np.float32))


def test_many_batches_and_levels():
    rng = np.random.default_rng(1)
    X = rng.normal(size=(400000, 3)).astype(np.float32)
    X[:, 1] = np.round(X[:, 1] * 40) / 40
    _same(X, 4)
    _same(X, 256)


def test_few_rows():
    rng = np.random.default_rng(4)
    for rows in (1, 2, 17):
        X = rng.normal(size=(rows, 3)).astype(np.float32)
        X[0, 0] = np.nan
        _same(X, 256)


def test_training_with_device_cuts():
    import xgboost as xgb
    rng = np.random.default_rng(5)
    X = rng.normal(size=(20000, 8)).astype(np.float32)
    X[rng.random(X.shape) < 0.05] = np.nan
    y = (np.nan_to_num(X) @ rng.normal(size=8)).astype(np.float32)
    params = {"tree_method": "hist", "device": "cuda", "max_depth": 6}
    host = xgb.train(params, xgb.DMatrix(X, label=y), 4).save_raw("json")
    os.environ["XGBB_SKETCH"] = "device"
    try:
        dev = xgb.train(params, xgb.DMatrix(X, label=y), 4).save_raw("json")
    finally:
        del os.environ["XGBB_SKETCH"]
    assert dev == host


def _same_as_oracle(X, max_bin, weights=None):
    import checkers as C
    cuts, counts, minima = C.oracle().sketch_cuts(X, max_bin, weights)
    got = P.sketch_device(X, max_bin, weights)
    np.testing.assert_array_equal(got[1], counts)
    np.testing.assert_array_equal(got[0].view(np.uint32), cuts.view(np.uint32))
    np.testing.assert_array_equal(got[2].view(np.uint32), minima.view(np.uint32))


@pytest.mark.parametrize("case", ["weighted_with_missing", "unweighted_ties_missing", "c4_like"])
def test_device_sketch_matches_oracle(case):
    """XGBBSketchDevice against the oracle's restatement of the reference's
    sketch (kernels/quantile.metal.h:19-400, src/quantile.cpp:22-213), bit
    for bit, with no product code on the checking side."""
    rng = np.random.default_rng({"weighted_with_missing": 11, "unweighted_ties_missing": 12, "c4_like": 13}[case])
    if case == "weighted_with_missing":
        n = 40000
        X = rng.normal(size=(n, 7)).astype(np.float32)
        X[:, 2] = rng.integers(0, 50, n)
        X[rng.random(X.shape) < 0.12] = np.nan
        w = (rng.random(n) * 4).astype(np.float32)
        w[::11] = 0.0
        for max_bin in (16, 256):
            _same_as_oracle(X, max_bin, w)
    elif case == "unweighted_ties_missing":
        n = 60000
        X = rng.integers(-40, 40, size=(n, 5)).astype(np.float32)
        X[:, 4] = rng.normal(size=n)
        X[rng.random(X.shape) < 0.3] = np.nan
        X[:, 1] = np.nan
        for max_bin in (2, 64, 256):
            _same_as_oracle(X, max_bin)
    else:
        X = rng.normal(size=(200000, 16)).astype(np.float32)
        X[rng.random(X.shape) < 0.05] = np.nan
        _same_as_oracle(X, 256)

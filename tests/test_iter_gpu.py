"""GPU checks of the host-side entry points around training: a QuantileDMatrix
or DMatrix built from a batch iterator trains the same trees as one built
from the concatenated arrays, in-place prediction equals DMatrix prediction,
and a round slice predicts like an iteration range."""
import numpy as np
import pytest

import xgboost as xgb
from test_ingest_cpu import Batches, _parts

pytestmark = pytest.mark.gpu

PARAMS = {"objective": "reg:squarederror", "tree_method": "hist", "device": "cuda",
          "max_depth": 5, "eta": 0.3, "max_bin": 64}


def _whole(parts):
    X = np.concatenate([p["data"] for p in parts])
    y = np.concatenate([p["label"] for p in parts])
    w = np.concatenate([p["weight"] for p in parts])
    return X, y, w


def test_iterator_matrices_train_like_arrays():
    rng = np.random.default_rng(11)
    parts = _parts(rng, [3000, 1, 2500, 1200], cols=7)
    X, y, w = _whole(parts)
    want = xgb.train(PARAMS, xgb.QuantileDMatrix(X, y, weight=w, max_bin=64), 4)
    got = xgb.train(PARAMS, xgb.QuantileDMatrix(Batches(parts), max_bin=64), 4)
    assert bytes(got.save_raw("json")) == bytes(want.save_raw("json"))
    lazy = xgb.train(PARAMS, xgb.DMatrix(Batches(parts)), 4)
    assert bytes(lazy.save_raw("json")) == bytes(want.save_raw("json"))
    # A validation matrix built from an iterator with the training cuts.
    ref = xgb.QuantileDMatrix(X, y, weight=w, max_bin=64)
    valid = xgb.QuantileDMatrix(Batches(parts[:2]), max_bin=64, ref=ref)
    assert valid.num_row() == 3001


def test_inplace_predict_and_slices_match_dmatrix_prediction():
    rng = np.random.default_rng(12)
    X = rng.normal(size=(4000, 5)).astype(np.float32)
    X[rng.random(X.shape) < 0.1] = np.nan
    y = (np.nan_to_num(X[:, 0]) - np.nan_to_num(X[:, 2]) + 0.2 * rng.normal(size=4000)).astype(np.float32)
    b = xgb.train(PARAMS, xgb.DMatrix(X, label=y), 6)
    dm = xgb.DMatrix(X)
    np.testing.assert_array_equal(b.inplace_predict(X), b.predict(dm))
    np.testing.assert_array_equal(b.inplace_predict(X.astype(np.float64), predict_type="margin"),
                                  b.predict(dm, output_margin=True))
    margin = rng.normal(size=4000).astype(np.float32)
    np.testing.assert_array_equal(b.inplace_predict(X, base_margin=margin),
                                  b.predict(xgb.DMatrix(X, base_margin=margin)))
    Xm = np.where(np.isnan(X), -999.0, X).astype(np.float32)
    np.testing.assert_array_equal(b.inplace_predict(Xm, missing=-999.0), b.predict(dm))
    np.testing.assert_array_equal(b[:3].predict(dm), b.predict(dm, iteration_range=(0, 3)))
    np.testing.assert_array_equal(b[2:5].predict(dm, output_margin=True) - 0.0,
                                  b.predict(dm, output_margin=True, iteration_range=(2, 5)))

"""Pins the oracle's weighted quantile sketch against the reference's own
sketch kernels (oracle/_ref: runs, batch summaries, the level reduction and
the cut rule of kernels/quantile.metal.h, compiled for the host) on the
weight and value families of the reference's own cut tests
(tests/test_quantiles.py:9-20 of the reference): unit, fractional, integer
and zero weights, a column of row numbers, integer ties, long runs of
repeated rows, 70 % missing values, an empty column and all-zero weights,
from 17 to 100,003 rows and 2 to 256 bins. Cut values, cut counts and
minima must be equal bit for bit, and so must the bins. The library's own
host sketch (XGBBSketchHost, which needs no GPU; the GPU sketch equals it
bit for bit in the GPU tests) is held to the same cuts."""
import numpy as np
import pytest

import checkers as C
import product as P

pytestmark = pytest.mark.skipif(not C.have_reference(),
                                reason="reference harness not built (no reference checkout)")

FAMILIES = [
    (17, 4, "unit"), (257, 16, "unit"), (8193, 64, "unit"), (100003, 256, "unit"), (259, 2, "unit"),
    (4099, 3, "unit"), (8193, 31, "unit"), (8193, 33, "unit"), (257, 16, "fractional"),
    (8193, 64, "fractional"), (8193, 64, "integer"), (8193, 64, "zero-weights"), (4099, 16, "ties"),
    (4099, 16, "runs"), (4099, 16, "missing"), (4099, 16, "empty-column"), (4099, 16, "all-zero-weights"),
    (17, 64, "exact"),
]


def _bits(a):
    return np.ascontiguousarray(a).view(np.uint32)


def _family(rows, kind):
    """Three features (the second the row number) and per-row weights, one
    change per kind, restated from the shapes the reference's tests use."""
    rng = np.random.default_rng(941 + rows)
    X = rng.normal(size=(rows, 3)).astype(np.float32)
    X[:, 1] = np.arange(rows, dtype=np.float32)
    w = np.ones(rows, np.float32)
    if kind in ("integer", "zero-weights"):
        w = rng.integers(0, 9, rows).astype(np.float32)
        if kind == "zero-weights":
            w[::2] = 0
    elif kind != "unit":
        w = rng.uniform(0, 2, rows).astype(np.float32)
    if kind in ("ties", "runs"):
        X = rng.integers(-100, 101, size=X.shape).astype(np.float32)
        if kind == "runs":
            X = np.repeat(X[::31], 31, axis=0)[:rows]
    if kind == "missing":
        X[rng.uniform(size=X.shape) < 0.7] = np.nan
    if kind == "empty-column":
        X[:, 1] = np.nan
    if kind == "all-zero-weights":
        w[:] = 0
    return X, w


@pytest.mark.parametrize("rows,bins,kind", FAMILIES)
def test_weighted_cuts_match_the_reference(rows, bins, kind):
    o, r = C.oracle(), C.reference()
    X, w = _family(rows, kind)
    weights = None if kind == "unit" else w
    co, cr = o.sketch_cuts(X, bins, weights), r.sketch_cuts(X, bins, weights)
    np.testing.assert_array_equal(co[1], cr[1])
    np.testing.assert_array_equal(_bits(co[0]), _bits(cr[0]))
    np.testing.assert_array_equal(_bits(co[2]), _bits(cr[2]))
    np.testing.assert_array_equal(o.quantize(X, co[0], co[1]), r.quantize(X, cr[0], cr[1]))
    assert (co[1] >= 1).all()
    cp = P.sketch(X, bins, weights)
    np.testing.assert_array_equal(cp[1], cr[1])
    np.testing.assert_array_equal(_bits(cp[0]), _bits(cr[0]))
    np.testing.assert_array_equal(_bits(cp[2]), _bits(cr[2]))

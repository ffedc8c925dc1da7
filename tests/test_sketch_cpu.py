"""The product's host quantile sketch (csrc/sketch.cpp) against the oracle,
bit for bit, on the CPU: the edge families of the golden vectors, weights,
wide and tall matrices, and every thread count."""
import numpy as np
import pytest

import checkers as C
import product as P


def _cases():
    rng = np.random.default_rng(41)
    out = {}
    for rows in (1, 2, 31, 33, 257, 2049):
        X = rng.normal(size=(rows, 3)).astype(np.float32)
        X[:, 1] = np.round(X[:, 1] * 2)
        X[rng.random(rows) < 0.2, 2] = np.nan
        out["rows%d" % rows] = (X, 256, None)
    X = rng.normal(size=(600, 4)).astype(np.float32)
    X[:, 0] = np.nan
    X[:, 1] = 7.0
    X[:, 2] = rng.integers(0, 5, 600).astype(np.float32)
    X[:, 3] = (rng.normal(size=600) * 1e-39).astype(np.float32)
    out["special"] = (X, 16, None)
    X = rng.normal(size=(20000, 5)).astype(np.float32)
    X[rng.random(X.shape) < 0.15] = np.nan
    out["nan15"] = (X, 256, None)
    out["nan15_mb7"] = (X, 7, None)
    out["weighted"] = (X, 64, rng.uniform(0, 3, 20000).astype(np.float32))
    Xi = rng.integers(0, 300, size=(30000, 40)).astype(np.float32)
    Xi[rng.random(Xi.shape) < 0.7] = 0
    out["integer_images"] = (Xi, 256, None)
    out["signed_zero"] = (np.array([[-0.0], [0.0], [1.0], [-0.0], [2.0]], np.float32), 4, None)
    return out


CASES = _cases()


@pytest.mark.parametrize("name", sorted(CASES))
def test_product_sketch_matches_oracle(name):
    X, mb, w = CASES[name]
    want = C.oracle().sketch_cuts(X, mb, weights=w)
    got = P.sketch(X, mb, weights=w)
    for a, b in zip(got, want):
        np.testing.assert_array_equal(np.asarray(a).view(np.uint32), np.asarray(b).view(np.uint32))


@pytest.mark.parametrize("threads", [1, 3, 8])
def test_thread_count_does_not_change_cuts(threads):
    X, mb, w = CASES["integer_images"]
    base = P.sketch(X, mb, threads=1)
    got = P.sketch(X, mb, threads=threads)
    for a, b in zip(got, base):
        np.testing.assert_array_equal(np.asarray(a).view(np.uint32), np.asarray(b).view(np.uint32))


def test_invalid_max_bin_is_rejected():
    with pytest.raises(RuntimeError, match="max_bin"):
        P.sketch(np.zeros((4, 2), np.float32), 300)

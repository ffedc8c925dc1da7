"""Extreme gradient magnitudes (the reference's gradient-precision families,
tests/test_gradient_precision.py:12-27 there): labels spanning 60 orders of
magnitude, residuals that cancel to zero, subnormal residuals, subnormal
and huge feature values. Gradients, their exact power-of-two scales and
whole training runs against the oracle, bit for bit."""
import numpy as np
import pytest

import checkers as C
import product as P
from test_gpu_parity import assert_same_trees, bits

pytestmark = pytest.mark.gpu


def _labels(kind, n, rng):
    if kind == "wide_range":
        return (rng.normal(size=n) * 10.0 ** rng.integers(-30, 30, n)).astype(np.float32)
    if kind == "ten_orders":
        return (rng.normal(size=n) * 10.0 ** rng.integers(-5, 5, n)).astype(np.float32)
    if kind == "cancelling":
        y = np.full(n, 0.5, np.float32)
        y[::97] = 0.75
        return y
    if kind == "subnormal":
        return (rng.normal(size=n) * 1e-40).astype(np.float32)
    raise ValueError(kind)


@pytest.mark.parametrize("kind", ["wide_range", "ten_orders", "cancelling", "subnormal"])
def test_gradients_and_scales(kind):
    rng = np.random.default_rng(41)
    n = 40000
    labels = _labels(kind, n, rng)
    margins = np.full((n, 1), 0.5, np.float32)
    want = C.oracle_gradients("reg:squarederror", margins, labels)
    pairs, scales = P.gradients("reg:squarederror", margins, labels)
    np.testing.assert_array_equal(bits(pairs), bits(want))
    np.testing.assert_array_equal(bits(scales), bits(C.oracle().gradient_scales(want)))


@pytest.mark.parametrize("kind", ["wide_range", "ten_orders", "cancelling", "subnormal"])
def test_training(kind):
    rng = np.random.default_rng(42)
    n = 12000
    X = rng.normal(size=(n, 5)).astype(np.float32)
    X[:, 3] *= 1e-42  # subnormal feature values
    X[:, 4] *= 1e35   # huge feature values
    y = _labels(kind, n, rng)
    params = C.train_params(dict(max_depth=6, base_score=0.0 if kind == "subnormal" else 0.5))
    trees_o, margins_o, _ = C.oracle_train(X, y, params, 3)
    trees_p, margins_p = P.train(X, y, {k: v for k, v in params.items() if k != "num_class"}, 3)
    assert_same_trees(trees_p, trees_o)
    np.testing.assert_array_equal(bits(margins_p), bits(margins_o))

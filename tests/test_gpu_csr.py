"""Sparse matrices: the level histograms come from each row's present codes
(the reference's CSR histogram, kernels/histogram_csr.metal.h:22-152,
dispatched per level by src/tree.cpp:863-872): every present (feature, code)
adds the row's exact (g, h), and each built node's missing bin is its total
minus its present bins. The models must equal the oracle's bit for bit, and
the built histograms must equal orc_histogram word for word."""
import numpy as np
import pytest

import checkers as C
import product as P
from test_gpu_hist_words import _check_level, _oracle_q

pytestmark = pytest.mark.gpu


def _sparse(rows, cols, density, seed):
    """X with NaN where a CSR matrix has no entry, and the CSR matrix."""
    import scipy.sparse as sp
    rng = np.random.default_rng(seed)
    mask = rng.random((rows, cols)) < density
    r, c = np.nonzero(mask)
    vals = rng.normal(size=len(r)).astype(np.float32)
    tied = rng.random(len(r)) < 0.3
    vals[tied] = np.round(vals[tied] * 4) / 4  # repeated values
    X = np.full((rows, cols), np.nan, np.float32)
    X[r, c] = vals
    csr = sp.csr_matrix((vals, (r, c)), shape=(rows, cols), dtype=np.float32)
    w = rng.normal(size=cols)
    y = (np.nan_to_num(X) @ w + 0.1 * rng.normal(size=rows)).astype(np.float32)
    return X, csr, y


@pytest.mark.parametrize("depth,objective", [(6, "reg:squarederror"), (10, "binary:logistic")])
def test_csr_input_trains_the_oracles_model(depth, objective):
    import xgboost as xgb
    X, csr, y = _sparse(40000, 48, 0.08, seed=depth)
    if objective == "binary:logistic":
        y = (y > np.median(y)).astype(np.float32)
    assert csr.nnz < 0.1 * X.size
    params = C.train_params(dict(objective=objective, max_depth=depth, eta=0.3))
    _, margins_o, _ = C.oracle_train(X, y, params, 3)
    d = xgb.DMatrix(csr, label=y)
    bst = xgb.train({"objective": objective, "max_depth": depth, "eta": 0.3, "max_bin": 256,
                     "tree_method": "hist", "device": "cuda", "cuda_profile": 1}, d, 3)
    assert bst.cuda_profile()["csr"] is True
    np.testing.assert_array_equal(bst.predict(d, output_margin=True).view(np.uint32),
                                  margins_o[:, 0].view(np.uint32))


def test_csr_level_histogram_words_match_oracle():
    import xgboost as xgb
    X, csr, y = _sparse(30000, 37, 0.1, seed=5)
    o = C.oracle()
    cuts, counts, _ = o.sketch_cuts(X, 256)
    bins = o.quantize(X, cuts, counts)
    q = _oracle_q("reg:squarederror", y, None)
    d = xgb.DMatrix(csr, label=y)
    params = {"objective": "reg:squarederror", "max_depth": 8, "eta": 0.3, "max_bin": 256,
              "tree_method": "hist", "device": "cuda", "cuda_csr_hist": 1}
    for depth in (0, 1, 4, 7):
        _check_level(xgb, d, params, X, bins, q, cuts.shape[1], depth)


def test_dense_and_csr_histograms_train_the_same_model():
    """cuda_csr_hist=0 forces the dense kernels on the same sparse matrix."""
    X, _, y = _sparse(20000, 30, 0.15, seed=9)
    base = dict(objective="reg:squarederror", max_depth=7, eta=0.3, max_bin=64)
    trees_c, m_c = P.train(X, y, dict(base, cuda_csr_hist=1), 3)
    trees_d, m_d = P.train(X, y, dict(base, cuda_csr_hist=0), 3)
    np.testing.assert_array_equal(m_c.view(np.uint32), m_d.view(np.uint32))
    for a, b in zip(trees_c, trees_d):
        assert a.tobytes() == b.tobytes()

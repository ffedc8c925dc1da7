"""The c4 workload at its full size: 50M rows x 128 features, 256 bins plus a
missing bin (uint16 codes), 5 % NaN, binary:logistic, max_depth 10.

At this size the product runs the paths smaller tests cannot reach: the GPU
sketch of 6.4G values, 19-bit histogram limbs with a carry interval of 15
feature steps, row tiles in the tens of thousands per level, and the last
level's leaf additions in several row-id passes. The checks are the ones a
matrix this large allows against the oracle:

- the root histogram of every feature sums, over its 257 bins, to the total
  of the quantised gradients (exact int64);
- the root and the deepest built level (9) match `orc_histogram` word for
  word on features from every 32-feature group, over all 50M rows (the
  reference's histogram semantics, kernels/boost.metal:700-733,
  kernels/histogram_missing.metal.h:13-60);
- the margins training leaves behind (the row partition and the last
  level's passes) equal, bit for bit, the margins of the same tree walked
  row by row on a second matrix (src/learner.cpp:933-976 there: the leaf of
  each row is the one the tree's splits give).

Feature values are the integers 0..255, so the bins are the values
themselves for any row count.
"""
import numpy as np
import pytest

import checkers as C
import product as P
from test_gpu_hist_words import _node_of_rows, _oracle_q, _tree_arrays

pytestmark = pytest.mark.gpu

ROWS, COLS, NAN = 50_000_000, 128, 0.05
SEL = (0, 31, 32, 70, 101, 127)  # features from all four 32-feature groups
MISSING = 0xFFFFFFFF


def _data():
    """Host X (float32, NaN = missing), the bins of the SEL features and the
    labels, generated on the GPU in 4M-row chunks."""
    import torch
    X = np.empty((ROWS, COLS), np.float32)
    bins = np.empty((ROWS, len(SEL)), np.uint32)
    g = torch.Generator(device="cuda")
    g.manual_seed(4101)
    sel = torch.tensor(SEL, device="cuda")
    step = 1 << 22
    for i in range(0, ROWS, step):
        n = min(step, ROWS - i)
        c = torch.randint(0, 256, (n, COLS), generator=g, device="cuda", dtype=torch.int32)
        m = torch.rand((n, COLS), generator=g, device="cuda") < NAN
        torch.from_numpy(X[i:i + n]).copy_(c.float().masked_fill_(m, float("nan")))
        b = c.masked_fill_(m, -1).index_select(1, sel)
        torch.from_numpy(bins[i:i + n].view(np.int32)).copy_(b)
        del c, m, b
    y = (torch.rand(ROWS, generator=g, device="cuda") < 0.4).float().cpu().numpy()
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    return X, bins, y


@pytest.fixture(scope="module")
def c4_full():
    import psutil
    if psutil.virtual_memory().available < (64 << 30):
        pytest.skip("the full-size c4 matrix needs 64 GB of free host memory")
    import xgboost as xgb
    X, bins, y = _data()
    q = np.ascontiguousarray(_oracle_q("binary:logistic", y, None))
    dtrain = xgb.DMatrix(X, label=y)
    params = {"objective": "binary:logistic", "max_depth": 10, "eta": 0.1, "max_bin": 256,
              "tree_method": "hist", "device": "cuda"}
    return xgb, X, bins, q, dtrain, params


def _level(xgb, dtrain, params, depth):
    bst = xgb.Booster(params, [dtrain])
    P.capture_level_histograms(bst, depth)
    bst.update(dtrain, 0)
    meta, hist, node_ids = P.level_histograms(bst)
    assert meta["depth"] == depth and meta["bins1"] == 257
    assert (meta["f_lo"], meta["f_hi"]) == (0, COLS)
    assert meta["pairs"] == len(node_ids) >= 1
    return bst, hist, node_ids


def test_root_histogram_sums_and_words(c4_full):
    xgb, X, bins, q, dtrain, params = c4_full
    _, hist, node_ids = _level(xgb, dtrain, params, 0)
    assert list(node_ids) == [0]
    total = q.sum(axis=0)
    np.testing.assert_array_equal(hist[0].sum(axis=1), np.broadcast_to(total, (COLS, 2)))
    want = C.oracle_histogram(bins, q, np.arange(ROWS, dtype=np.uint32), 256)
    np.testing.assert_array_equal(hist[0][list(SEL)], want)


def test_last_level_words_and_training_margins(c4_full):
    xgb, X, bins, q, dtrain, params = c4_full
    bst, hist, node_ids = _level(xgb, dtrain, params, 9)
    tree = _tree_arrays(bst)
    node = _node_of_rows(X, tree, 9)
    order = np.argsort(node, kind="stable").astype(np.uint32)
    counts = np.bincount(node, minlength=len(tree[0]))
    starts = np.concatenate(([0], np.cumsum(counts)))
    parent = {int(c): p for p, (l, r) in enumerate(zip(tree[0], tree[1])) if l >= 0 for c in (l, r)}
    for p, nid in enumerate(node_ids):
        nid = int(nid)
        pl = int(tree[0][parent[nid]])
        sib = pl + 1 if nid == pl else pl
        # The smaller child of the pair is built; a tie builds the left one.
        assert counts[nid] < counts[sib] or (counts[nid] == counts[sib] and nid == pl), (p, nid)
        rows = order[starts[nid]:starts[nid + 1]]
        assert hist[p].sum(axis=1).tolist() == [q[rows].sum(axis=0).tolist()] * COLS, (p, nid)
        want = C.oracle_histogram(bins, q, rows, 256)
        np.testing.assert_array_equal(hist[p][list(SEL)], want, err_msg="pair %d node %d" % (p, nid))
    trained = bst.predict(dtrain, output_margin=True)
    walked = bst.predict(xgb.DMatrix(X), output_margin=True)
    assert trained.shape == walked.shape == (ROWS,)
    np.testing.assert_array_equal(trained.view(np.uint32), walked.view(np.uint32))

"""The c3 shape at its full size: 1M rows x 784 features, integer values
0..254 with 80 % exact zeros, 10 balanced classes, multi:softprob,
max_depth 6, max_bin 256. Each feature has 255 bins, so the codes are uint8
(255 bins plus the missing code); the cut stride stays max_bin, so the
built histograms have 257 bins, the missing one last.

784 features are 24.5 groups of 32, so the last histogram feature group is
half full, and every round grows 10 trees. The values are drawn so that each
feature takes every integer 0..254: the bins are the values themselves. At
1M rows the first round's quantised gradients are 44 bits wide, so the
staged three-limb histogram kernel builds these levels. The checks:

- class 0's root and its deepest built level (5) match `orc_histogram` word
  for word on features of the first, a middle and the half-full last feature
  group, over all 1M rows (kernels/boost.metal:700-733 and
  kernels/histogram_missing.metal.h:13-60 there), and every feature's bins
  sum to the node's total;
- the margins of all 10 classes that training leaves behind equal, bit for
  bit, those of the same trees walked on a second matrix.
"""
import numpy as np
import pytest

import checkers as C
import product as P
from test_gpu_hist_words import _node_of_rows, _oracle_q, _tree_arrays

pytestmark = pytest.mark.gpu

ROWS, COLS, CLASSES, ZEROS = 1_000_000, 784, 10, 0.8
NBINS = 255  # distinct values per feature
SEL = (0, 17, 31, 32, 400, 767, 768, 775, 783)


def _data():
    import torch
    X = np.empty((ROWS, COLS), np.float32)
    bins = np.empty((ROWS, len(SEL)), np.uint32)
    g = torch.Generator(device="cuda")
    g.manual_seed(3101)
    sel = torch.tensor(SEL, device="cuda")
    step = 1 << 18
    for i in range(0, ROWS, step):
        n = min(step, ROWS - i)
        c = torch.randint(1, NBINS, (n, COLS), generator=g, device="cuda", dtype=torch.int32)
        c.masked_fill_(torch.rand((n, COLS), generator=g, device="cuda") < ZEROS, 0)
        torch.from_numpy(X[i:i + n]).copy_(c.float())
        torch.from_numpy(bins[i:i + n].view(np.int32)).copy_(c.index_select(1, sel))
        del c
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    y = (np.arange(ROWS) % CLASSES)[np.random.default_rng(3102).permutation(ROWS)].astype(np.float32)
    return X, bins, y


@pytest.fixture(scope="module")
def c3_full():
    import xgboost as xgb
    X, bins, y = _data()
    q = np.ascontiguousarray(_oracle_q("multi:softprob", y, None, CLASSES))
    assert int(np.abs(q).max()).bit_length() > 42
    dtrain = xgb.DMatrix(X, label=y)
    params = {"objective": "multi:softprob", "num_class": CLASSES, "max_depth": 6, "eta": 0.3,
              "max_bin": 256, "tree_method": "hist", "device": "cuda"}
    return xgb, X, bins, q, dtrain, params


@pytest.mark.parametrize("depth", [0, 5])
def test_class0_level_words(c3_full, depth):
    xgb, X, bins, q, dtrain, params = c3_full
    bst = xgb.Booster(params, [dtrain])
    P.capture_level_histograms(bst, depth)
    bst.update(dtrain, 0)
    meta, hist, node_ids = P.level_histograms(bst)
    assert meta["depth"] == depth and meta["bins1"] == 257
    assert (meta["f_lo"], meta["f_hi"]) == (0, COLS)
    assert meta["pairs"] == len(node_ids) >= 1
    tree = _tree_arrays(bst)
    node = _node_of_rows(X, tree, depth)
    order = np.argsort(node, kind="stable").astype(np.uint32)
    counts = np.bincount(node, minlength=len(tree[0]))
    starts = np.concatenate(([0], np.cumsum(counts)))
    parent = {int(c): p for p, (l, r) in enumerate(zip(tree[0], tree[1])) if l >= 0 for c in (l, r)}
    for p, nid in enumerate(node_ids):
        nid = int(nid)
        if depth:
            pl = int(tree[0][parent[nid]])
            sib = pl + 1 if nid == pl else pl
            # The smaller child of the pair is built; a tie builds the left one.
            assert counts[nid] < counts[sib] or (counts[nid] == counts[sib] and nid == pl), (p, nid)
        rows = order[starts[nid]:starts[nid + 1]]
        assert hist[p].sum(axis=1).tolist() == [q[rows].sum(axis=0).tolist()] * COLS, (p, nid)
        want = C.oracle_histogram(bins, q, rows, 256)
        np.testing.assert_array_equal(hist[p][list(SEL)], want, err_msg="pair %d node %d" % (p, nid))


def test_training_margins_equal_a_walk_of_the_trees(c3_full):
    xgb, X, bins, q, dtrain, params = c3_full
    bst = xgb.train(params, dtrain, 2)
    trained = bst.predict(dtrain, output_margin=True)
    walked = bst.predict(xgb.DMatrix(X), output_margin=True)
    assert trained.shape == walked.shape == (ROWS, CLASSES)
    np.testing.assert_array_equal(trained.view(np.uint32), walked.view(np.uint32))

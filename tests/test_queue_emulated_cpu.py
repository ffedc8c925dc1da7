"""Host-driven trees with the GPU backend's block functions
(csrc/queue_par.h: node histograms dense or from sparse rows, row
partitions, the margin walk) run on
the CPU by the serial executor (csrc/exec.h HostExec), split evaluation by
the oracle: every histogram equals the oracle's for the same rows, and the
trees and margins equal the oracle's host-driven grower. Covers uint8 and
uint16 codes, all three missing-code conventions, segments longer than one
histogram tile (2048 rows) and one partition tile (1024 rows)."""
import ctypes
import os
import subprocess

import numpy as np
import pytest

import checkers as C
import product as P

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CSRC = os.path.join(ROOT, "xgboost-metal_b200", "csrc")
ORACLE = os.path.join(ROOT, "oracle")
BASE = dict(eta=0.3, reg_lambda=1.0, reg_alpha=0.0, min_child_weight=1.0, max_delta_step=0.0,
            min_split_loss=0.0)


@pytest.fixture(scope="module")
def harness(tmp_path_factory):
    C.build()
    out = str(tmp_path_factory.mktemp("queue") / "libqueue_harness.so")
    cuda_inc = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "include")
    subprocess.run(["g++", "-std=c++20", "-O2", "-fPIC", "-shared", "-ffp-contract=off", "-Wall",
                    "-I", CSRC, "-I", ORACLE, "-I", cuda_inc,
                    os.path.join(ROOT, "tests", "native", "queue_harness.cpp"), os.path.join(CSRC, "grower.cpp"),
                    "-L", ORACLE, "-loracle", "-Wl,-rpath," + ORACLE, "-o", out], check=True)
    lib = ctypes.CDLL(out)
    lib.queue_harness.restype = ctypes.c_int
    return lib


def _inputs(seed, rows=6000, cols=6, max_bin=32, nan=0.1):
    o = C.oracle()
    rng = np.random.default_rng(seed)
    X = rng.normal(size=(rows, cols)).astype(np.float32)
    X[rng.random(X.shape) < nan] = np.nan
    cuts, counts, minima = o.sketch_cuts(X, max_bin)
    bins = o.quantize(X, cuts, counts)
    y = np.nan_to_num(X[:, 0]) * 2 - np.nan_to_num(X[:, 2 % cols]) + np.sin(np.nan_to_num(X[:, 1 % cols]) * 3)
    pairs = np.stack([(0.5 - y + 0.3 * rng.normal(size=rows)), 0.5 + rng.random(rows)], 1).astype(np.float32)
    scale = o.gradient_scales(pairs[:, None, :])[0]
    q = o.quantize_gradients(pairs[:, None, :], scale[None])[:, 0, :]
    return bins, q, pairs, scale, cuts, counts, minima


def _run(lib, inputs, params, lossguide=False, max_leaves=0, wide=False, sparse=False):
    bins, q, pairs, scale, cuts, counts, minima = inputs
    rows, cols = bins.shape
    cap = 2 * rows + 1
    nodes = np.zeros(cap, P.DEVNODE_DTYPE)
    margins = np.zeros(rows, np.float32)
    stats = np.zeros(2, np.uint64)
    tp = C._TreeParams(params["max_depth"], params["eta"], params["reg_lambda"], params["reg_alpha"],
                       params["min_child_weight"], params["max_delta_step"], params["min_split_loss"])
    p = lambda a: a.ctypes.data_as(ctypes.c_void_p)  # noqa: E731
    u32 = ctypes.c_uint32
    bins = np.ascontiguousarray(bins, np.uint32)
    q = np.ascontiguousarray(q, np.int64)
    pairs = np.ascontiguousarray(pairs, np.float32)
    scale = np.ascontiguousarray(scale, np.float32)
    n = lib.queue_harness(p(bins), u32(rows), u32(cols), p(q), p(pairs), p(scale), p(cuts), u32(cuts.shape[1]),
                          p(counts), p(minima), ctypes.byref(tp), u32(int(lossguide)), u32(max_leaves),
                          ctypes.c_int(int(wide)), ctypes.c_int(int(sparse)), ctypes.c_float(0.25), p(nodes),
                          u32(cap), p(margins), p(stats))
    assert n > 0, n
    return nodes[:n], margins, stats


def _check(lib, inputs, params, lossguide=False, max_leaves=0, wide=False, sparse=False):
    bins, q, pairs, scale, cuts, counts, minima = inputs
    want, leaf = C.grow_tree_queue(bins, q, scale, cuts, counts, minima, params, lossguide=lossguide,
                                   max_leaves=max_leaves)
    got, margins, stats = _run(lib, inputs, params, lossguide, max_leaves, wide, sparse)
    assert stats[0] == 0 and stats[1] > 0, stats
    assert len(got) == len(want)
    for f in ("left", "right", "feature", "parent"):
        np.testing.assert_array_equal(got[f], want[f], err_msg=f)
    for f in ("leaf", "cover"):
        np.testing.assert_array_equal(got[f].view(np.uint32), want[f].view(np.uint32), err_msg=f)
    split = want["left"] >= 0
    np.testing.assert_array_equal(got["split_bin"][split], want["split_bin"][split])
    np.testing.assert_array_equal(margins.view(np.uint32), (np.float32(0.25) + leaf).view(np.uint32))
    return got


@pytest.mark.parametrize("wide", [False, True])
def test_depthwise_deep(harness, wide):
    _check(harness, _inputs(1), dict(BASE, max_depth=13, min_child_weight=0.0), wide=wide)


@pytest.mark.parametrize("max_leaves", [0, 9, 40])
def test_lossguide(harness, max_leaves):
    _check(harness, _inputs(2, rows=9000), dict(BASE, max_depth=0 if max_leaves else 12), lossguide=True,
           max_leaves=max_leaves)


def test_missing_code_conventions(harness):
    # 256 cuts with missing values (uint8, missing code 255 needs <= 255
    # bins, so uint16 here), 256 cuts without missing values (uint8, code
    # 0x100 unused) and fewer cuts (missing code = cut stride).
    rng = np.random.default_rng(3)
    for nan in (0.2, 0.0):
        inputs = _inputs(4, rows=8000, cols=4, max_bin=256, nan=nan)
        assert inputs[5].max() == 256
        _check(harness, inputs, dict(BASE, max_depth=7))
    inputs = _inputs(5, rows=5000, cols=3, max_bin=255, nan=0.3)
    _check(harness, inputs, dict(BASE, max_depth=0), lossguide=True, max_leaves=30)
    del rng


def test_wide_batches_and_regularisation(harness):
    inputs = _inputs(6, rows=30000, cols=5, max_bin=64, nan=0.02)
    _check(harness, inputs, dict(BASE, max_depth=11, min_child_weight=0.0, reg_alpha=0.3, max_delta_step=0.5))


@pytest.mark.parametrize("wide", [False, True])
def test_sparse_row_histograms(harness, wide):
    # Mostly missing values: each node histogram from the rows' present codes
    # and its missing bin from the node total.
    inputs = _inputs(7, rows=12000, cols=20, max_bin=64, nan=0.9)
    _check(harness, inputs, dict(BASE, max_depth=9), sparse=True, wide=wide)
    _check(harness, inputs, dict(BASE, max_depth=0), lossguide=True, max_leaves=25, sparse=True, wide=wide)


def test_sparse_rows_without_missing_values(harness):
    # Every code present (uint8 with 256 bins and no missing value).
    inputs = _inputs(8, rows=6000, cols=3, max_bin=256, nan=0.0)
    _check(harness, inputs, dict(BASE, max_depth=12), sparse=True)


def _inputs_from(X, pairs, max_bin):
    o = C.oracle()
    cuts, counts, minima = o.sketch_cuts(X, max_bin)
    bins = o.quantize(X, cuts, counts)
    pairs = np.ascontiguousarray(pairs, np.float32)
    scale = o.gradient_scales(pairs[:, None, :])[0]
    q = o.quantize_gradients(pairs[:, None, :], scale[None])[:, 0, :]
    return bins, q, pairs, scale, cuts, counts, minima


@pytest.mark.parametrize("max_bin", [2, 33, 256])
@pytest.mark.parametrize("lossguide", [False, True])
def test_reference_split_scan_family(harness, max_bin, lossguide):
    """The split-scan family of the reference's tests
    (tests/test_split_scan.py:8-31 of the reference): values on a 1/64 grid,
    feature 1 a copy of feature 0, missing values in three features, the
    caller's gradients in quarters and hessians of 1.25 or -0.5, alpha 0.17,
    lambda 0.4, max_delta_step 1, min_child_weight 0.5; depth 4, or
    loss-guided with at most 15 leaves."""
    rng = np.random.default_rng(833)
    X = rng.integers(-200, 201, (1025, 7)).astype(np.float32) / 64
    X[:, 1] = X[:, 0]
    X[::11, 2] = np.nan
    X[::13, 4] = np.nan
    X[::17, 6] = np.nan
    row = np.arange(len(X))
    pairs = np.stack([(row % 7 - 3) / 4, np.where(row % 5, 1.25, -0.5)], 1)
    params = dict(BASE, eta=0.2, reg_lambda=0.4, reg_alpha=0.17, min_child_weight=0.5, max_delta_step=1.0,
                  max_depth=0 if lossguide else 4)
    got = _check(harness, _inputs_from(X, pairs, max_bin), params, lossguide=lossguide,
                 max_leaves=15 if lossguide else 0)
    assert len(got) > 3
    assert not (got["feature"] == 1).any()  # ties with feature 0 go to the smaller feature


@pytest.mark.parametrize("sparse", [False, True])
@pytest.mark.parametrize("lossguide", [False, True])
def test_reference_missing_family(harness, sparse, lossguide):
    """The missing-value family of the reference's tests
    (tests/test_histogram_missing.py:11-20 of the reference): about 95 % of
    the cells missing, explicit zeros in feature 0, every 29th row and the
    last feature entirely missing; node histograms dense or from the rows'
    present codes."""
    rng = np.random.default_rng(7315)
    X = rng.normal(size=(2049, 7)).astype(np.float32)
    y = X[:, 0] - X[:, 1] * X[:, 2] + X[:, 3] ** 2
    X[rng.random(X.shape) >= 0.05] = np.nan
    X[1::17, 0] = 0.0
    X[::29] = np.nan
    X[:, -1] = np.nan
    pairs = np.stack([-y, np.ones(len(y))], 1)
    params = dict(BASE, max_depth=0 if lossguide else 4)
    got = _check(harness, _inputs_from(X, pairs, 16), params, lossguide=lossguide,
                 max_leaves=12 if lossguide else 0, sparse=sparse)
    assert len(got) > 3

"""The product's host-driven grower (csrc/grower.cpp: the reference's
fallback driver for loss-guided trees, leaf budgets and depths beyond ten,
src/tree.cpp:291-349, 1031-1120) checked on the CPU: a test harness drives it
with a backend that evaluates and partitions through the oracle, and the node
tables must equal the oracle's own host-driven grower field for field. The
GPU backend (csrc/queue.cu) is checked against the oracle in
test_zzzz_queue_gpu.py."""
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


@pytest.fixture(scope="module")
def harness(tmp_path_factory):
    C.build()
    out = str(tmp_path_factory.mktemp("grower") / "libgrower_harness.so")
    cuda_inc = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "include")
    subprocess.run(["g++", "-std=c++20", "-O2", "-fPIC", "-shared", "-ffp-contract=off", "-Wall",
                    "-I", CSRC, "-I", ORACLE, "-I", cuda_inc,
                    os.path.join(ROOT, "tests", "native", "grower_harness.cpp"), os.path.join(CSRC, "grower.cpp"),
                    "-L", ORACLE, "-loracle", "-Wl,-rpath," + ORACLE, "-o", out], check=True)
    lib = ctypes.CDLL(out)
    lib.grower_harness.restype = ctypes.c_int
    return lib


BASE = dict(eta=0.3, reg_lambda=1.0, reg_alpha=0.0, min_child_weight=1.0, max_delta_step=0.0,
            min_split_loss=0.0)


def _inputs(seed, rows=3000, cols=6, max_bin=32, nan=0.1):
    o = C.oracle()
    rng = np.random.default_rng(seed)
    X = rng.normal(size=(rows, cols)).astype(np.float32)
    X[rng.random(X.shape) < nan] = np.nan
    cuts, counts, minima = o.sketch_cuts(X, max_bin)
    bins = o.quantize(X, cuts, counts)
    y = np.nan_to_num(X[:, 0]) * 2 - np.nan_to_num(X[:, 2]) + np.sin(np.nan_to_num(X[:, 1]) * 3)
    pairs = np.stack([(0.5 - y + 0.3 * rng.normal(size=rows)), np.ones(rows)], 1).astype(np.float32)[:, None, :]
    scale = o.gradient_scales(pairs)[0]
    q = o.quantize_gradients(pairs, scale[None])[:, 0, :]
    return bins, q, scale, cuts, counts, minima


def _grow(lib, inputs, params, lossguide=False, max_leaves=0):
    bins, q, scale, cuts, counts, minima = inputs
    rows, cols = bins.shape
    cap = 2 * rows + 1
    nodes = np.zeros(cap, P.DEVNODE_DTYPE)
    tp = C._TreeParams(params["max_depth"], params["eta"], params["reg_lambda"], params["reg_alpha"],
                       params["min_child_weight"], params["max_delta_step"], params["min_split_loss"])
    u32 = ctypes.c_uint32
    ptr = lambda a: a.ctypes.data_as(ctypes.c_void_p)  # noqa: E731
    bins = np.ascontiguousarray(bins, np.uint32)
    q = np.ascontiguousarray(q, np.int64)
    scale = np.ascontiguousarray(scale, np.float32)
    n = lib.grower_harness(ptr(bins), u32(rows), u32(cols), ptr(q), ptr(scale), ptr(cuts), u32(cuts.shape[1]),
                           ptr(counts), ptr(minima), ctypes.byref(tp), u32(int(lossguide)), u32(max_leaves),
                           ptr(nodes), u32(cap))
    assert n > 0, n
    return nodes[:n]


def _assert_same(got, want):
    assert len(got) == len(want)
    for f in ("left", "right", "feature", "parent"):
        np.testing.assert_array_equal(got[f], want[f], err_msg=f)
    for f in ("leaf", "cover"):
        np.testing.assert_array_equal(got[f].view(np.uint32), want[f].view(np.uint32), err_msg=f)
    split = want["left"] >= 0
    for f in ("threshold", "gain"):
        np.testing.assert_array_equal(got[f][split].view(np.uint32), want[f][split].view(np.uint32), err_msg=f)
    for f in ("default_left", "split_bin"):
        np.testing.assert_array_equal(got[f][split], want[f][split], err_msg=f)
    # Leaves carry the device driver's conventions.
    assert np.all(got["split_bin"][~split] == -1)
    assert np.all(got["flags"][split] & 2)


def _check(lib, inputs, params, lossguide=False, max_leaves=0):
    want, _ = C.grow_tree_queue(*inputs, params, lossguide=lossguide, max_leaves=max_leaves)
    got = _grow(lib, inputs, params, lossguide, max_leaves)
    _assert_same(got, want)
    return got


@pytest.mark.parametrize("seed,max_depth", [(1, 1), (2, 4), (3, 8), (4, 14)])
def test_depthwise(harness, seed, max_depth):
    _check(harness, _inputs(seed), dict(BASE, max_depth=max_depth, min_child_weight=0.0))


@pytest.mark.parametrize("max_depth", [0, 3, 7])
def test_lossguide(harness, max_depth):
    params = dict(BASE, max_depth=max_depth or 20)
    # max_depth 0 is unlimited; the oracle's depth limit of 20 never binds here.
    _check(harness, _inputs(7, rows=2000), dict(params, max_depth=max_depth), lossguide=True)


@pytest.mark.parametrize("lossguide", [False, True])
@pytest.mark.parametrize("max_leaves", [2, 5, 17, 64])
def test_leaf_budget(harness, lossguide, max_leaves):
    nodes = _check(harness, _inputs(9), dict(BASE, max_depth=0 if lossguide else 9), lossguide, max_leaves)
    assert int(np.sum(nodes["left"] < 0)) <= max_leaves


def test_levels_wider_than_one_batch(harness):
    # More than 256 expanding leaves at one depth: the depth-wise queue pops
    # them in several batches of 256, which number the next level's nodes in
    # batch order.
    inputs = _inputs(12, rows=40000, cols=5, max_bin=128, nan=0.02)
    nodes = _check(harness, inputs, dict(BASE, max_depth=12, min_child_weight=0.0))
    depth = np.zeros(len(nodes), int)
    for i, n in enumerate(nodes):
        if n["left"] >= 0:
            depth[n["left"]] = depth[n["right"]] = depth[i] + 1
    assert max(np.sum((depth == d) & (nodes["left"] >= 0)) for d in range(13)) > 256


def test_regularised_applied_statistics(harness):
    # alpha, max_delta_step and min_split_loss change the applied parent
    # weights the grower derives from the child sums.
    params = dict(BASE, max_depth=7, reg_alpha=0.7, reg_lambda=2.5, max_delta_step=0.3, min_split_loss=0.05,
                  min_child_weight=3.0)
    nodes = _check(harness, _inputs(13), params)
    split = nodes["left"] >= 0
    assert np.any(np.abs(nodes["base_weight"][split]) == np.float32(0.3))
    _check(harness, _inputs(14), dict(params, max_depth=0), lossguide=True, max_leaves=40)


def test_single_row_and_constant_inputs(harness):
    inputs = _inputs(15, rows=1, cols=3)
    nodes = _check(harness, inputs, dict(BASE, max_depth=12))
    assert len(nodes) == 1
    bins, q, scale, cuts, counts, minima = _inputs(16, rows=500, cols=3)
    bins[:] = bins[0]
    nodes = _check(harness, (bins, q, scale, cuts, counts, minima), dict(BASE, max_depth=0), lossguide=True)
    assert len(nodes) == 1


def test_growth_parameters_are_validated_without_a_gpu():
    # The reference's limits (src/learner.cpp:247, 258-260); settings outside
    # the level-synchronous driver select host-driven growth.
    import json

    import xgboost as xgb
    for ok in (dict(grow_policy="lossguide", max_depth=0, max_leaves=8), dict(max_depth=25),
               dict(max_depth=40, max_leaves=10), dict(max_depth=6, max_leaves=4)):
        cfg = json.loads(xgb.Booster(ok).save_config())
        train = cfg["learner"]["gradient_booster"]["tree_train_param"]
        assert train["max_depth"] == str(ok["max_depth"])
    for bad, msg in ((dict(grow_policy="levelwise"), "grow_policy must be depthwise or lossguide"),
                     (dict(max_depth=0), "cannot both be unconstrained"),
                     (dict(max_depth=31), "must not exceed 30"),
                     (dict(max_leaves=2 ** 31), "node index range")):
        with pytest.raises(xgb.XGBoostError, match=msg):
            xgb.Booster(bad).save_config()

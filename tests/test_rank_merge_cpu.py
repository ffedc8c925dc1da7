"""The split a row-sharded job picks for each node: every rank evaluates only
its feature range (the feature count padded to a multiple of the ranks, some
ranks with few or no real features) and the ranks' best keys are merged.
The product's key, range and merge functions (csrc/split_select.h) run here
on the CPU and must pick, for every node and every rank count, the split the
oracle's serial selection picks (largest gain, smallest feature on ties;
the reference's select_splits, kernels/boost.metal:1245-1302)."""
import ctypes
import os
import subprocess

import numpy as np
import pytest

import checkers as C

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CSRC = os.path.join(ROOT, "xgboost-metal_b200", "csrc")


@pytest.fixture(scope="module")
def harness(tmp_path_factory):
    out = str(tmp_path_factory.mktemp("merge") / "librank_merge.so")
    subprocess.run(["g++", "-std=c++20", "-O2", "-fPIC", "-shared", "-Wall", "-I", CSRC,
                    os.path.join(ROOT, "tests", "native", "rank_merge_harness.cpp"), "-o", out], check=True)
    lib = ctypes.CDLL(out)
    lib.rank_merge.restype = ctypes.c_int
    return lib


def _merge(lib, gains, world):
    gains = np.ascontiguousarray(gains, np.float32)
    nodes, cols = gains.shape
    feature = np.zeros(nodes, np.int32)
    gain = np.zeros(nodes, np.float32)
    p = lambda a: a.ctypes.data_as(ctypes.c_void_p)  # noqa: E731
    assert lib.rank_merge(p(gains), ctypes.c_uint32(nodes), ctypes.c_uint32(cols), ctypes.c_uint32(world),
                          p(feature), p(gain)) == 0
    return feature, gain


def _oracle_level(cols, seed, dup):
    """Split candidates of 8 nodes from real histograms: random rows per node,
    quantised gradients, the oracle's evaluation; `dup` copies columns so
    that equal gains sit in different ranks."""
    rng = np.random.default_rng(seed)
    rows = 4000
    base = rng.normal(size=(rows, cols)).astype(np.float32)
    for a, b in dup:
        base[:, b] = base[:, a]
    base[rng.random(base.shape) < 0.1] = np.nan
    o = C.oracle()
    cuts, counts, minima = o.sketch_cuts(base, 32)
    bins = o.quantize(base, cuts, counts)
    y = (np.nan_to_num(base) @ rng.normal(size=cols) + rng.normal(size=rows)).astype(np.float32)
    pairs = np.stack([-y, np.ones(rows, np.float32)], 1)[:, None, :]
    scale = o.gradient_scales(pairs)[0]
    q = o.quantize_gradients(pairs, scale[None])[:, 0, :]
    stride = cuts.shape[1]
    hists, sums = [], []
    for n in range(8):
        sel = np.sort(rng.choice(rows, size=rng.integers(50, 1500), replace=False)).astype(np.uint32)
        hists.append(C.oracle_histogram(bins, q, sel, stride))
        sums.append(q[sel].sum(axis=0))
    hist = np.stack(hists)
    params = dict(reg_lambda=1.0, reg_alpha=0.0, min_child_weight=1.0, max_delta_step=0.0)
    cand = o.evaluate_splits(hist, scale, cuts, counts, minima, params, 1, np.stack(sums).astype(np.int64))
    best = o.select_splits(cand, scale, params)
    return cand["gain"], best


@pytest.mark.parametrize("cols,dup", [(13, [(0, 12), (3, 7)]), (8, [(1, 6)]), (5, []), (33, [(2, 30), (2, 17)])])
def test_ranks_pick_the_oracles_split(harness, cols, dup):
    gains, best = _oracle_level(cols, seed=cols, dup=dup)
    for world in range(1, 9):
        feature, gain = _merge(harness, gains, world)
        for n in range(len(best)):
            if best["feature"][n] >= 0:
                assert feature[n] == best["feature"][n], (world, n)
                assert gain[n].view(np.uint32) == best["gain"][n].view(np.uint32), (world, n)
            else:
                assert feature[n] == -1 or not np.isfinite(gain[n]), (world, n)


def test_ties_go_to_the_smallest_feature_across_ranks(harness):
    """Equal gains in different ranks, -0 against +0, and every candidate
    invalid (-inf) on some nodes."""
    gains = np.array([[1.0, 2.0, 2.0, 0.5, 2.0],
                      [-0.0, 0.0, -1.0, -0.0, -2.0],
                      [-np.inf] * 5,
                      [3.0, -np.inf, 3.0, 3.0, 2.9999998]], np.float32)
    for world in range(1, 9):
        feature, _ = _merge(harness, gains, world)
        assert list(feature[[0, 1, 3]]) == [1, 0, 0], world
        assert feature[2] == 0, world

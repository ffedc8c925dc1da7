"""The GPU sketch's data-parallel algorithms (csrc/sketch_par.h: run
extraction chunk by chunk, batch summaries by bitonic sort and exact prefix
sums, prune and combine by binary search and running maxima) run on the CPU
through a test harness with the serial executor, and compared bit for bit
with the host sketch (which the oracle pins). The CUDA kernels run the same
functions with one thread block per task (test_zzzz_sketch_gpu.py)."""
import ctypes
import os
import subprocess

import numpy as np
import pytest

import product as P

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CSRC = os.path.join(ROOT, "xgboost-metal_b200", "csrc")


@pytest.fixture(scope="module")
def harness(tmp_path_factory):
    out = str(tmp_path_factory.mktemp("sketch") / "libsketch_harness.so")
    subprocess.run(["g++", "-std=c++20", "-O2", "-fPIC", "-shared", "-ffp-contract=off", "-Wall", "-I", CSRC,
                    os.path.join(ROOT, "tests", "native", "sketch_harness.cpp"), "-o", out], check=True)
    lib = ctypes.CDLL(out)
    lib.sketch_harness.restype = ctypes.c_int
    return lib


def _parallel(lib, X, max_bin, weights=None, chunk=64, segments=1, tree=0):
    X = np.ascontiguousarray(X, np.float32)
    rows, cols = X.shape
    stride = max(1, min(max_bin, rows))
    cuts = np.zeros((cols, stride), np.float32)
    counts = np.zeros(cols, np.uint32)
    minima = np.zeros(cols, np.float32)
    w = None if weights is None else np.ascontiguousarray(weights, np.float32)
    p = lambda a: None if a is None else a.ctypes.data_as(ctypes.c_void_p)  # noqa: E731
    u32 = ctypes.c_uint32
    serial = np.zeros(5, np.uint64)
    assert lib.sketch_harness(p(X), u32(rows), u32(cols), p(w), u32(max_bin), u32(chunk), u32(segments), u32(tree),
                              p(cuts), p(counts), p(minima), p(serial)) == 0
    return cuts, counts, minima, serial


# (segments, tree): the single pass with the level-by-level reduction, and the
# GPU's forms: rows in segments linked afterwards, and the merge tree.
MODES = [(1, 0), (3, 1), (7, 1)]


def _same(lib, X, max_bin, weights=None, chunk=64, serial_prefix=False):
    want = P.sketch(X, max_bin, weights)
    for segments, tree in MODES:
        got = _parallel(lib, X, max_bin, weights, chunk, segments, tree)
        msg = "segments %d tree %d" % (segments, tree)
        np.testing.assert_array_equal(got[1], want[1], err_msg=msg)
        np.testing.assert_array_equal(got[0].view(np.uint32), want[0].view(np.uint32), err_msg=msg)
        np.testing.assert_array_equal(got[2].view(np.uint32), want[2].view(np.uint32), err_msg=msg)
        # The data-parallel prune and combine ran throughout; batch prefix sums
        # are serial only for non-integer weights.
        assert got[3][0] == 0 and got[3][1] == 0, (msg, got[3])
        assert (got[3][2] > 0) == serial_prefix, (msg, got[3])
    return want


@pytest.mark.parametrize("max_bin", [2, 16, 64, 256])
@pytest.mark.parametrize("chunk", [7, 1024])
def test_continuous_values_with_missing(harness, max_bin, chunk):
    rng = np.random.default_rng(max_bin + chunk)
    X = rng.normal(size=(6000, 5)).astype(np.float32)
    X[rng.random(X.shape) < 0.1] = np.nan
    _same(harness, X, max_bin, chunk=chunk)


def test_many_batches_and_levels(harness):
    # A small budget makes hundreds of batches per feature, so the level
    # reduction carries through many levels.
    rng = np.random.default_rng(1)
    X = rng.normal(size=(120000, 2)).astype(np.float32)
    X[:, 1] = np.round(X[:, 1] * 40) / 40  # ties between batches
    _, counts, _ = _same(harness, X, 4, chunk=4096)
    assert counts.max() <= 4


def test_runs_ties_constants_and_signed_zeros(harness):
    rng = np.random.default_rng(2)
    n = 20000
    X = np.zeros((n, 6), np.float32)
    X[:, 0] = np.sort(rng.integers(0, 30, n))            # long runs in row order
    X[:, 1] = 3.0                                          # one run
    X[:, 2] = rng.integers(0, 3, n)                        # short runs, few values
    X[:, 3] = np.where(rng.random(n) < 0.5, 0.0, -0.0)     # -0 reads as +0
    X[:, 4] = np.nan                                       # empty feature
    X[:, 5] = rng.normal(size=n)
    X[rng.random(n) < 0.3, 5] = np.nan                     # runs spanning missing rows
    for chunk in (5, 256):
        _same(harness, X, 32, chunk=chunk)
        _same(harness, X, 256, chunk=chunk)


def test_weights(harness):
    rng = np.random.default_rng(3)
    n = 15000
    X = rng.normal(size=(n, 3)).astype(np.float32)
    X[:, 1] = np.sort(rng.integers(0, 100, n)).astype(np.float32)
    X[rng.random(X.shape) < 0.05] = np.nan
    w = rng.random(n).astype(np.float32) * 3
    w[::7] = 0.0
    for max_bin in (8, 64, 256):
        _same(harness, X, max_bin, weights=w, chunk=100, serial_prefix=True)
    # Integer weights: the batch prefix sums take the exact integer path.
    wi = rng.integers(0, 4, n).astype(np.float32)
    _same(harness, X, 64, weights=wi, chunk=1000)


def test_few_rows(harness):
    rng = np.random.default_rng(4)
    for rows in (1, 2, 3, 17):
        X = rng.normal(size=(rows, 3)).astype(np.float32)
        X[0, 0] = np.nan
        _same(harness, X, 256, chunk=2)


def test_merge_tree_takes_distinct_values_and_hands_ties_to_the_serial_reduction(harness):
    """Continuous features over many batches reduce through the merge tree
    (every merge of two summaries overflows the limit); a feature with few
    distinct values does not, and takes the level-by-level reduction. Both
    give the host sketch's cuts."""
    rng = np.random.default_rng(5)
    X = rng.normal(size=(60000, 3)).astype(np.float32)
    X[:, 2] = rng.integers(0, 20, 60000)
    X[rng.random(X.shape) < 0.05] = np.nan
    want = P.sketch(X, 8)
    got = _parallel(harness, X, 8, chunk=512, segments=5, tree=1)
    np.testing.assert_array_equal(got[1], want[1])
    np.testing.assert_array_equal(got[0].view(np.uint32), want[0].view(np.uint32))
    assert got[3][3] == 2 and got[3][4] == 1, got[3]


def test_segments_link_runs_spanning_many_segments(harness):
    """A run that spans whole segments, with unit and with float weights (the
    weighted continuation is summed row by row as the single pass does)."""
    rng = np.random.default_rng(6)
    n = 9000
    X = np.zeros((n, 3), np.float32)
    X[:, 0] = np.repeat(rng.normal(size=9), 1000)      # runs of 1000 rows
    X[:, 1] = np.where(np.arange(n) < 7000, 1.5, 2.5)  # one run over most segments
    X[:, 2] = rng.normal(size=n)
    X[rng.random(n) < 0.2, 1] = np.nan                 # the long run skips missing rows
    w = (rng.random(n) * 2).astype(np.float32)
    for weights in (None, w):
        want = P.sketch(X, 16, weights)
        for segments in (2, 9, 40):
            got = _parallel(harness, X, 16, weights, chunk=128, segments=segments, tree=1)
            np.testing.assert_array_equal(got[1], want[1])
            np.testing.assert_array_equal(got[0].view(np.uint32), want[0].view(np.uint32))


@pytest.mark.skipif(not __import__("checkers").have_reference(), reason="reference harness not built")
@pytest.mark.parametrize("family", range(18))
def test_reference_cut_families_against_the_reference_kernels(harness, family):
    """The weight and value families of the reference's own cut tests
    (tests/test_quantiles.py:9-20 of the reference; restated in
    test_oracle_pin_sketch.py) through the GPU sketch's data-parallel
    functions, in every mode the kernels use, against the reference's own
    sketch kernels compiled for the host: cuts, counts and minima bit for
    bit."""
    import checkers as C
    import test_oracle_pin_sketch as F
    rows, bins, kind = F.FAMILIES[family]
    X, w = F._family(rows, kind)
    weights = None if kind == "unit" else w
    want = C.reference().sketch_cuts(X, bins, weights)
    for segments, tree in MODES:
        got = _parallel(harness, X, bins, weights, 1024, segments, tree)
        msg = "%s: segments %d tree %d" % (kind, segments, tree)
        np.testing.assert_array_equal(got[1], want[1], err_msg=msg)
        np.testing.assert_array_equal(got[0].view(np.uint32), want[0].view(np.uint32), err_msg=msg)
        np.testing.assert_array_equal(got[2].view(np.uint32), want[2].view(np.uint32), err_msg=msg)

"""Pins the oracle against the reference's own serial kernel functions
(oracle/_ref, compiled for the host from the reference checkout) at the
widths the GPU parity tests run the CUDA path at: c4's 128 features with
5 % missing values and 256 bins, grown to depth 10, and c3's 784 features of
integer pixel values, about 80 % zeros, 10 classes at depth 6. The GPU tests
compare the CUDA path with the oracle at these widths (test_gpu_hist_words,
test_zzzz_full_size_gpu, test_zzzz_c3_full_size_gpu); these tests compare
the oracle with the reference there, so the chain reaches the reference at
the benchmark's own shapes. Cuts, bins, gradient scales, quantised
gradients, node tables and leaf values must be equal bit for bit over two
boosting rounds."""
import numpy as np
import pytest

import checkers as C

pytestmark = pytest.mark.skipif(not C.have_reference(),
                                reason="reference harness not built (no reference checkout)")


def _bits(a):
    return np.ascontiguousarray(a).view(np.uint32 if a.dtype == np.float32 else a.dtype)


def _tree_params(max_depth, eta):
    return dict(max_depth=max_depth, eta=eta, reg_lambda=1.0, reg_alpha=0.0, min_child_weight=1.0,
                max_delta_step=0.0, min_split_loss=0.0)


def _same_cuts(X, max_bin):
    o, r = C.oracle(), C.reference()
    co, cr = o.sketch_cuts(X, max_bin), r.sketch_cuts(X, max_bin)
    for a, b in zip(co, cr):
        np.testing.assert_array_equal(_bits(a), _bits(b))
    bins = o.quantize(X, co[0], co[1])
    np.testing.assert_array_equal(bins, r.quantize(X, cr[0], cr[1]))
    return co, bins


def _boost(objective, bins, cuts, y, groups, tp, rounds):
    """`rounds` rounds of one tree per output group. The oracle's gradient
    pairs feed both growers (the reference's own gradients kernel takes the
    host libm's exp, which may differ from the oracle's by an ulp); every
    step after them is compared bit for bit."""
    o, r = C.oracle(), C.reference()
    margins = np.zeros((len(y), groups), np.float32)
    nodes_total = 0
    for _ in range(rounds):
        pairs = C.oracle_gradients(objective, margins, y)
        scales = o.gradient_scales(pairs)
        np.testing.assert_array_equal(_bits(scales), _bits(r.gradient_scales(pairs)))
        q = o.quantize_gradients(pairs, scales)
        np.testing.assert_array_equal(q, r.quantize_gradients(pairs, scales))
        for g in range(groups):
            no, lo = o.grow_tree(bins, q[:, g, :], scales[g], cuts[0], cuts[1], cuts[2], tp)
            nr, lr = r.grow_tree(bins, q[:, g, :], scales[g], cuts[0], cuts[1], cuts[2], tp)
            assert no.tobytes() == nr.tobytes(), "round tree %d differs" % g
            # The harness reports each row's leaf through the reference's
            # predict kernel, as base 0 + leaf: a leaf whose gradient sum is
            # exactly 0 (as many positive as negative rows at margin 0) has
            # weight -0.0 in both node tables and reads +0.0 there.
            np.testing.assert_array_equal(_bits(np.float32(0) + lo), _bits(lr))
            margins[:, g] += lo
            nodes_total += len(no)
    return nodes_total


def test_c4_width_two_rounds_match_reference():
    """c4's shape at 24k rows: 128 N(0, 1) features, 5 % NaN, 256 bins,
    logistic labels from a sparse linear score with one interaction, depth
    10 (trees of several hundred nodes, many with missing values routed by
    their default direction)."""
    rng = np.random.default_rng(4401)
    rows, cols = 24_000, 128
    X = rng.normal(size=(rows, cols)).astype(np.float32)
    mask = rng.random(X.shape) < 0.05
    w = rng.normal(0, 0.1, cols).astype(np.float32)
    Xz = np.where(mask, 0, X)
    logits = Xz @ w + 0.5 * Xz[:, 0] * Xz[:, 1]
    y = (rng.random(rows) < 1 / (1 + np.exp(-logits))).astype(np.float32)
    X[mask] = np.nan
    cuts, bins = _same_cuts(X, 256)
    assert (bins == C.MISSING).any()
    nodes = _boost("binary:logistic", bins, cuts, y, 1, _tree_params(10, 0.1), 2)
    assert nodes > 200


def test_c3_shape_two_rounds_match_reference():
    """c3's shape at 20k rows: 784 integer-valued features in [0, 255], each
    class's cells below the 80th percentile of its pattern held at 0, the
    rest Poisson around the pattern; 10 classes (one tree per class per
    round), depth 6, 256 bins. A fifth of the labels are redrawn at random:
    with clean labels one split separates each class and the trees stop at
    three nodes; with the noise they grow to a few dozen."""
    rng = np.random.default_rng(4402)
    rows, cols, K = 20_000, 784, 10
    P = rng.uniform(0, 255, size=(K, cols)).astype(np.float32)
    keep = P >= np.quantile(P, 0.8, axis=1, keepdims=True)
    labels = rng.permutation(np.arange(rows) % K)
    X = np.clip(rng.poisson(P[labels]), 0, 255).astype(np.float32)
    X = np.where(keep[labels], X, 0).astype(np.float32)
    assert 0.75 < (X == 0).mean() < 0.85
    y = np.where(rng.random(rows) < 0.2, rng.integers(0, K, rows), labels).astype(np.float32)
    cuts, bins = _same_cuts(X, 256)
    nodes = _boost("multi:softprob", bins, cuts, y, K, _tree_params(6, 0.3), 2)
    assert nodes > 2 * K * 20


def test_reference_softmax_gradients_agree_with_the_oracle():
    """The reference's softmax gradients kernel (host libm exp) against the
    oracle's restatement (deterministic exp) on c3's 10 classes: most pairs
    are equal, and the rest differ by one rounding of the probability, at
    most 2^-24 in absolute value (p - 1 for the label's class cancels, so
    the difference can span many ulps of a small gradient)."""
    rng = np.random.default_rng(4403)
    rows, K = 5_000, 10
    margins = (rng.normal(size=(rows, K)) * 2).astype(np.float32)
    y = rng.integers(0, K, rows).astype(np.float32)
    got = C.reference_gradients("multi:softprob", margins, y)
    want = C.oracle_gradients("multi:softprob", margins, y)
    diff = np.abs(got.astype(np.float64) - want.astype(np.float64))
    assert diff.max() <= 2.0 ** -24
    assert (diff == 0).mean() > 0.7


def test_reference_level_loop_at_c4_width_matches_its_serial_form():
    """The bench's reference arm (the reference's functions over its
    feature-major uint16 bins, the smaller child of each pair built and its
    sibling subtracted, on all host threads) grows the same depth-10 tree as
    the reference's serial form and the oracle at c4's width."""
    o, r = C.oracle(), C.reference()
    rng = np.random.default_rng(4404)
    rows, cols = 16_000, 128
    X = rng.normal(size=(rows, cols)).astype(np.float32)
    X[rng.random(X.shape) < 0.05] = np.nan
    y = (rng.random(rows) < 0.4).astype(np.float32)
    cuts, counts, minima = r.sketch_cuts(X, 256)
    bins = r.quantize(X, cuts, counts)
    fm = C.reference_quantize_fm(X, cuts, counts)
    pairs = C.oracle_gradients("binary:logistic", np.zeros((rows, 1), np.float32), y)
    scale = r.gradient_scales(pairs)[0]
    q = r.quantize_gradients(pairs, scale[None])[:, 0, :]
    tp = _tree_params(10, 0.1)
    nf, lf = C.reference_grow_tree_fm(fm, q, scale, cuts, counts, minima, tp)
    ns, ls = r.grow_tree(bins, q, scale, cuts, counts, minima, tp)
    no, lo = o.grow_tree(bins, q, scale, cuts, counts, minima, tp)
    assert len(no) > 100
    assert nf.tobytes() == ns.tobytes() == no.tobytes()
    np.testing.assert_array_equal(_bits(lf), _bits(ls))
    np.testing.assert_array_equal(_bits(np.float32(0) + lo), _bits(ls))


def test_c2_full_size_matches_reference():
    """c2 at its full size, the north_star's 10x configuration: 262,144 rows
    of 64 N(0, 1) features, a linear label with noise, squared error, 256
    bins, depth 8, two rounds (trees of up to 511 nodes). The GPU tests hold
    the CUDA path to the oracle at this size (test_c2_full_size_matches_oracle);
    this holds the oracle to the reference."""
    rng = np.random.default_rng(1337)
    X = rng.normal(size=(262_144, 64)).astype(np.float32)
    w = np.random.default_rng(1338).normal(size=64)
    y = (X @ w + 0.1 * rng.normal(size=len(X))).astype(np.float32)
    cuts, bins = _same_cuts(X, 256)
    nodes = _boost("reg:squarederror", bins, cuts, y, 1, _tree_params(8, 0.3), 2)
    assert nodes > 800


@pytest.mark.parametrize("nan", [0.0, 0.15])
def test_c0_and_c1_full_size_match_reference(nan):
    """c0 and c1 at their full size: 100,000 rows of 32 N(0, 1) features, a
    linear label with noise computed before masking, 15 % NaN for c1;
    squared error, 256 bins, depth 6, eta 0.3, three rounds."""
    rng = np.random.default_rng(1337)
    X = rng.normal(size=(100_000, 32)).astype(np.float32)
    w = np.random.default_rng(1338).normal(size=32)
    y = (X @ w + 0.1 * rng.normal(size=len(X))).astype(np.float32)
    if nan:
        X[rng.random(X.shape) < nan] = np.nan
    cuts, bins = _same_cuts(X, 256)
    nodes = _boost("reg:squarederror", bins, cuts, y, 1, _tree_params(6, 0.3), 3)
    assert nodes > 300

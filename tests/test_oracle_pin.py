"""Pins the oracle: against the golden vectors generated from the reference's
own serial kernel functions (everywhere), and against those functions live on
random inputs where the compiled reference harness is present."""
import os

import numpy as np
import pytest

import checkers as C

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "reference_vectors.npz")


@pytest.fixture(scope="module")
def golden():
    return np.load(GOLDEN)


def _bits(a):
    return np.ascontiguousarray(a).view(np.uint32 if a.dtype == np.float32 else a.dtype)


def _cases(g, prefix):
    return sorted({k.split("_")[1] for k in g.files if k.startswith(prefix)})


def test_golden_cuts_and_bins(golden):
    o = C.oracle()
    names = sorted({k[2:-2] for k in golden.files if k.startswith("q_") and k.endswith("_X")})
    assert len(names) >= 10
    for name in names:
        X = golden["q_%s_X" % name]
        mb = int(golden["q_%s_maxbin" % name][0])
        cuts, counts, minima = o.sketch_cuts(X, mb)
        np.testing.assert_array_equal(counts, golden["q_%s_counts" % name], err_msg=name)
        np.testing.assert_array_equal(_bits(cuts), _bits(golden["q_%s_cuts" % name]), err_msg=name)
        np.testing.assert_array_equal(o.quantize(X, cuts, counts), golden["q_%s_bins" % name],
                                      err_msg=name)


def test_golden_gradient_scales(golden):
    o = C.oracle()
    for k in range(3):
        pairs = golden["g%d_pairs" % k]
        scales = o.gradient_scales(pairs)
        np.testing.assert_array_equal(_bits(scales), _bits(golden["g%d_scales" % k]))
        np.testing.assert_array_equal(o.quantize_gradients(pairs, scales), golden["g%d_q" % k])


def test_golden_trees(golden):
    o = C.oracle()
    fields = ("max_depth", "eta", "reg_lambda", "reg_alpha", "min_child_weight",
              "max_delta_step", "min_split_loss")
    for k in range(3):
        X, pairs = golden["t%d_X" % k], golden["t%d_pairs" % k]
        vals = golden["t%d_params" % k]
        tp = {f: (int(v) if f == "max_depth" else float(np.float32(v))) for f, v in zip(fields, vals)}
        cuts, counts, minima = o.sketch_cuts(X, 64)
        bins = o.quantize(X, cuts, counts)
        scale = o.gradient_scales(pairs)[0]
        q = o.quantize_gradients(pairs, scale[None])[:, 0, :]
        nodes, leaf = o.grow_tree(bins, q, scale, cuts, counts, minima, tp)
        want = golden["t%d_nodes" % k]
        assert len(nodes) == len(want)
        assert nodes.tobytes() == want.tobytes()
        np.testing.assert_array_equal(_bits(leaf), _bits(golden["t%d_leaf" % k]))


needs_ref = pytest.mark.skipif(not C.have_reference(),
                               reason="reference harness not built (no reference checkout)")


@needs_ref
@pytest.mark.parametrize("seed", range(4))
def test_live_splits_match_reference(seed):
    o, r = C.oracle(), C.reference()
    rng = np.random.default_rng(100 + seed)
    rows, cols = 4000, 5
    X = rng.normal(size=(rows, cols)).astype(np.float32)
    X[rng.random(X.shape) < 0.1 * (seed % 3)] = np.nan
    cuts, counts, minima = o.sketch_cuts(X, [16, 64, 256, 33][seed])
    bins = o.quantize(X, cuts, counts)
    pairs = np.stack([rng.normal(size=rows), rng.random(rows) * 2], 1).astype(np.float32)[:, None, :]
    scale = o.gradient_scales(pairs)[0]
    q = o.quantize_gradients(pairs, scale[None])[:, 0, :]
    stride = cuts.shape[1]
    sel = [np.arange(rows), np.nonzero(rng.random(rows) < 0.3)[0]]
    hist = np.zeros((2, cols, stride + 1, 2), np.int64)
    for s, idx in enumerate(sel):
        for f in range(cols):
            b = bins[idx, f].astype(np.int64)
            b[b == C.MISSING] = stride
            np.add.at(hist[s, f, :, 0], b, q[idx, 0])
            np.add.at(hist[s, f, :, 1], b, q[idx, 1])
    sums = np.stack([q[idx].sum(0) for idx in sel]).astype(np.int64)
    params = dict(reg_lambda=[1.0, 0.0, 2.5, 1.0][seed], reg_alpha=[0.0, 0.3, 0.0, 2.0][seed],
                  min_child_weight=[1.0, 0.0, 4.0, 0.5][seed], max_delta_step=[0.0, 0.3, 0.0, 1.0][seed])
    for ups in (0, 1):
        eo = o.evaluate_splits(hist, scale, cuts, counts, minima, params, ups, sums)
        er = r.evaluate_splits(hist, scale, cuts, counts, minima, params, ups, sums)
        assert eo.tobytes() == er.tobytes()
        assert o.select_splits(eo, scale, params).tobytes() == r.select_splits(er, scale, params).tobytes()


@needs_ref
@pytest.mark.parametrize("seed", range(3))
def test_live_cuts_and_trees_match_reference(seed):
    o, r = C.oracle(), C.reference()
    rng = np.random.default_rng(200 + seed)
    rows, cols = [5000, 20000, 700][seed], 4
    X = rng.normal(size=(rows, cols)).astype(np.float32)
    X[rng.random(X.shape) < 0.15 * seed] = np.nan
    mb = [256, 32, 128][seed]
    co, cr = o.sketch_cuts(X, mb), r.sketch_cuts(X, mb)
    for a, b in zip(co, cr):
        np.testing.assert_array_equal(_bits(a), _bits(b))
    bins = o.quantize(X, *co[:2])
    np.testing.assert_array_equal(bins, r.quantize(X, *cr[:2]))
    y = (np.nan_to_num(X[:, 0]) + rng.normal(size=rows)).astype(np.float32)
    pairs = np.stack([-y, np.ones(rows, np.float32)], 1)[:, None, :]
    scale = o.gradient_scales(pairs)[0]
    q = o.quantize_gradients(pairs, scale[None])[:, 0, :]
    tp = dict(max_depth=[3, 6, 9][seed], eta=0.3, reg_lambda=1.0, reg_alpha=0.0,
              min_child_weight=1.0, max_delta_step=0.0, min_split_loss=0.0)
    no, lo = o.grow_tree(bins, q, scale, co[0], co[1], co[2], tp)
    nr, lr = r.grow_tree(bins, q, scale, cr[0], cr[1], cr[2], tp)
    assert no.tobytes() == nr.tobytes()
    np.testing.assert_array_equal(_bits(lo), _bits(lr))


def test_oracle_signed_zero_reads_as_positive():
    # [ours]: the summary of +0/-0 mixtures is the one of +0 only.
    o = C.oracle()
    X = np.array([[0.0], [-0.0], [1.0], [-0.0], [2.0], [0.0]], np.float32)
    c1 = o.sketch_cuts(X, 256)
    c2 = o.sketch_cuts(np.abs(X), 256)
    np.testing.assert_array_equal(_bits(c1[0]), _bits(c2[0]))


def test_det_exp_is_correctly_rounded_on_a_grid():
    o = C.oracle()
    import ctypes
    f = o._l.lib.orc_expf
    f.restype = ctypes.c_float
    f.argtypes = [ctypes.c_float]
    xs = np.linspace(-87, 88, 20001).astype(np.float32)
    got = np.array([f(float(x)) for x in xs], np.float32)
    want = np.exp(xs.astype(np.float64)).astype(np.float32)
    assert np.array_equal(got, want)


@pytest.mark.skipif(not C.have_reference(), reason="reference harness not built")
@pytest.mark.parametrize("seed", [0, 1])
def test_reference_cpu_path_matches_its_serial_form(seed):
    """The bench's reference arm runs the reference's functions on all host
    threads over its feature-major uint16 bins, building the smaller child of
    each pair and subtracting the sibling. Its trees and leaf values equal the
    serial harness's (every node built) and the oracle's, bit for bit, and
    the reference's gradients kernel equals the oracle's restatement."""
    o, r = C.oracle(), C.reference()
    rng = np.random.default_rng(300 + seed)
    rows, cols = [6000, 9000][seed], 7
    X = rng.normal(size=(rows, cols)).astype(np.float32)
    X[rng.random(X.shape) < 0.1 * seed] = np.nan
    cuts, counts, minima = r.sketch_cuts(X, 64)
    bins = r.quantize(X, cuts, counts)
    fm = C.reference_quantize_fm(X, cuts, counts)
    want_fm = np.where(bins == C.MISSING, 0xFFFF, bins).T.astype(np.uint16)
    np.testing.assert_array_equal(fm, want_fm)
    objective = ["reg:squarederror", "binary:logistic"][seed]
    y = (rng.random(rows) < 0.4).astype(np.float32) if seed else rng.normal(size=rows).astype(np.float32)
    margins = (rng.normal(size=(rows, 1)) * 0.5).astype(np.float32)
    pairs = C.reference_gradients(objective, margins, y)
    want = C.oracle_gradients(objective, margins, y)
    if objective == "reg:squarederror":
        np.testing.assert_array_equal(_bits(pairs), _bits(want))
    else:
        # The harness's sigmoid takes the host libm's exp, the oracle's the
        # deterministic det_expf: a few values differ by an ulp or two.
        assert np.abs(_bits(pairs).astype(np.int64) - _bits(want).astype(np.int64)).max() <= 2
    scale = r.gradient_scales(pairs)[0]
    q = r.quantize_gradients(pairs, scale[None])[:, 0, :]
    tp = dict(max_depth=[6, 8][seed], eta=0.3, reg_lambda=1.0, reg_alpha=0.0,
              min_child_weight=1.0, max_delta_step=0.0, min_split_loss=0.0)
    nf, lf = C.reference_grow_tree_fm(fm, q, scale, cuts, counts, minima, tp)
    ns, ls = r.grow_tree(bins, q, scale, cuts, counts, minima, tp)
    no, lo = o.grow_tree(bins, q, scale, cuts, counts, minima, tp)
    assert nf.tobytes() == ns.tobytes() == no.tobytes()
    np.testing.assert_array_equal(_bits(lf), _bits(ls))
    np.testing.assert_array_equal(_bits(lf), _bits(lo))

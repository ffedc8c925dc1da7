"""Generates the golden vectors in this directory from the reference's own
serial kernel functions (oracle/_ref/libxgbref.so, built from the reference
checkout by oracle/Makefile). Run here, where the reference exists:

    make -C oracle && python tests/golden/make_golden.py

Each case stores its inputs and the reference's outputs; the tests check the
oracle (everywhere) and the CUDA product (on a GPU) against them.
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))
import checkers as C  # noqa: E402


def quantile_cases(rng):
    """Edge-case families of the reference's histogram tests
    (tests/test_histogram_missing.py:11-20, 63-80; tests/test_gpu_tree.py:36-80):
    row counts around SIMD/tile sizes, entirely missing and constant columns,
    ties, subnormal values."""
    cases = {}
    for rows in (1, 31, 32, 33, 255, 256, 257, 2049):
        X = rng.normal(size=(rows, 3)).astype(np.float32)
        X[:, 1] = np.round(X[:, 1] * 2)          # ties
        X[rng.random(rows) < 0.2, 2] = np.nan   # missing
        cases["rows%d" % rows] = (X, 256)
    X = rng.normal(size=(600, 4)).astype(np.float32)
    X[:, 0] = np.nan                                 # entirely missing
    X[:, 1] = 7.0                                    # constant
    X[:, 2] = rng.integers(0, 5, 600).astype(np.float32)
    X[:, 3] = (rng.normal(size=600) * 1e-39).astype(np.float32)  # subnormals
    cases["special"] = (X, 16)
    X = rng.normal(size=(20000, 2)).astype(np.float32)
    X[rng.random(X.shape) < 0.15] = np.nan
    cases["nan15_mb256"] = (X, 256)
    cases["nan15_mb7"] = (X, 7)
    return cases


def main():
    ref = C.reference()
    rng = np.random.default_rng(20261201)
    out = {}
    for name, (X, mb) in quantile_cases(rng).items():
        # -0 is read as +0 by the oracle and the product (the reference keeps
        # the first signed zero it meets), so inputs carry +0 only.
        X = (X + np.float32(0)).astype(np.float32)
        cuts, counts, minima = ref.sketch_cuts(X, mb)
        bins = ref.quantize(X, cuts, counts)
        out["q_%s_X" % name] = X
        out["q_%s_maxbin" % name] = np.array([mb])
        out["q_%s_cuts" % name] = cuts
        out["q_%s_counts" % name] = counts
        out["q_%s_bins" % name] = bins
    # Gradient scales and fixed-point gradients, incl. an all-zero column,
    # subnormal and huge magnitudes (tests/test_gradient_precision.py:12-27).
    for k, n in enumerate((1, 100, 5000)):
        pairs = np.stack([rng.normal(size=n) * 10.0 ** rng.integers(-20, 20, n),
                          np.abs(rng.normal(size=n))], 1).astype(np.float32)[:, None, :]
        if k == 2:
            pairs[:50, 0, 0] = np.float32(3e-42)
            pairs[50:60, 0, 0] = np.float32(3e38)
            pairs[:, 0, 1] = 0
        scales = ref.gradient_scales(pairs)
        out["g%d_pairs" % k] = pairs
        out["g%d_scales" % k] = scales
        out["g%d_q" % k] = ref.quantize_gradients(pairs, scales)
    # Whole trees (histograms, split scan, selection, driver, replay) under
    # several regularisation settings.
    settings = [
        dict(max_depth=6, eta=0.3, reg_lambda=1.0, reg_alpha=0.0, min_child_weight=1.0,
             max_delta_step=0.0, min_split_loss=0.0),
        dict(max_depth=4, eta=0.1, reg_lambda=0.0, reg_alpha=0.7, min_child_weight=3.0,
             max_delta_step=0.5, min_split_loss=2.0),
        dict(max_depth=8, eta=1.0, reg_lambda=5.0, reg_alpha=0.0, min_child_weight=0.0,
             max_delta_step=0.0, min_split_loss=0.0),
    ]
    for k, tp in enumerate(settings):
        rows, cols = 3000, 6
        X = rng.normal(size=(rows, cols)).astype(np.float32)
        X[rng.random(X.shape) < 0.1 * k] = np.nan
        y = (np.nan_to_num(X[:, 0]) * 2 + np.nan_to_num(X[:, 1]) ** 2 +
             rng.normal(size=rows)).astype(np.float32)
        h = np.ones(rows, np.float32) if k != 1 else (rng.random(rows) * 2).astype(np.float32)
        pairs = np.stack([-y, h], 1).astype(np.float32)[:, None, :]
        cuts, counts, minima = ref.sketch_cuts(X, 64)
        bins = ref.quantize(X, cuts, counts)
        scale = ref.gradient_scales(pairs)[0]
        q = ref.quantize_gradients(pairs, scale[None])[:, 0, :]
        nodes, leaf = ref.grow_tree(bins, q, scale, cuts, counts, minima, tp)
        out["t%d_X" % k] = X
        out["t%d_pairs" % k] = pairs
        out["t%d_params" % k] = np.array([tp[f] for f in (
            "max_depth", "eta", "reg_lambda", "reg_alpha", "min_child_weight", "max_delta_step",
            "min_split_loss")], np.float64)
        out["t%d_nodes" % k] = nodes
        out["t%d_leaf" % k] = leaf
    np.savez_compressed(os.path.join(HERE, "reference_vectors.npz"), **out)
    print("wrote", len(out), "arrays")


if __name__ == "__main__":
    main()

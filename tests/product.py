"""ctypes bindings to the product library's kernel-level test entry points
(include/xgb_b200.h)."""
import ctypes
import json
import os

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_PATH = os.path.join(ROOT, "xgboost-metal_b200", "xgboost", "lib", "libxgboost.so")

DEVNODE_DTYPE = np.dtype([
    ("left", "<i4"), ("right", "<i4"), ("parent", "<i4"), ("feature", "<i4"),
    ("split_bin", "<i4"), ("default_left", "<u4"), ("threshold", "<f4"), ("leaf", "<f4"),
    ("cover", "<f4"), ("gain", "<f4"), ("base_weight", "<f4"), ("flags", "<u4")])
assert DEVNODE_DTYPE.itemsize == 48

_lib = None


def lib():
    global _lib
    if _lib is None:
        _lib = ctypes.CDLL(LIB_PATH)
        _lib.XGBGetLastError.restype = ctypes.c_char_p
    return _lib


def _ptr(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def check(ret):
    if ret != 0:
        raise RuntimeError(lib().XGBGetLastError().decode())


def quantize(X, max_bin):
    X = np.ascontiguousarray(X, np.float32)
    rows, cols = X.shape
    stride = max(1, min(max_bin, rows))
    cuts = np.zeros((cols, stride), np.float32)
    counts = np.zeros(cols, np.uint32)
    minima = np.zeros(cols, np.float32)
    bins = np.zeros((rows, cols), np.uint32)
    check(lib().XGBBQuantizeHost(_ptr(X), ctypes.c_uint64(rows), ctypes.c_uint64(cols),
                                 ctypes.c_uint32(max_bin), _ptr(cuts), _ptr(counts), _ptr(minima),
                                 _ptr(bins)))
    return cuts, counts, minima, bins


def gradients(objective, margins, labels, weights=None, scale_pos_weight=1.0):
    margins = np.ascontiguousarray(margins, np.float32)
    rows, groups = margins.shape
    pairs = np.zeros((groups, rows, 2), np.float32)
    scales = np.zeros((groups, 2), np.float32)
    code = {"reg:squarederror": 0, "binary:logistic": 1, "multi:softprob": 3}[objective]
    check(lib().XGBBGradientsHost(ctypes.c_int(code), _ptr(margins),
                                  _ptr(np.ascontiguousarray(labels, np.float32)),
                                  _ptr(None if weights is None else np.ascontiguousarray(weights, np.float32)),
                                  ctypes.c_uint64(rows), ctypes.c_uint32(groups),
                                  ctypes.c_float(scale_pos_weight), _ptr(pairs), _ptr(scales)))
    return pairs.transpose(1, 0, 2).copy(), scales


def train(X, y, params, rounds, weights=None):
    X = np.ascontiguousarray(X, np.float32)
    rows, cols = X.shape
    groups = int(params.get("num_class", 1)) if params.get("objective", "").startswith("multi") else 1
    depth = int(params.get("max_depth", 6))
    tree_cap = 2 * rows + 1
    if 0 < depth < 31:
        tree_cap = min(tree_cap, (2 << depth) - 1)
    cap = rounds * groups * tree_cap
    nodes = np.zeros(cap, DEVNODE_DTYPE)
    sizes = np.zeros(rounds * groups, np.uint32)
    margins = np.zeros((rows, groups), np.float32)
    p = {k: str(v) for k, v in params.items()}
    check(lib().XGBBTrainHost(_ptr(X), ctypes.c_uint64(rows), ctypes.c_uint64(cols),
                              _ptr(np.ascontiguousarray(y, np.float32)),
                              _ptr(None if weights is None else np.ascontiguousarray(weights, np.float32)),
                              json.dumps(p).encode(), ctypes.c_uint32(rounds), _ptr(nodes),
                              ctypes.c_uint64(cap), _ptr(sizes), _ptr(margins)))
    trees, off = [], 0
    for s in sizes:
        trees.append(nodes[off:off + s])
        off += int(s)
    return trees, margins


def sketch_device(X, max_bin, weights=None):
    """The GPU sketch (XGBBSketchDevice): cuts, counts, minima."""
    X = np.ascontiguousarray(X, np.float32)
    rows, cols = X.shape
    stride = max(1, min(max_bin, rows))
    cuts = np.zeros((cols, stride), np.float32)
    counts = np.zeros(cols, np.uint32)
    minima = np.zeros(cols, np.float32)
    w = None if weights is None else np.ascontiguousarray(weights, np.float32)
    check(lib().XGBBSketchDevice(_ptr(X), ctypes.c_uint64(rows), ctypes.c_uint64(cols), _ptr(w),
                                 ctypes.c_uint32(max_bin), _ptr(cuts), _ptr(counts), _ptr(minima)))
    return cuts, counts, minima


def sketch(X, max_bin, weights=None, threads=0):
    """The product's host sketch (no GPU): cuts, counts, minima."""
    X = np.ascontiguousarray(X, np.float32)
    rows, cols = X.shape
    stride = max(1, min(max_bin, rows))
    cuts = np.zeros((cols, stride), np.float32)
    counts = np.zeros(cols, np.uint32)
    minima = np.zeros(cols, np.float32)
    w = None if weights is None else np.ascontiguousarray(weights, np.float32)
    check(lib().XGBBSketchHost(_ptr(X), ctypes.c_uint64(rows), ctypes.c_uint64(cols), _ptr(w),
                               ctypes.c_uint32(max_bin), ctypes.c_int(threads), _ptr(cuts),
                               _ptr(counts), _ptr(minima)))
    return cuts, counts, minima


def capture_level_histograms(booster, depth):
    """Ask the booster's next round to keep the built histograms of level
    `depth` of its first tree (XGBoosterCaptureLevelHistograms)."""
    check(lib().XGBoosterCaptureLevelHistograms(booster.handle, ctypes.c_int(depth)))


def level_histograms(booster):
    """The captured level: (meta dict, hist int64 [pairs][features][bins + 1][2],
    node id of each built histogram)."""
    meta = ctypes.c_char_p()
    hist = ctypes.POINTER(ctypes.c_int64)()
    ids = ctypes.POINTER(ctypes.c_uint32)()
    check(lib().XGBoosterGetLevelHistograms(booster.handle, ctypes.byref(meta), ctypes.byref(hist),
                                            ctypes.byref(ids)))
    m = json.loads(meta.value.decode())
    nf = m["f_hi"] - m["f_lo"]
    n = m["pairs"] * nf * m["bins1"] * 2
    h = np.ctypeslib.as_array(hist, shape=(n,)).copy() if n else np.zeros(0, np.int64)
    node_ids = (np.ctypeslib.as_array(ids, shape=(m["pairs"],)).copy() if m["pairs"]
                else np.zeros(0, np.uint32))
    return m, h.reshape(m["pairs"], nf, m["bins1"], 2), node_ids

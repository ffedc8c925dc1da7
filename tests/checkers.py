"""ctypes bindings to the CPU checkers under oracle/ (test infrastructure).

liboracle.so is the C restatement of the reference's training semantics;
_ref/libxgbref.so holds the reference's own serial kernel functions compiled
for the host. Tests use both only to check results; the product never loads
either library.
"""
import ctypes
import os

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
ORACLE_DIR = os.path.join(ROOT, "oracle")

SPLIT_DTYPE = np.dtype([
    ("gain", "<f4"), ("threshold", "<f4"), ("applied_parent_weight", "<f4"), ("left_h", "<f4"),
    ("applied_parent_hessian", "<f4"), ("right_h", "<f4"), ("feature", "<i4"),
    ("default_left", "<u4"), ("left_weight", "<f4"), ("right_weight", "<f4"), ("total_g", "<f4"),
    ("total_h", "<f4"), ("split_type", "<u4"), ("category_begin", "<u4"),
    ("category_count", "<u4"), ("parent_weight", "<f4"), ("left_sum_g", "<i8"),
    ("left_sum_h", "<i8"), ("right_sum_g", "<i8"), ("right_sum_h", "<i8")])
assert SPLIT_DTYPE.itemsize == 96

NODE_DTYPE = np.dtype([
    ("left", "<i4"), ("right", "<i4"), ("feature", "<i4"), ("parent", "<i4"),
    ("threshold", "<f4"), ("leaf", "<f4"), ("cover", "<f4"), ("gain", "<f4"),
    ("default_left", "<u4"), ("split_bin", "<i4")])
assert NODE_DTYPE.itemsize == 40

MISSING = 0xFFFFFFFF

_P = ctypes.c_void_p
_U32 = ctypes.c_uint32
_F = ctypes.c_float


def _ptr(a):
    return None if a is None else a.ctypes.data_as(_P)


def _load(path):
    if not os.path.exists(path):
        return None
    return ctypes.CDLL(path)


def build():
    """Build the checkers in place (the reference harness only where the
    reference checkout exists)."""
    import subprocess
    subprocess.run(["make", "-s", "-C", ORACLE_DIR], check=True)


class _Lib:
    def __init__(self, lib, prefix):
        self.lib = lib
        self.p = prefix

    def fn(self, name, restype=None):
        f = getattr(self.lib, self.p + name)
        f.restype = restype
        return f


class Checker:
    """Common interface over the oracle and the reference harness."""

    def __init__(self, kind):
        if kind == "oracle":
            lib = _load(os.path.join(ORACLE_DIR, "liboracle.so"))
            prefix = "orc_"
        else:
            lib = _load(os.path.join(ORACLE_DIR, "_ref", "libxgbref.so"))
            prefix = "xgbref_"
        if lib is None:
            raise FileNotFoundError(kind)
        self.kind = kind
        self._l = _Lib(lib, prefix)

    def sketch_cuts(self, X, max_bin, weights=None):
        X = np.ascontiguousarray(X, dtype=np.float32)
        rows, cols = X.shape
        stride = max(1, min(max_bin, rows))
        cuts = np.zeros((cols, stride), np.float32)
        counts = np.zeros(cols, np.uint32)
        minima = np.zeros(cols, np.float32)
        w = None if weights is None else np.ascontiguousarray(weights, dtype=np.float32)
        got = self._l.fn("sketch_cuts", ctypes.c_int)(
            _ptr(X), _U32(rows), _U32(cols), _ptr(w), _U32(max_bin), _ptr(cuts), _ptr(counts),
            _ptr(minima))
        assert got == stride
        return cuts, counts, minima

    def quantize(self, X, cuts, counts):
        X = np.ascontiguousarray(X, dtype=np.float32)
        rows, cols = X.shape
        out = np.zeros((rows, cols), np.uint32)
        self._l.fn("quantize")(_ptr(X), _U32(rows), _U32(cols), _ptr(cuts), _U32(cuts.shape[1]),
                               _ptr(counts), _ptr(out))
        return out

    def gradient_scales(self, pairs):
        pairs = np.ascontiguousarray(pairs, dtype=np.float32)
        rows, groups = pairs.shape[0], pairs.shape[1]
        scales = np.zeros((groups, 2), np.float32)
        self._l.fn("gradient_scales")(_ptr(pairs), _U32(rows), _U32(groups), _ptr(scales))
        return scales

    def quantize_gradients(self, pairs, scales):
        pairs = np.ascontiguousarray(pairs, dtype=np.float32)
        rows, groups = pairs.shape[0], pairs.shape[1]
        q = np.zeros((rows, groups, 2), np.int64)
        self._l.fn("quantize_gradients")(_ptr(pairs), _U32(rows), _U32(groups),
                                         _ptr(np.ascontiguousarray(scales, np.float32)), _ptr(q))
        return q

    def evaluate_splits(self, hist, scale, cuts, counts, minima, params, use_parent_sums,
                        node_sums):
        nodes, cols, b1, _ = hist.shape
        out = np.zeros(nodes * cols, SPLIT_DTYPE)
        self._l.fn("evaluate_splits")(
            _ptr(np.ascontiguousarray(hist, np.int64)), _U32(nodes), _U32(cols), _U32(b1 - 1),
            _ptr(np.ascontiguousarray(scale, np.float32)), _ptr(cuts), _ptr(counts), _ptr(minima),
            _F(params["reg_lambda"]), _F(params["reg_alpha"]), _F(params["min_child_weight"]),
            _F(params["max_delta_step"]), _U32(use_parent_sums),
            _ptr(np.ascontiguousarray(node_sums, np.int64)), _ptr(out))
        return out.reshape(nodes, cols)

    def select_splits(self, candidates, scale, params):
        nodes, cols = candidates.shape
        best = np.zeros(nodes, SPLIT_DTYPE)
        self._l.fn("select_splits")(
            _ptr(np.ascontiguousarray(candidates)), _U32(nodes), _U32(cols),
            _ptr(np.ascontiguousarray(scale, np.float32)), _F(params["reg_lambda"]),
            _F(params["reg_alpha"]), _F(params["max_delta_step"]), _ptr(best))
        return best

    def grow_tree(self, bins, q, scale, cuts, counts, minima, params):
        rows, cols = bins.shape
        cap = (2 << params["max_depth"]) - 1
        nodes = np.zeros(cap, NODE_DTYPE)
        leaf = np.zeros(rows, np.float32)
        args = [_ptr(np.ascontiguousarray(bins, np.uint32)), _U32(rows), _U32(cols),
                _ptr(np.ascontiguousarray(q, np.int64)), _ptr(np.ascontiguousarray(scale, np.float32)),
                _ptr(cuts), _U32(cuts.shape[1]), _ptr(counts), _ptr(minima)]
        if self.kind == "oracle":
            tp = (ctypes.c_uint32 * 1)(params["max_depth"])
            buf = np.array([params["max_depth"]], np.uint32).tobytes() + np.array(
                [params["eta"], params["reg_lambda"], params["reg_alpha"],
                 params["min_child_weight"], params["max_delta_step"], params["min_split_loss"]],
                np.float32).tobytes()
            tpb = ctypes.create_string_buffer(buf, len(buf))
            del tp
            n = self._l.fn("grow_tree", ctypes.c_int)(*args, tpb, _ptr(nodes), _U32(cap), _ptr(leaf))
        else:
            n = self._l.fn("grow_tree", ctypes.c_int)(
                *args, _U32(params["max_depth"]), _F(params["eta"]), _F(params["reg_lambda"]),
                _F(params["reg_alpha"]), _F(params["min_child_weight"]),
                _F(params["max_delta_step"]), _F(params["min_split_loss"]), _ptr(nodes), _U32(cap),
                _ptr(leaf))
        assert n > 0, n
        return nodes[:n], leaf


def grow_tree_queue(bins, q, scale, cuts, counts, minima, params, lossguide=False, max_leaves=0,
                    capacity=None):
    """The oracle's host-driven grower (queue of leaves; max_depth 0 =
    unlimited): (nodes, per-row leaf values)."""
    lib = ctypes.CDLL(os.path.join(ORACLE_DIR, "liboracle.so"))
    fn = lib.orc_grow_tree_queue
    fn.restype = ctypes.c_int
    rows, cols = bins.shape
    cap = capacity or max(2 * rows + 1, 3)
    nodes = np.zeros(cap, NODE_DTYPE)
    leaf = np.zeros(rows, np.float32)
    tp = _TreeParams(params["max_depth"], params["eta"], params["reg_lambda"], params["reg_alpha"],
                     params["min_child_weight"], params["max_delta_step"], params["min_split_loss"])
    n = fn(_ptr(np.ascontiguousarray(bins, np.uint32)), _U32(rows), _U32(cols),
           _ptr(np.ascontiguousarray(q, np.int64)), _ptr(np.ascontiguousarray(scale, np.float32)),
           _ptr(cuts), _U32(cuts.shape[1]), _ptr(counts), _ptr(minima), ctypes.byref(tp),
           _U32(int(lossguide)), _U32(max_leaves), _ptr(nodes), _U32(cap), _ptr(leaf))
    assert n > 0, n
    return nodes[:n], leaf


def oracle():
    return Checker("oracle")


def reference():
    return Checker("reference")


def have_reference():
    return os.path.exists(os.path.join(ORACLE_DIR, "_ref", "libxgbref.so"))


# --- whole-run training through the oracle -----------------------------------

class _TreeParams(ctypes.Structure):
    _fields_ = [("max_depth", ctypes.c_uint32), ("eta", ctypes.c_float),
                ("reg_lambda", ctypes.c_float), ("reg_alpha", ctypes.c_float),
                ("min_child_weight", ctypes.c_float), ("max_delta_step", ctypes.c_float),
                ("min_split_loss", ctypes.c_float)]


class _TrainParams(ctypes.Structure):
    _fields_ = [("objective", ctypes.c_int), ("num_class", ctypes.c_uint32),
                ("max_bin", ctypes.c_uint32), ("rounds", ctypes.c_uint32),
                ("scale_pos_weight", ctypes.c_float), ("has_base_score", ctypes.c_int),
                ("base_score", ctypes.c_float), ("tree", _TreeParams),
                ("lossguide", ctypes.c_uint32), ("max_leaves", ctypes.c_uint32)]


OBJECTIVES = {"reg:squarederror": 0, "binary:logistic": 1, "multi:softprob": 3}


def train_params(params):
    """Full parameter set with the upstream defaults (the Booster's own)."""
    p = {"objective": "reg:squarederror", "max_depth": 6, "eta": 0.3, "reg_lambda": 1.0,
         "reg_alpha": 0.0, "min_child_weight": 1.0, "max_delta_step": 0.0,
         "min_split_loss": 0.0, "max_bin": 256, "scale_pos_weight": 1.0, "num_class": 0}
    p.update(params)
    return p


def oracle_train(X, y, params, rounds, weights=None):
    """Returns (list of per-tree NODE_DTYPE arrays, margins [rows, groups], base margins)."""
    p = train_params(params)
    X = np.ascontiguousarray(X, np.float32)
    y = np.ascontiguousarray(y, np.float32)
    rows, cols = X.shape
    obj = OBJECTIVES[p["objective"]]
    groups = int(p["num_class"]) if obj == 3 else 1
    tp = _TrainParams(obj, int(p["num_class"]), int(p["max_bin"]), int(rounds),
                      float(p["scale_pos_weight"]), int("base_score" in p),
                      float(p.get("base_score", 0.0)),
                      _TreeParams(int(p["max_depth"]), float(p["eta"]), float(p["reg_lambda"]),
                                  float(p["reg_alpha"]), float(p["min_child_weight"]),
                                  float(p["max_delta_step"]), float(p["min_split_loss"])),
                      int(p.get("grow_policy", "depthwise") == "lossguide"), int(p.get("max_leaves", 0)))
    depth = int(p["max_depth"])
    tree_cap = 2 * rows + 1
    if 0 < depth < 31:
        tree_cap = min(tree_cap, (2 << depth) - 1)
    cap = rounds * groups * tree_cap
    nodes = np.zeros(cap, NODE_DTYPE)
    sizes = np.zeros(rounds * groups, np.uint32)
    margins = np.zeros((rows, groups), np.float32)
    base = np.zeros(groups, np.float32)
    w = None if weights is None else np.ascontiguousarray(weights, np.float32)
    lib = oracle()._l.lib
    lib.orc_train.restype = ctypes.c_int64
    n = lib.orc_train(_ptr(X), _U32(rows), _U32(cols), _ptr(y), _ptr(w), ctypes.byref(tp),
                      _ptr(nodes), ctypes.c_uint64(cap), _ptr(sizes), _ptr(margins), _ptr(base))
    assert n >= 0, n
    trees, off = [], 0
    for s in sizes:
        trees.append(nodes[off:off + s])
        off += int(s)
    return trees, margins, base


def oracle_gradients(objective, margins, labels, weights=None, scale_pos_weight=1.0):
    margins = np.ascontiguousarray(margins, np.float32)
    rows, groups = margins.shape
    pairs = np.zeros((rows, groups, 2), np.float32)
    lib = oracle()._l.lib
    lib.orc_gradients(ctypes.c_int(OBJECTIVES[objective]), _ptr(margins),
                      _ptr(np.ascontiguousarray(labels, np.float32)),
                      _ptr(None if weights is None else np.ascontiguousarray(weights, np.float32)),
                      _U32(rows), _U32(groups), _F(scale_pos_weight), _ptr(pairs))
    return pairs


def oracle_histogram(bins, q, rows, stride):
    """orc_histogram: exact int64 (g, h) sums [cols][stride + 1][2] of the rows
    `rows` (uint32 ids) of the row-major bins, the missing bin last."""
    bins = np.ascontiguousarray(bins, np.uint32)
    q = np.ascontiguousarray(q, np.int64)
    rows = np.ascontiguousarray(rows, np.uint32)
    cols = bins.shape[1]
    hist = np.zeros((cols, stride + 1, 2), np.int64)
    oracle()._l.lib.orc_histogram(_ptr(bins), _U32(cols), _U32(stride), _ptr(q), _ptr(rows),
                                  _U32(len(rows)), _ptr(hist))
    return hist


def oracle_base_margin(objective, labels, weights=None, groups=1, scale_pos_weight=1.0):
    """orc_base_score: the intercept as margins [groups]."""
    labels = np.ascontiguousarray(labels, np.float32)
    score = np.zeros(groups, np.float32)
    margin = np.zeros(groups, np.float32)
    oracle()._l.lib.orc_base_score(ctypes.c_int(OBJECTIVES[objective]), _ptr(labels),
                                   _ptr(None if weights is None else np.ascontiguousarray(weights, np.float32)),
                                   _U32(len(labels)), _U32(groups), _F(scale_pos_weight), _ptr(score),
                                   _ptr(margin))
    return margin


# --- the reference's own CPU path for the bench's reference arm ---------------

def reference_quantize_fm(X, cuts, counts):
    """Feature-major uint16 bins [cols][rows] (0xffff = missing) from the
    reference's quantize kernel (xgbref_quantize_fm)."""
    X = np.ascontiguousarray(X, np.float32)
    rows, cols = X.shape
    out = np.zeros((cols, rows), np.uint16)
    reference()._l.fn("quantize_fm")(_ptr(X), _U32(rows), _U32(cols), _ptr(cuts), _U32(cuts.shape[1]),
                                     _ptr(counts), _ptr(out))
    return out


def reference_gradients(objective, margins, labels, weights=None, scale_pos_weight=1.0):
    """Gradient pairs [rows][groups][2] from the reference's gradients kernel."""
    margins = np.ascontiguousarray(margins, np.float32)
    rows, groups = margins.shape
    pairs = np.zeros((rows, groups, 2), np.float32)
    reference()._l.fn("gradients")(ctypes.c_int(OBJECTIVES[objective]), _ptr(margins),
                                   _ptr(np.ascontiguousarray(labels, np.float32)),
                                   _ptr(None if weights is None else np.ascontiguousarray(weights, np.float32)),
                                   _U32(rows), _U32(groups), _F(scale_pos_weight), _ptr(pairs))
    return pairs


def reference_grow_tree_fm(fm, q, scale, cuts, counts, minima, params):
    """xgbref_grow_tree_fm: (nodes, per-row leaf values) over feature-major
    uint16 bins, smaller child built and sibling subtracted per level."""
    cols, rows = fm.shape
    cap = (2 << params["max_depth"]) - 1
    nodes = np.zeros(cap, NODE_DTYPE)
    leaf = np.zeros(rows, np.float32)
    n = reference()._l.fn("grow_tree_fm", ctypes.c_int)(
        _ptr(np.ascontiguousarray(fm, np.uint16)), _U32(rows), _U32(cols),
        _ptr(np.ascontiguousarray(q, np.int64)), _ptr(np.ascontiguousarray(scale, np.float32)),
        _ptr(cuts), _U32(cuts.shape[1]), _ptr(counts), _ptr(minima), _U32(params["max_depth"]),
        _F(params["eta"]), _F(params["reg_lambda"]), _F(params["reg_alpha"]), _F(params["min_child_weight"]),
        _F(params["max_delta_step"]), _F(params["min_split_loss"]), _ptr(nodes), _U32(cap), _ptr(leaf))
    assert n > 0, n
    return nodes[:n], leaf

"""GPU checks of the host-side entry points around training: a QuantileDMatrix
or DMatrix built from a batch iterator trains the same trees as one built
from the concatenated arrays, in-place prediction equals DMatrix prediction,
a round slice predicts like an iteration range, and custom objectives
(XGBoosterTrainOneIter / XGBoosterBoostOneIter) train through the same
kernels."""
import numpy as np
import pytest

import xgboost as xgb
from test_ingest_cpu import Batches, _parts
from xgboost import core

pytestmark = pytest.mark.gpu

PARAMS = {"objective": "reg:squarederror", "tree_method": "hist", "device": "cuda",
          "max_depth": 5, "eta": 0.3, "max_bin": 64}


def _whole(parts):
    X = np.concatenate([p["data"] for p in parts])
    y = np.concatenate([p["label"] for p in parts])
    w = np.concatenate([p["weight"] for p in parts])
    return X, y, w


def test_iterator_matrices_train_like_arrays():
    rng = np.random.default_rng(11)
    parts = _parts(rng, [3000, 1, 2500, 1200], cols=7)
    X, y, w = _whole(parts)
    want = xgb.train(PARAMS, xgb.QuantileDMatrix(X, y, weight=w, max_bin=64), 4)
    got = xgb.train(PARAMS, xgb.QuantileDMatrix(Batches(parts), max_bin=64), 4)
    assert bytes(got.save_raw("json")) == bytes(want.save_raw("json"))
    lazy = xgb.train(PARAMS, xgb.DMatrix(Batches(parts)), 4)
    assert bytes(lazy.save_raw("json")) == bytes(want.save_raw("json"))
    # A validation matrix built from an iterator with the training cuts.
    ref = xgb.QuantileDMatrix(X, y, weight=w, max_bin=64)
    valid = xgb.QuantileDMatrix(Batches(parts[:2]), max_bin=64, ref=ref)
    assert valid.num_row() == 3001


def test_inplace_predict_and_slices_match_dmatrix_prediction():
    rng = np.random.default_rng(12)
    X = rng.normal(size=(4000, 5)).astype(np.float32)
    X[rng.random(X.shape) < 0.1] = np.nan
    y = (np.nan_to_num(X[:, 0]) - np.nan_to_num(X[:, 2]) + 0.2 * rng.normal(size=4000)).astype(np.float32)
    b = xgb.train(PARAMS, xgb.DMatrix(X, label=y), 6)
    dm = xgb.DMatrix(X)
    np.testing.assert_array_equal(b.inplace_predict(X), b.predict(dm))
    np.testing.assert_array_equal(b.inplace_predict(X.astype(np.float64), predict_type="margin"),
                                  b.predict(dm, output_margin=True))
    margin = rng.normal(size=4000).astype(np.float32)
    np.testing.assert_array_equal(b.inplace_predict(X, base_margin=margin),
                                  b.predict(xgb.DMatrix(X, base_margin=margin)))
    Xm = np.where(np.isnan(X), -999.0, X).astype(np.float32)
    np.testing.assert_array_equal(b.inplace_predict(Xm, missing=-999.0), b.predict(dm))
    np.testing.assert_array_equal(b[:3].predict(dm), b.predict(dm, iteration_range=(0, 3)))
    np.testing.assert_array_equal(b[2:5].predict(dm, output_margin=True) - 0.0,
                                  b.predict(dm, output_margin=True, iteration_range=(2, 5)))


def _squared_error(pred, dtrain):
    y = dtrain.get_label()
    w = dtrain.get_weight()
    g = (pred - y).astype(np.float32)
    h = np.ones_like(g)
    if len(w):
        g, h = (g * w).astype(np.float32), w.astype(np.float32)
    return g, h


@pytest.mark.parametrize("weighted", [False, True])
def test_custom_squared_error_trains_the_builtin_model(weighted):
    """Gradients from Python equal to the built-in ones give the same model
    bytes: the quantised histograms, splits and leaves do not depend on
    where the gradients came from (the built-in unweighted round counts rows
    instead of summing unit Hessians, with the same exact sums)."""
    rng = np.random.default_rng(13)
    X = rng.normal(size=(6000, 6)).astype(np.float32)
    X[rng.random(X.shape) < 0.1] = np.nan
    y = (np.nan_to_num(X[:, 1]) * 2 + rng.normal(size=6000)).astype(np.float32)
    w = rng.random(6000).astype(np.float32) if weighted else None
    params = dict(PARAMS, base_score=0.5)
    want = xgb.train(params, xgb.DMatrix(X, label=y, weight=w), 5)
    got = xgb.train(params, xgb.DMatrix(X, label=y, weight=w), 5, obj=_squared_error)
    assert bytes(got.save_raw("json")) == bytes(want.save_raw("json"))
    # The flat legacy entry point trains the same round.
    d = xgb.DMatrix(X, label=y, weight=w)
    b = xgb.Booster(params, [d])
    for i in range(5):
        g, h = _squared_error(b.predict(d, output_margin=True, training=True), d)
        assert core._LIB.XGBoosterBoostOneIter(
            b.handle, d.handle, g.ctypes.data_as(core.ctypes.POINTER(core.ctypes.c_float)),
            h.ctypes.data_as(core.ctypes.POINTER(core.ctypes.c_float)), core.c_bst_ulong(g.size)) == 0
    assert bytes(b.save_raw("json")) == bytes(want.save_raw("json"))


def test_custom_softmax_objective_learns_and_continues_from_a_model():
    rng = np.random.default_rng(14)
    n, k = 3000, 3
    X = rng.normal(size=(n, 4)).astype(np.float32)
    y = np.argmax(X[:, :k] + 0.3 * rng.normal(size=(n, k)), axis=1).astype(np.float32)

    def softmax_obj(pred, dtrain):
        labels = dtrain.get_label().astype(int)
        p = np.exp(pred - pred.max(axis=1, keepdims=True))
        p /= p.sum(axis=1, keepdims=True)
        onehot = np.eye(k, dtype=np.float32)[labels]
        g = (p - onehot).astype(np.float32)
        h = np.maximum(2.0 * p * (1.0 - p), 1e-6).astype(np.float32)
        return g, h

    params = {"objective": "multi:softprob", "num_class": k, "tree_method": "hist", "device": "cuda",
              "max_depth": 4, "eta": 0.3}
    d = xgb.DMatrix(X, label=y)
    b = xgb.train(params, d, 8, obj=softmax_obj)
    fresh = xgb.DMatrix(X)
    margin = b.predict(fresh, output_margin=True)
    assert margin.shape == (n, k)
    assert np.mean(np.argmax(margin, axis=1) == y) > 0.7
    more = xgb.train(params, d, 2, obj=softmax_obj, xgb_model=b)
    assert more.num_boosted_rounds() == 10 and b.num_boosted_rounds() == 8
    np.testing.assert_array_equal(more[:8].predict(fresh, output_margin=True), margin)


def test_native_evaluation_and_early_stopping():
    rng = np.random.default_rng(15)
    X = rng.normal(size=(4000, 5)).astype(np.float32)
    y = (X[:, 0] > 0).astype(np.float32)
    Xv = rng.normal(size=(1500, 5)).astype(np.float32)
    yv = (Xv[:, 0] > 0).astype(np.float32)
    d, dv = xgb.DMatrix(X, label=y), xgb.DMatrix(Xv, label=yv)
    params = {"objective": "binary:logistic", "tree_method": "hist", "device": "cuda", "max_depth": 3,
              "eval_metric": ["logloss", "auc", "error"]}
    hist = {}
    b = xgb.train(params, d, 4, evals=[(d, "train"), (dv, "valid")], evals_result=hist, verbose_eval=False)
    assert sorted(hist) == ["train", "valid"] and sorted(hist["valid"]) == ["auc", "error", "logloss"]
    assert all(len(v) == 4 for v in hist["valid"].values())
    p = b.predict(dv)
    ll = float(np.mean(-yv * np.log(np.maximum(p, 1e-16)) - (1 - yv) * np.log(np.maximum(1 - p, 1e-16))))
    assert hist["valid"]["logloss"][-1] == pytest.approx(ll, rel=1e-5)
    assert hist["valid"]["error"][-1] == pytest.approx(float(np.mean((p > 0.5) != (yv > 0.5))), abs=1e-9)
    line = b.eval(dv, "v", 7)
    assert line.startswith("[7]\tv-logloss:") and "\tv-auc:" in line
    # Pure-noise labels: the validation loss stops improving quickly.
    noise = xgb.DMatrix(X, label=rng.random(4000).astype(np.float32))
    vnoise = xgb.DMatrix(Xv, label=rng.random(1500).astype(np.float32))
    es = xgb.train({"tree_method": "hist", "device": "cuda", "max_depth": 6, "eta": 1.0}, noise, 50,
                   evals=[(vnoise, "valid")], early_stopping_rounds=2, verbose_eval=False)
    assert es.num_boosted_rounds() < 50
    assert es.num_boosted_rounds() == es.best_iteration + 1 + 2
    best_line = es[: es.best_iteration + 1].eval(vnoise, "valid")
    assert float(best_line.rsplit(":", 1)[1]) == pytest.approx(es.best_score, rel=1e-9)


def test_device_inputs_prediction_variants_and_cut_export():
    import ctypes
    import json as _json

    import torch
    rng = np.random.default_rng(16)
    X = rng.normal(size=(3000, 4)).astype(np.float32)
    X[rng.random(X.shape) < 0.1] = np.nan
    y = (np.nan_to_num(X[:, 0]) + 0.1 * rng.normal(size=3000)).astype(np.float32)
    b = xgb.train(PARAMS, xgb.DMatrix(X, label=y), 4)
    want = b.predict(xgb.DMatrix(X))
    L = core._LIB
    shape = ctypes.POINTER(core.c_bst_ulong)()
    dims = core.c_bst_ulong()
    res = ctypes.POINTER(ctypes.c_float)()

    def out():
        n = int(np.prod([shape[i] for i in range(dims.value)]))
        return np.ctypeslib.as_array(res, (n,)).copy()
    cfg = _json.dumps({"type": 0, "training": False, "iteration_begin": 0, "iteration_end": 0,
                       "strict_shape": False, "missing": None}).encode()
    # A CUDA tensor through the CUDA array interface, as a matrix and in place.
    t = torch.from_numpy(X).cuda()
    cai = _json.dumps(dict(t.__cuda_array_interface__, data=[t.data_ptr(), False])).encode()
    h = ctypes.c_void_p()
    core._check_call(L.XGDMatrixCreateFromCudaArrayInterface(cai, b"{}", ctypes.byref(h)))
    dm = xgb.DMatrix.__new__(xgb.DMatrix)
    dm.handle = h
    np.testing.assert_array_equal(b.predict(dm), want)
    core._check_call(L.XGBoosterPredictFromCudaArray(b.handle, cai, cfg, None, ctypes.byref(shape),
                                                     ctypes.byref(dims), ctypes.byref(res)))
    np.testing.assert_array_equal(out(), want)
    # Columnar host input.
    cols = [np.ascontiguousarray(X[:, c]) for c in range(4)]
    col_json = _json.dumps([_json.loads(core._array_interface(c)) for c in cols]).encode()
    core._check_call(L.XGBoosterPredictFromColumnar(b.handle, col_json, cfg, None, ctypes.byref(shape),
                                                    ctypes.byref(dims), ctypes.byref(res)))
    np.testing.assert_array_equal(out(), want)
    # Into the caller's buffer.
    buf = np.zeros(3000, np.float32)
    dx = xgb.DMatrix(X)
    core._check_call(L.XGBoosterPredictToBuffer(b.handle, dx.handle, cfg,
                                                buf.ctypes.data_as(ctypes.POINTER(ctypes.c_float)),
                                                core.c_bst_ulong(3000), ctypes.byref(shape), ctypes.byref(dims)))
    np.testing.assert_array_equal(buf, want)
    # Cuts of a quantised matrix: per feature -inf, then increasing cut values.
    q = xgb.QuantileDMatrix(X, label=y, max_bin=16)
    ip, vals = ctypes.c_char_p(), ctypes.c_char_p()
    core._check_call(L.XGDMatrixGetQuantileCut(q.handle, b"{}", ctypes.byref(ip), ctypes.byref(vals)))
    ip_ai, v_ai = _json.loads(ip.value.decode()), _json.loads(vals.value.decode())
    indptr = np.ctypeslib.as_array(ctypes.cast(ip_ai["data"][0], ctypes.POINTER(ctypes.c_uint64)), (5,)).copy()
    values = np.ctypeslib.as_array(ctypes.cast(v_ai["data"][0], ctypes.POINTER(ctypes.c_float)),
                                   (int(indptr[-1]),)).copy()
    assert indptr[0] == 0 and np.all(np.diff(indptr) >= 2) and np.all(np.diff(indptr) <= 17)
    for f in range(4):
        seg = values[indptr[f]:indptr[f + 1]]
        assert seg[0] == -np.inf and np.all(np.diff(seg[1:]) > 0)
        assert seg[-1] > np.nanmax(X[:, f])


def test_cross_validation_and_training_callbacks(tmp_path):
    import json as _json

    from xgboost import training
    rng = np.random.default_rng(17)
    X = rng.normal(size=(2400, 5)).astype(np.float32)
    y = (X[:, 0] - 2 * X[:, 3] + 0.3 * rng.normal(size=2400)).astype(np.float32)
    d = xgb.DMatrix(X, label=y)
    res = xgb.cv(PARAMS, d, 5, nfold=3, metrics=["mae"], seed=3, as_pandas=False)
    assert sorted(res) == ["test-mae-mean", "test-mae-std", "train-mae-mean", "train-mae-std"]
    assert all(len(v) == 5 for v in res.values())
    # The same folds trained one by one give the reported test mean.
    packs = training._make_folds(d, 3, PARAMS, 3, False, True, None, ["mae"])
    maes = []
    for p in packs:
        b = xgb.train(PARAMS, p.dtrain, 5)
        maes.append(float(np.mean(np.abs(b.predict(p.dtest) - p.dtest.get_label()))))
    assert res["test-mae-mean"][-1] == pytest.approx(np.mean(maes), rel=1e-5)
    assert res["test-mae-std"][-1] == pytest.approx(np.std(maes), rel=1e-4, abs=1e-7)
    # Callbacks: a learning-rate schedule and checkpoints.
    sched = xgb.callback.LearningRateScheduler([0.3, 0.2, 0.1])
    ckpt = xgb.callback.TrainingCheckPoint(tmp_path, interval=1)
    b = xgb.train(PARAMS, d, 3, evals=[(d, "train")], callbacks=[sched, ckpt], verbose_eval=False)
    ttp = _json.loads(b.save_config())["learner"]["gradient_booster"]["tree_train_param"]
    assert float(ttp["learning_rate"]) == pytest.approx(0.1)
    assert sorted(p.name for p in tmp_path.iterdir()) == ["model_1.json", "model_2.json"]


def test_leaf_prediction_matches_a_host_walk_of_the_model():
    import json as _json
    rng = np.random.default_rng(18)
    X = rng.normal(size=(1500, 4)).astype(np.float32)
    X[rng.random(X.shape) < 0.1] = np.nan
    params = {"objective": "multi:softprob", "num_class": 3, "tree_method": "hist", "device": "cuda",
              "max_depth": 4}
    yk = (np.nan_to_num(X[:, 0]) > 0).astype(np.float32) + (np.nan_to_num(X[:, 1]) > 0.5)
    b = xgb.train(params, xgb.DMatrix(X, label=yk), 3)
    d = xgb.DMatrix(X)
    leaves = b.predict(d, pred_leaf=True)
    assert leaves.shape == (1500, 9)
    trees = _json.loads(bytes(b.save_raw("json")).decode())["learner"]["gradient_booster"]["model"]["trees"]
    want = np.zeros((1500, 9), np.float32)
    for t, tree in enumerate(trees):
        for r in range(1500):
            n = 0
            while tree["left_children"][n] >= 0:
                v = X[r, tree["split_indices"][n]]
                go_left = bool(tree["default_left"][n]) if np.isnan(v) else v < np.float32(tree["split_conditions"][n])
                n = tree["left_children"][n] if go_left else tree["right_children"][n]
            want[r, t] = n
    np.testing.assert_array_equal(leaves, want)
    strict = b.predict(d, pred_leaf=True, strict_shape=True, iteration_range=(1, 3))
    assert strict.shape == (1500, 2, 3, 1)
    np.testing.assert_array_equal(strict.reshape(1500, 6), want[:, 3:])

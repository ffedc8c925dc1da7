"""Evaluation metrics of XGBoosterEvalOneIter, checked on the host through
XGBBMetricHost against direct numpy formulas (the per-row terms of the
reference's metric_partial kernel, kernels/boost.metal:2225-2270) and
scikit-learn's ROC AUC; plus the evaluation-line parsing and metric settings
of the Python training loop."""
import ctypes
import json

import numpy as np
import pytest

import xgboost as xgb
from test_model_io import _model
from xgboost import core, training


def metric(name, pred, labels, weights=None, multiclass=False):
    pred = np.ascontiguousarray(pred, np.float32)
    labels = np.ascontiguousarray(labels, np.float32)
    groups = pred.shape[1] if pred.ndim == 2 else 1
    w = None if weights is None else np.ascontiguousarray(weights, np.float32)
    out = ctypes.c_double()
    fp = ctypes.POINTER(ctypes.c_float)
    ret = core._LIB.XGBBMetricHost(name.encode(), pred.ctypes.data_as(fp), core.c_bst_ulong(len(labels)),
                                   ctypes.c_uint32(groups), labels.ctypes.data_as(fp),
                                   None if w is None else w.ctypes.data_as(fp), ctypes.c_int(int(multiclass)),
                                   ctypes.byref(out))
    if ret != 0:
        raise xgb.XGBoostError(core._LIB.XGBGetLastError().decode())
    return out.value


@pytest.fixture
def data():
    rng = np.random.default_rng(21)
    n = 2000
    y = (rng.random(n) < 0.4).astype(np.float32)
    p = np.clip(0.3 * y + rng.random(n) * 0.7, 0, 1).astype(np.float32)
    p[:50] = np.round(p[:50], 1)  # ties
    w = rng.random(n).astype(np.float32)
    return p, y, w


@pytest.mark.parametrize("weighted", [False, True])
def test_regression_and_binary_metrics_match_numpy(data, weighted):
    p, y, w = data
    ww = w if weighted else np.ones_like(w)
    wsum = ww.astype(np.float64).sum()

    def mean(terms):
        return float((ww * terms).astype(np.float64).sum() / wsum)
    t = y + 0.5
    assert metric("rmse", p, t, w if weighted else None) == pytest.approx(
        np.sqrt(mean((p - t) ** 2)), rel=1e-9)
    assert metric("mae", p, t, w if weighted else None) == pytest.approx(mean(np.abs(p - t)), rel=1e-9)
    assert metric("rmsle", p, t, w if weighted else None) == pytest.approx(
        np.sqrt(mean((np.log1p(p) - np.log1p(t)) ** 2)), rel=1e-6)
    assert metric("mape", p, t, w if weighted else None) == pytest.approx(mean(np.abs((p - t) / t)), rel=1e-6)
    ll = -y * np.log(np.maximum(p, 1e-16)) - (1 - y) * np.log(np.maximum(1 - p, 1e-16))
    assert metric("logloss", p, y, w if weighted else None) == pytest.approx(mean(ll), rel=1e-6)
    assert metric("error", p, y, w if weighted else None) == pytest.approx(
        mean(np.where(p > 0.5, 1 - y, y)), rel=1e-12)
    assert metric("error@0.7", p, y, w if weighted else None) == pytest.approx(
        mean(np.where(p > 0.7, 1 - y, y)), rel=1e-12)


@pytest.mark.parametrize("weighted", [False, True])
def test_auc_matches_scikit_learn(data, weighted):
    sk = pytest.importorskip("sklearn.metrics")
    p, y, w = data
    got = metric("auc", p, y, w if weighted else None)
    assert got == pytest.approx(sk.roc_auc_score(y, p, sample_weight=w if weighted else None), rel=1e-9)
    assert np.isnan(metric("auc", p, np.zeros_like(y)))
    with pytest.raises(xgb.XGBoostError, match="AUC labels"):
        metric("auc", p, y * 2)


def test_multiclass_metrics(data):
    sk = pytest.importorskip("sklearn.metrics")
    rng = np.random.default_rng(22)
    n, k = 1500, 4
    logits = rng.normal(size=(n, k))
    prob = (np.exp(logits) / np.exp(logits).sum(1, keepdims=True)).astype(np.float32)
    y = rng.integers(0, k, n).astype(np.float32)
    w = rng.random(n).astype(np.float32)
    w64 = w.astype(np.float64)
    picked = prob[np.arange(n), y.astype(int)]
    assert metric("mlogloss", prob, y, w, True) == pytest.approx(
        float((w64 * -np.log(picked)).sum() / w64.sum()), rel=1e-6)
    assert metric("merror", prob, y, w, True) == pytest.approx(
        float((w64 * (np.argmax(prob, 1) != y)).sum() / w64.sum()), rel=1e-9)
    # One class against the rest, weighted by each class's positive weight.
    per = [sk.roc_auc_score(y == c, prob[:, c], sample_weight=w) for c in range(k)]
    pos = [w[y == c].astype(np.float64).sum() for c in range(k)]
    assert metric("auc", prob, y, w, True) == pytest.approx(np.dot(per, pos) / np.sum(pos), rel=1e-9)
    with pytest.raises(xgb.XGBoostError, match="out of range"):
        metric("merror", prob, y + k, None, True)
    with pytest.raises(xgb.XGBoostError, match="not been implemented"):
        metric("ndcg", prob, y, None, True)


def test_eval_line_parsing_and_maximize_rules():
    line = "[3]\ttrain-rmse:0.5\tvalid-set-auc:0.75\tvalid-set-error@0.6:0.125"
    assert training._parse_eval(line) == [("train", "rmse", 0.5), ("valid", "set-auc", 0.75),
                                          ("valid", "set-error@0.6", 0.125)]
    assert training._maximize("auc", None) and training._maximize("ndcg@5", None)
    assert not training._maximize("rmse", None) and training._maximize("rmse", True)


def test_eval_metric_settings_accumulate_in_the_config():
    b = xgb.Booster({"eval_metric": ["auc", "logloss", "auc"]})
    b.load_model(bytearray(json.dumps(_model()).encode()))
    b.set_param("eval_metric", "error@0.7")
    cfg = json.loads(b.save_config())
    assert [m["name"] for m in cfg["learner"]["metrics"]] == ["auc", "logloss", "error@0.7"]
    c = xgb.Booster()
    c.load_config(b.save_config())
    assert json.loads(c.save_config())["learner"]["metrics"] == cfg["learner"]["metrics"]


def _sums(name, pred, labels, weights=None, multiclass=False):
    pred = np.ascontiguousarray(pred, np.float32)
    labels = np.ascontiguousarray(labels, np.float32)
    groups = pred.shape[1] if pred.ndim == 2 else 1
    w = None if weights is None else np.ascontiguousarray(weights, np.float32)
    out = (ctypes.c_double * 2)()
    fp = ctypes.POINTER(ctypes.c_float)
    ret = core._LIB.XGBBMetricSumsHost(name.encode(), pred.ctypes.data_as(fp), core.c_bst_ulong(len(labels)),
                                       ctypes.c_uint32(groups), labels.ctypes.data_as(fp),
                                       None if w is None else w.ctypes.data_as(fp), ctypes.c_int(int(multiclass)),
                                       out)
    if ret != 0:
        raise xgb.XGBoostError(core._LIB.XGBGetLastError().decode())
    return out[0], out[1]


def _from_sums(name, loss, weight):
    out = ctypes.c_double()
    ret = core._LIB.XGBBMetricFromSums(name.encode(), ctypes.c_double(loss), ctypes.c_double(weight),
                                       ctypes.byref(out))
    if ret != 0:
        raise xgb.XGBoostError(core._LIB.XGBGetLastError().decode())
    return out.value


@pytest.mark.parametrize("name", ["rmse", "mae", "rmsle", "logloss", "error", "error@0.3", "mape"])
def test_row_shards_sum_to_the_whole_matrix_metric(data, name):
    # Row-sharded evaluation adds every shard's (weighted loss, weight) and
    # finishes once: the metric of all rows, whatever the split.
    p, y, w = data
    y = y + 0.5 if name in ("mape", "rmsle") else y
    whole = metric(name, p, y, w)
    for cuts in ([1000], [1, 700, 1999], [0, 2000]):
        parts = np.split(np.arange(len(y)), cuts)
        sums = [_sums(name, p[i], y[i], w[i]) for i in parts]
        got = _from_sums(name, sum(s[0] for s in sums), sum(s[1] for s in sums))
        assert got == pytest.approx(whole, rel=1e-12)


def test_row_shards_of_multiclass_metrics(data):
    rng = np.random.default_rng(4)
    probs = rng.random((900, 5)).astype(np.float32)
    probs /= probs.sum(1, keepdims=True)
    labels = rng.integers(0, 5, 900).astype(np.float32)
    for name in ("merror", "mlogloss"):
        whole = metric(name, probs, labels, multiclass=True)
        a = _sums(name, probs[:300], labels[:300], multiclass=True)
        b = _sums(name, probs[300:], labels[300:], multiclass=True)
        assert _from_sums(name, a[0] + b[0], a[1] + b[1]) == pytest.approx(whole, rel=1e-12)


def test_auc_is_not_a_row_sum(data):
    p, y, _ = data
    with pytest.raises(xgb.XGBoostError, match="not a sum over rows"):
        _sums("auc", p, y)
    with pytest.raises(xgb.XGBoostError, match="has not been implemented"):
        _from_sums("ndcg", 1.0, 1.0)

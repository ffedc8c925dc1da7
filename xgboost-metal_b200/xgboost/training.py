"""xgboost.train and xgboost.cv (python-package/xgboost/training.py in the
reference): one boosting round per iteration (XGBoosterUpdateOneIter, or
XGBoosterTrainOneIter with a custom objective), evaluation through
XGBoosterEvalOneIter, and the callbacks of callback.py (early stopping,
printing, learning-rate schedules, checkpoints)."""
import ctypes

import numpy as np

from . import callback as cb
from .core import Booster, DMatrix, XGBoostError, _check_call, _LIB

__all__ = ["train", "cv"]


def _parse_eval(line):
    """"[i]\\tname-metric:value..." -> [(name, metric, value)]."""
    return [tuple(k.split("-", 1)) + (v,) for k, v in cb.parse_eval(line)]


def _maximize(metric, maximize):
    if maximize is not None:
        return bool(maximize)
    return metric != "mape" and any(metric.startswith(m) for m in cb._MAXIMIZE)


def _standard_callbacks(callbacks, verbose_eval, early_stopping_rounds, maximize, show_stdv=False):
    callbacks = list(callbacks or [])
    if verbose_eval:
        period = 1 if verbose_eval is True else int(verbose_eval)
        callbacks.append(cb.EvaluationMonitor(period=period, show_stdv=show_stdv))
    if early_stopping_rounds:
        callbacks.append(cb.EarlyStopping(rounds=early_stopping_rounds, maximize=maximize))
    return callbacks


def train(params, dtrain, num_boost_round=10, *, evals=None, obj=None, maximize=None,
          early_stopping_rounds=None, evals_result=None, verbose_eval=True, xgb_model=None,
          callbacks=None, custom_metric=None):
    """Boosts num_boost_round rounds on dtrain; xgb_model (a Booster, a model
    file or its bytes) is continued. Returns the booster (all rounds; with
    early stopping best_iteration and best_score are set)."""
    evals = list(evals or [])
    # The first matrix is the training set; the others share its booster cache.
    bst = Booster(params, [dtrain] + [d for d, _ in evals], model_file=xgb_model)
    container = cb.CallbackContainer(
        _standard_callbacks(callbacks, verbose_eval if evals else False, early_stopping_rounds, maximize),
        metric=custom_metric, output_margin=callable(obj))
    bst = container.before_training(bst)
    for i in range(int(num_boost_round)):
        if container.before_iteration(bst, i, dtrain, evals):
            break
        bst.update(dtrain, i, fobj=obj)
        if container.after_iteration(bst, i, dtrain, evals):
            break
    bst = container.after_training(bst)
    if evals_result is not None:
        evals_result.update(container.history)
    return bst


class _CVPack:
    """One fold: its booster, training and test matrices."""

    def __init__(self, dtrain, dtest, params):
        self.dtrain, self.dtest = dtrain, dtest
        self.watchlist = [(dtrain, "train"), (dtest, "test")]
        self.bst = Booster(params, [dtrain, dtest])

    def update(self, iteration, fobj):
        self.bst.update(self.dtrain, iteration, fobj)

    def eval(self, iteration, feval, output_margin):
        return self.bst.eval_set(self.watchlist, iteration, feval, output_margin)


class _PackedBooster:
    """The folds seen as one model by the callbacks."""

    def __init__(self, cvfolds):
        self.cvfolds = cvfolds

    def update(self, iteration, obj):
        for fold in self.cvfolds:
            fold.update(iteration, obj)

    def eval(self, iteration, feval, output_margin):
        return [f.eval(iteration, feval, output_margin) for f in self.cvfolds]

    def set_attr(self, **kwargs):
        for f in self.cvfolds:
            f.bst.set_attr(**kwargs)

    def attr(self, key):
        return self.cvfolds[0].bst.attr(key)

    def set_param(self, params, value=None):
        for f in self.cvfolds:
            f.bst.set_param(params, value)

    def num_boosted_rounds(self):
        return self.cvfolds[0].bst.num_boosted_rounds()

    @property
    def best_iteration(self):
        return int(self.cvfolds[0].bst.attr("best_iteration"))

    @property
    def best_score(self):
        return float(self.cvfolds[0].bst.attr("best_score"))


def _make_folds(dall, nfold, params, seed, stratified, shuffle, folds, metrics):
    params = dict(params) if not isinstance(params, dict) else dict(params)
    if metrics:
        existing = params.get("eval_metric")
        existing = [existing] if isinstance(existing, str) else list(existing or [])
        params["eval_metric"] = existing + [m for m in metrics if m not in existing]
    if folds is None:
        train = (ctypes.c_void_p * nfold)()
        test = (ctypes.c_void_p * nfold)()
        _check_call(_LIB.XGDMatrixBuildCVFolds(dall.handle, ctypes.c_int(nfold),
                                               ctypes.c_uint(int(seed) & 0xFFFFFFFF),
                                               ctypes.c_int(int(shuffle)), ctypes.c_int(int(stratified)),
                                               train, test))
        pairs = [(DMatrix._from_handle(train[k]), DMatrix._from_handle(test[k])) for k in range(nfold)]
    else:
        if hasattr(folds, "split"):
            labels = dall.get_label()
            idx = list(folds.split(np.zeros(dall.num_row()), labels))
        else:
            idx = [(np.asarray(tr), np.asarray(te)) for tr, te in folds]
        pairs = [(dall.slice(tr), dall.slice(te)) for tr, te in idx]
    return [_CVPack(tr, te, params) for tr, te in pairs]


def cv(params, dtrain, num_boost_round=10, *, nfold=3, stratified=False, folds=None, metrics=(),
       obj=None, maximize=None, early_stopping_rounds=None, fpreproc=None, as_pandas=True,
       verbose_eval=None, show_stdv=True, seed=0, callbacks=None, shuffle=True, custom_metric=None):
    """Cross-validation: nfold boosters trained side by side, each evaluated
    on its train and test folds; returns per-round mean and standard deviation
    of every metric ("test-rmse-mean", ...), cut after the best round when
    early stopping ends the run."""
    if fpreproc is not None:
        raise XGBoostError("fpreproc is not implemented.")
    if isinstance(metrics, str):
        metrics = [metrics]
    cvfolds = _make_folds(dtrain, nfold, params, seed, stratified, shuffle, folds, metrics)
    model = _PackedBooster(cvfolds)
    container = cb.CallbackContainer(
        _standard_callbacks(callbacks, verbose_eval, early_stopping_rounds, maximize, show_stdv=show_stdv),
        metric=custom_metric, output_margin=callable(obj), is_cv=True)
    model = container.before_training(model)
    results = {}
    for i in range(int(num_boost_round)):
        if container.before_iteration(model, i, dtrain, None):
            break
        model.update(i, obj)
        stop = container.after_iteration(model, i, dtrain, None)
        for key, mean, std in container.aggregated_cv:
            results.setdefault(key + "-mean", []).append(mean)
            results.setdefault(key + "-std", []).append(std)
        if stop:
            break
    model = container.after_training(model)
    if early_stopping_rounds and model.attr("best_iteration") is not None:
        keep = model.best_iteration + 1
        results = {k: v[:keep] for k, v in results.items()}
    if as_pandas:
        try:
            import pandas as pd
            return pd.DataFrame.from_dict(results)
        except ImportError:
            pass
    return results


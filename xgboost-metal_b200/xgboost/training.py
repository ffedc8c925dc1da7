"""xgboost.train (python-package/xgboost/training.py:60-207 in the reference):
one XGBoosterUpdateOneIter per round, optional evaluation printing."""
import numpy as np

from .core import Booster, XGBoostError

__all__ = ["train"]


def _metric(name, y, pred, w):
    w = np.ones_like(y) if w is None or len(w) == 0 else w
    if name == "rmse":
        return float(np.sqrt(np.sum(w * (pred - y) ** 2) / np.sum(w)))
    if name == "logloss":
        p = np.clip(pred, 1e-16, 1 - 1e-16)
        return float(-np.sum(w * (y * np.log(p) + (1 - y) * np.log(1 - p))) / np.sum(w))
    if name == "mlogloss":
        p = np.clip(pred[np.arange(len(y)), y.astype(int)], 1e-16, 1)
        return float(-np.sum(w * np.log(p)) / np.sum(w))
    if name == "error":
        return float(np.sum(w * ((pred > 0.5) != (y > 0.5))) / np.sum(w))
    if name == "merror":
        return float(np.sum(w * (np.argmax(pred, 1) != y)) / np.sum(w))
    raise XGBoostError("Unsupported eval_metric: %s" % name)


def _default_metric(params):
    obj = params.get("objective", "reg:squarederror")
    if obj.startswith("binary:"):
        return "logloss"
    if obj in ("multi:softprob", "multi:softmax"):
        return "mlogloss"
    return "rmse"


def train(params, dtrain, num_boost_round=10, *, evals=None, obj=None, maximize=None,
          early_stopping_rounds=None, evals_result=None, verbose_eval=True, xgb_model=None,
          callbacks=None, custom_metric=None):
    params = dict(params or {})
    metrics = params.pop("eval_metric", None)
    if isinstance(metrics, str):
        metrics = [metrics]
    evals = list(evals or [])
    # xgb_model (a Booster, a model file or its bytes) is trained on: the new
    # rounds are appended to its trees.
    bst = Booster(params, [dtrain] + [d for d, _ in evals], model_file=xgb_model)
    history = {}
    for i in range(int(num_boost_round)):
        bst.update(dtrain, i, fobj=obj)
        if evals:
            names = metrics or [_default_metric(params)]
            parts = []
            for dm, name in evals:
                y = dm.get_label()
                pred = bst.predict(dm)
                if params.get("objective") == "multi:softmax":
                    names = ["merror" if m == "mlogloss" else m for m in names]
                    pred = np.eye(int(params["num_class"]))[pred.astype(int)]
                for m in names:
                    v = _metric(m, y, pred, dm.get_weight())
                    history.setdefault(name, {}).setdefault(m, []).append(v)
                    parts.append("%s-%s:%.5f" % (name, m, v))
            if verbose_eval and (verbose_eval is True or i % int(verbose_eval) == 0):
                print("[%d]\t%s" % (i, "\t".join(parts)))
    if evals_result is not None:
        evals_result.update(history)
    return bst

"""xgboost.train (python-package/xgboost/training.py:60-207 in the reference):
one boosting round per iteration (XGBoosterUpdateOneIter, or
XGBoosterTrainOneIter with a custom objective), evaluation through
XGBoosterEvalOneIter plus an optional custom metric, and early stopping
(python-package/xgboost/callback.py EarlyStopping)."""
from .core import Booster, XGBoostError

__all__ = ["train"]

_MAXIMIZE = ("auc", "aucpr", "pre", "pre@", "map", "ndcg", "auc@", "aucpr@", "map@", "ndcg@")


def _parse_eval(line):
    """"[i]\\tname-metric:value..." -> [(name, metric, value)]."""
    out = []
    for item in line.split()[1:]:
        key, value = item.rsplit(":", 1)
        data_name, metric = key.split("-", 1)
        out.append((data_name, metric, float(value)))
    return out


def _maximize(metric, maximize):
    if maximize is not None:
        return bool(maximize)
    return metric in _MAXIMIZE or any(metric.startswith(m) for m in _MAXIMIZE if m.endswith("@"))


def train(params, dtrain, num_boost_round=10, *, evals=None, obj=None, maximize=None,
          early_stopping_rounds=None, evals_result=None, verbose_eval=True, xgb_model=None,
          callbacks=None, custom_metric=None):
    if callbacks:
        raise XGBoostError("Training callbacks are not implemented; use early_stopping_rounds, "
                           "evals_result and verbose_eval.")
    evals = list(evals or [])
    if early_stopping_rounds and not evals:
        raise ValueError("Must have at least 1 validation dataset for early stopping.")
    # xgb_model (a Booster, a model file or its bytes) is trained on: the new
    # rounds are appended to its trees.
    bst = Booster(params, [dtrain] + [d for d, _ in evals], model_file=xgb_model)
    history = {}
    best = None  # (score, iteration)
    stale = 0
    period = 1 if verbose_eval is True else int(verbose_eval or 0)
    for i in range(int(num_boost_round)):
        bst.update(dtrain, i, fobj=obj)
        if not evals:
            continue
        line = bst.eval_set(evals, i, feval=custom_metric, output_margin=callable(obj))
        scores = _parse_eval(line)
        for data_name, metric, value in scores:
            history.setdefault(data_name, {}).setdefault(metric, []).append(value)
        if period and (i % period == 0 or i + 1 == num_boost_round):
            print("[%d]\t%s" % (i, "\t".join("%s-%s:%.5f" % s for s in scores)), flush=True)
        if early_stopping_rounds:
            # The last metric of the last evaluation set decides.
            data_name = scores[-1][0]
            metric, score = [(m, v) for d, m, v in scores if d == data_name][-1]
            better = best is None or (score > best[0] if _maximize(metric, maximize) else score < best[0])
            if better:
                best, stale = (score, i), 0
            else:
                stale += 1
            bst.set_attr(best_score=repr(best[0]), best_iteration=str(best[1]))
            if stale >= early_stopping_rounds:
                break
    if evals_result is not None:
        evals_result.update(history)
    return bst

"""Scikit-learn estimators (python-package/xgboost/sklearn.py in the
reference): XGBRegressor and XGBClassifier over train()."""
import json

import numpy as np

from .core import Booster, DMatrix, XGBoostError
from .training import train

__all__ = ["XGBModel", "XGBRegressor", "XGBClassifier", "XGBRanker", "XGBRFRegressor", "XGBRFClassifier"]

# With scikit-learn present the estimators take its mixins (score(), the
# estimator type tags), as upstream's do.
try:
    from sklearn.base import BaseEstimator as _Base
    from sklearn.base import ClassifierMixin as _ClassifierBase
    from sklearn.base import RegressorMixin as _RegressorBase
except ImportError:  # pragma: no cover - scikit-learn is optional
    _Base = object
    _ClassifierBase = object
    _RegressorBase = object

_PARAM_NAMES = (
    "max_depth", "max_leaves", "max_bin", "grow_policy", "learning_rate", "verbosity",
    "objective", "booster", "tree_method", "n_jobs", "gamma", "min_child_weight",
    "max_delta_step", "subsample", "sampling_method", "colsample_bytree", "colsample_bylevel",
    "colsample_bynode", "reg_alpha", "reg_lambda", "scale_pos_weight", "base_score",
    "random_state", "missing", "num_parallel_tree", "monotone_constraints",
    "interaction_constraints", "importance_type", "device", "validate_parameters",
    "enable_categorical", "feature_types", "max_cat_to_onehot", "max_cat_threshold",
    "multi_strategy", "eval_metric", "early_stopping_rounds", "callbacks")


class XGBModel(_Base):
    def __init__(self, *, n_estimators=100, objective=None, **kwargs):
        self.n_estimators = n_estimators
        self.objective = objective
        for k in _PARAM_NAMES:
            if k != "objective":
                setattr(self, k, kwargs.pop(k, None))
        self.kwargs = kwargs
        self._Booster = None

    def get_params(self, deep=True):
        out = {"n_estimators": self.n_estimators, "objective": self.objective}
        for k in _PARAM_NAMES:
            if k != "objective":
                out[k] = getattr(self, k)
        out.update(self.kwargs)
        return out

    def set_params(self, **params):
        for k, v in params.items():
            if k in _PARAM_NAMES or k in ("n_estimators", "objective"):
                setattr(self, k, v)
            else:
                self.kwargs[k] = v
        return self

    def get_xgb_params(self):
        skip = {"n_estimators", "missing", "n_jobs", "random_state", "importance_type",
                "enable_categorical", "feature_types", "early_stopping_rounds", "callbacks",
                "eval_metric"}
        params = {k: v for k, v in self.get_params().items() if v is not None and k not in skip}
        if self.random_state is not None:
            params["seed"] = self.random_state
        params.setdefault("device", "cuda")
        params.setdefault("tree_method", "hist")
        return params

    def get_booster(self):
        if self._Booster is None:
            raise XGBoostError("need to call fit or load_model beforehand")
        return self._Booster

    @property
    def feature_importances_(self):
        """Importance per input feature (importance_type, default "gain"),
        normalised to sum to one; unused features score zero."""
        b = self.get_booster()
        score = b.get_score(importance_type=self.importance_type or "gain")
        names = b.feature_names or ["f%d" % i for i in range(self.n_features_in_)]
        values = np.array([score.get(f, 0.0) for f in names], dtype=np.float32)
        total = values.sum()
        return values if total == 0 else values / total

    def evals_result(self):
        return self.evals_result_

    # Model files (python-package/xgboost/sklearn.py save_model / load_model):
    # the estimator's own attributes travel in the model's "scikit_learn"
    # attribute.
    def save_model(self, fname):
        meta = {"n_features_in_": getattr(self, "n_features_in_", None)}
        if hasattr(self, "classes_"):
            meta["classes_"] = np.asarray(self.classes_).tolist()
            meta["n_classes_"] = int(self.n_classes_)
        booster = self.get_booster()
        booster.set_attr(scikit_learn=json.dumps(meta))
        booster.save_model(fname)
        booster.set_attr(scikit_learn=None)

    def load_model(self, fname):
        self._Booster = Booster(model_file=fname)
        meta = self._Booster.attr("scikit_learn")
        if meta:
            meta = json.loads(meta)
            if meta.get("n_features_in_") is not None:
                self.n_features_in_ = meta["n_features_in_"]
            if "classes_" in meta:
                self.classes_ = np.asarray(meta["classes_"])
                self.n_classes_ = meta["n_classes_"]
            self._Booster.set_attr(scikit_learn=None)

    def _fit(self, X, y, sample_weight, eval_set, verbose, params, xgb_model=None, base_margin=None,
             sample_weight_eval_set=None, base_margin_eval_set=None):
        missing = np.nan if self.missing is None else self.missing
        dtrain = DMatrix(X, y, weight=sample_weight, base_margin=base_margin, missing=missing,
                         feature_types=self.feature_types)
        evals = []
        eval_set = list(eval_set or [])
        for name, extra in (("sample_weight_eval_set", sample_weight_eval_set),
                            ("base_margin_eval_set", base_margin_eval_set)):
            if extra is not None and len(extra) != len(eval_set):
                raise ValueError("%s must have one entry per eval_set pair" % name)
        for i, (ex, ey) in enumerate(eval_set):
            w = sample_weight_eval_set[i] if sample_weight_eval_set is not None else None
            m = base_margin_eval_set[i] if base_margin_eval_set is not None else None
            evals.append((DMatrix(ex, ey, weight=w, base_margin=m, missing=missing,
                                  feature_types=self.feature_types), "validation_%d" % i))
        self.evals_result_ = {}
        if self.eval_metric is not None:
            params["eval_metric"] = self.eval_metric
        self._Booster = train(params, dtrain, self.n_estimators, evals=evals,
                              evals_result=self.evals_result_, verbose_eval=verbose,
                              early_stopping_rounds=self.early_stopping_rounds,
                              xgb_model=xgb_model.get_booster() if isinstance(xgb_model, XGBModel)
                              else xgb_model)
        self.n_features_in_ = dtrain.num_col()
        if hasattr(X, "columns"):
            self.feature_names_in_ = np.asarray([str(c) for c in X.columns], dtype=object)
        return self

    def _iteration_range(self, iteration_range):
        """All rounds, or up to the best one after early stopping
        (python-package/xgboost/sklearn.py _get_iteration_range)."""
        if iteration_range is not None and tuple(iteration_range) != (0, 0):
            return tuple(iteration_range)
        best = self.get_booster().attr("best_iteration")
        return (0, int(best) + 1) if best is not None else (0, 0)

    @property
    def best_iteration(self):
        return self.get_booster().best_iteration

    @property
    def best_score(self):
        return self.get_booster().best_score

    def predict(self, X, output_margin=False, validate_features=True, base_margin=None,
                iteration_range=None):
        dm = DMatrix(X, missing=np.nan if self.missing is None else self.missing,
                     base_margin=base_margin)
        # As upstream's in-place prediction: names are checked for data
        # frames, only the width for plain arrays.
        b = self.get_booster()
        if validate_features and not hasattr(X, "columns") and dm.num_col() != b.num_features():
            raise ValueError("Feature shape mismatch, expected: %d, got %d" % (b.num_features(), dm.num_col()))
        return b.predict(dm, output_margin=output_margin, validate_features=validate_features and
                         hasattr(X, "columns"), iteration_range=self._iteration_range(iteration_range))


class XGBRegressor(_RegressorBase, XGBModel):
    def __init__(self, *, objective="reg:squarederror", **kwargs):
        super().__init__(objective=objective, **kwargs)

    def fit(self, X, y, *, sample_weight=None, base_margin=None, eval_set=None, verbose=True,
            xgb_model=None, sample_weight_eval_set=None, base_margin_eval_set=None,
            feature_weights=None):
        return self._fit(X, y, sample_weight, eval_set, verbose, self.get_xgb_params(), xgb_model,
                         base_margin, sample_weight_eval_set, base_margin_eval_set)


class XGBClassifier(_ClassifierBase, XGBModel):
    def __init__(self, *, objective="binary:logistic", **kwargs):
        super().__init__(objective=objective, **kwargs)

    def fit(self, X, y, *, sample_weight=None, base_margin=None, eval_set=None, verbose=True,
            xgb_model=None, sample_weight_eval_set=None, base_margin_eval_set=None,
            feature_weights=None):
        y = np.asarray(y)
        self.classes_ = np.unique(y)
        self.n_classes_ = len(self.classes_)
        encoded = np.searchsorted(self.classes_, y).astype(np.float32)
        params = self.get_xgb_params()
        if self.n_classes_ > 2:
            if params.get("objective", "").startswith("binary:"):
                params["objective"] = "multi:softprob"
            params["num_class"] = self.n_classes_
        eval_set = [(ex, np.searchsorted(self.classes_, np.asarray(ey)).astype(np.float32))
                    for ex, ey in (eval_set or [])]
        return self._fit(X, encoded, sample_weight, eval_set, verbose, params, xgb_model,
                         base_margin, sample_weight_eval_set, base_margin_eval_set)

    def predict_proba(self, X, validate_features=True, base_margin=None, iteration_range=None):
        p = super().predict(X, base_margin=base_margin, iteration_range=iteration_range)
        if p.ndim == 1:
            return np.stack([1 - p, p], axis=1)
        return p

    def predict(self, X, output_margin=False, validate_features=True, base_margin=None,
                iteration_range=None):
        if output_margin:
            return super().predict(X, output_margin=True, base_margin=base_margin,
                                   iteration_range=iteration_range)
        p = self.predict_proba(X, base_margin=base_margin, iteration_range=iteration_range)
        return self.classes_[np.argmax(p, axis=1)]


class XGBRanker(XGBModel):
    """Learning to rank needs query groups and ranking objectives, which the
    CUDA backend does not train; fit raises."""

    def __init__(self, *, objective="rank:ndcg", **kwargs):
        super().__init__(objective=objective, **kwargs)

    def fit(self, X, y, *args, **kwargs):
        raise XGBoostError("Ranking objectives and query groups are not implemented by the CUDA backend.")


class XGBRFRegressor(XGBRegressor):
    """Random forests need num_parallel_tree > 1 with row and column
    sampling, which the CUDA backend does not train; fit raises."""

    def fit(self, X, y, *args, **kwargs):
        raise XGBoostError("Random forests (num_parallel_tree > 1, subsample, colsample_*) are not "
                           "implemented by the CUDA backend.")


class XGBRFClassifier(XGBClassifier):
    """See XGBRFRegressor."""

    def fit(self, X, y, *args, **kwargs):
        raise XGBoostError("Random forests (num_parallel_tree > 1, subsample, colsample_*) are not "
                           "implemented by the CUDA backend.")

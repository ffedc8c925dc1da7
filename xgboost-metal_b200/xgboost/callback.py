"""Training callbacks (python-package/xgboost/callback.py in the reference):
the TrainingCallback interface and its stock implementations, driven by a
container that evaluates the model after every round (XGBoosterEvalOneIter)
and keeps the evaluation history."""
import collections
import collections.abc
import math
import os
import pickle
import sys

from .core import Booster

__all__ = ["TrainingCallback", "LearningRateScheduler", "EarlyStopping", "EvaluationMonitor",
           "TrainingCheckPoint", "CallbackContainer"]

_MAXIMIZE = ("auc", "aucpr", "pre", "pre@", "map", "ndcg", "auc@", "aucpr@", "map@", "ndcg@")


class TrainingCallback:
    """Hooks around training: the before/after_training hooks return the
    model, the iteration hooks return True to stop training."""

    def before_training(self, model):
        return model

    def after_training(self, model):
        return model

    def before_iteration(self, model, epoch, evals_log):
        return False

    def after_iteration(self, model, epoch, evals_log):
        return False


def parse_eval(line):
    """"[i]\\tname-metric:value..." -> [("name-metric", value)]."""
    out = []
    for item in line.split()[1:]:
        key, value = item.rsplit(":", 1)
        out.append((key, float(value)))
    return out


def aggregate_cv(lines):
    """Per-fold evaluation lines -> [("name-metric", mean, std)] (population
    standard deviation), in the order the metrics appear."""
    table = collections.OrderedDict()
    for line in lines:
        for position, (key, value) in enumerate(parse_eval(line)):
            table.setdefault((position, key), []).append(value)
    out = []
    for (_, key), values in table.items():
        mean = math.fsum(values) / len(values)
        std = math.sqrt(math.fsum((v - mean) ** 2 for v in values) / len(values))
        out.append((key, mean, std))
    return out


class CallbackContainer:
    """Runs the callbacks and records evaluation history as
    history[data_name][metric_name] = [score, ...] (cv: (mean, std))."""

    def __init__(self, callbacks, metric=None, output_margin=True, is_cv=False):
        self.callbacks = list(dict.fromkeys(callbacks))
        for cb in self.callbacks:
            if not isinstance(cb, TrainingCallback):
                raise TypeError("callback must be an instance of `TrainingCallback`.")
        if metric is not None and not callable(metric):
            raise TypeError("metric must be callable object for monitoring.")
        self.metric = metric
        self.history = collections.OrderedDict()
        self._output_margin = output_margin
        self.is_cv = is_cv
        self.aggregated_cv = None

    def before_training(self, model):
        for cb in self.callbacks:
            model = cb.before_training(model=model)
        return model

    def after_training(self, model):
        for cb in self.callbacks:
            model = cb.after_training(model=model)
        return model

    def before_iteration(self, model, epoch, dtrain, evals):
        return any(cb.before_iteration(model, epoch, self.history) for cb in self.callbacks)

    def _update_history(self, scores):
        for item in scores:
            key = item[0]
            value = (item[1], item[2]) if self.is_cv else item[1]
            data_name, metric_name = key.split("-", 1)
            self.history.setdefault(data_name, collections.OrderedDict()).setdefault(
                metric_name, []).append(value)

    def after_iteration(self, model, epoch, dtrain, evals):
        if self.is_cv:
            scores = aggregate_cv(model.eval(epoch, self.metric, self._output_margin))
            self.aggregated_cv = scores
        else:
            evals = evals or []
            for _, name in evals:
                if "-" in name:
                    raise ValueError("Dataset name should not contain `-`")
            scores = parse_eval(model.eval_set(evals, epoch, self.metric, self._output_margin))
        self._update_history(scores)
        return any(cb.after_iteration(model, epoch, self.history) for cb in self.callbacks)


class LearningRateScheduler(TrainingCallback):
    """Sets learning_rate after every round from a function of the round or a
    sequence."""

    def __init__(self, learning_rates):
        if callable(learning_rates):
            self.learning_rates = learning_rates
        elif isinstance(learning_rates, collections.abc.Sequence):
            self.learning_rates = lambda epoch: learning_rates[epoch]
        else:
            raise TypeError("Invalid learning rates, expecting callable or sequence, got: %s"
                            % type(learning_rates))

    def after_iteration(self, model, epoch, evals_log):
        model.set_param("learning_rate", self.learning_rates(epoch))
        return False


class EarlyStopping(TrainingCallback):
    """Stops when the watched metric (default: the last metric of the last
    evaluation set) has not improved by more than min_delta for `rounds`
    rounds; records best_iteration / best_score on the model, and with
    save_best returns the model cut after the best round."""

    def __init__(self, *, rounds, metric_name=None, data_name=None, maximize=None, save_best=False,
                 min_delta=0.0):
        if min_delta < 0:
            raise ValueError("min_delta must be greater or equal to 0.")
        self.rounds = rounds
        self.metric_name = metric_name
        self.data = data_name
        self.maximize = maximize
        self.save_best = save_best
        self._min_delta = min_delta
        self.best = None
        self.current_rounds = 0
        self.starting_round = 0

    def before_training(self, model):
        self.starting_round = model.num_boosted_rounds()
        if not isinstance(model, Booster) and self.save_best:
            raise ValueError("`save_best` is not applicable to the `cv` function as it doesn't return a model.")
        return model

    def after_iteration(self, model, epoch, evals_log):
        epoch += self.starting_round
        if not evals_log:
            raise ValueError("Must have at least 1 validation dataset for early stopping.")
        data_name = self.data or list(evals_log.keys())[-1]
        if data_name not in evals_log:
            raise ValueError("No dataset named: %s" % data_name)
        metric_name = self.metric_name or list(evals_log[data_name].keys())[-1]
        if metric_name not in evals_log[data_name]:
            raise ValueError("No metric named: %s" % metric_name)
        score = evals_log[data_name][metric_name][-1]
        value = score[0] if isinstance(score, tuple) else score
        if self.maximize is None:
            self.maximize = metric_name != "mape" and any(metric_name.startswith(m) for m in _MAXIMIZE)
        if self.best is None:
            improved = True
        elif self.maximize:
            improved = value - self._min_delta > self.best
        else:
            improved = self.best - self._min_delta > value
        if improved:
            self.best, self.current_rounds = value, 0
            model.set_attr(best_score=str(value), best_iteration=str(epoch))
        else:
            self.current_rounds += 1
        return self.current_rounds >= self.rounds

    def after_training(self, model):
        if not self.save_best:
            return model
        best_iteration, best_score = model.best_iteration, model.best_score
        model = model[: best_iteration + 1]
        model.set_attr(best_iteration=str(best_iteration), best_score=str(best_score))
        return model


class EvaluationMonitor(TrainingCallback):
    """Prints the latest scores every `period` rounds (and the last skipped
    line at the end)."""

    def __init__(self, rank=0, period=1, show_stdv=False, logger=None):
        if period <= 0:
            raise ValueError("period must be positive")
        self.printer_rank = rank
        self.period = period
        self.show_stdv = show_stdv
        self._logger = logger or (lambda msg: print(msg, end="", file=sys.stdout, flush=True))
        self._latest = None

    def _fmt(self, data, metric, score, std):
        if std is not None and self.show_stdv:
            return "\t%s-%s:%.5f+%.5f" % (data, metric, score, std)
        return "\t%s-%s:%.5f" % (data, metric, score)

    def after_iteration(self, model, epoch, evals_log):
        if not evals_log:
            return False
        from . import collective
        if collective.get_rank() != self.printer_rank:
            return False
        msg = "[%d]" % epoch
        for data, metrics in evals_log.items():
            for metric, log in metrics.items():
                last = log[-1]
                score, std = (last[0], last[1]) if isinstance(last, tuple) else (last, None)
                msg += self._fmt(data, metric, score, std)
        msg += "\n"
        if epoch % self.period == 0 or self.period == 1:
            self._logger(msg)
            self._latest = None
        else:
            self._latest = msg
        return False

    def after_training(self, model):
        if self._latest is not None:
            self._logger(self._latest)
        return model


class TrainingCheckPoint(TrainingCallback):
    """Saves the model every `interval` rounds as <directory>/<name>_<n>.json
    (or .pkl with as_pickle)."""

    def __init__(self, directory, name="model", as_pickle=False, interval=100):
        self._path = os.fspath(directory)
        self._name = name
        self._as_pickle = as_pickle
        self._interval = interval
        self._epoch = 0
        os.makedirs(self._path, exist_ok=True)

    def after_iteration(self, model, epoch, evals_log):
        if self._epoch == self._interval:
            path = os.path.join(self._path, "%s_%d.%s" % (self._name, epoch,
                                                          "pkl" if self._as_pickle else "json"))
            self._epoch = 0
            if self._as_pickle:
                with open(path, "wb") as fd:
                    pickle.dump(model, fd)
            else:
                model.save_model(path)
        self._epoch += 1
        return False

"""Training callbacks and cross-validation bookkeeping without a GPU
(python-package/xgboost/callback.py and training.py cv in the reference):
early-stopping decisions, printing, history layout and fold aggregation, on
a stand-in model that records attributes."""
import collections

import pytest

from xgboost import callback as cb


class FakeModel:
    def __init__(self, rounds=0):
        self.attrs = {}
        self.rounds = rounds
        self.params = {}

    def set_attr(self, **kw):
        self.attrs.update(kw)

    def num_boosted_rounds(self):
        return self.rounds

    def set_param(self, k, v=None):
        self.params[k] = v


def _log(**series):
    out = collections.OrderedDict()
    for key, values in series.items():
        data, metric = key.split("__")
        out.setdefault(data, collections.OrderedDict())[metric] = list(values)
    return out


def test_early_stopping_minimises_by_default_and_counts_from_the_model():
    es = cb.EarlyStopping(rounds=2)
    m = es.before_training(FakeModel(rounds=10))
    scores = [0.5, 0.4, 0.45, 0.41, 0.39]
    stops = []
    for i in range(len(scores)):
        stops.append(es.after_iteration(m, i, _log(train__rmse=[0] * (i + 1), valid__rmse=scores[: i + 1])))
        if stops[-1]:
            break
    assert stops == [False, False, False, True]  # two rounds without improving on 0.4
    assert m.attrs == {"best_score": "0.4", "best_iteration": "11"}


def test_early_stopping_maximises_auc_and_honours_min_delta():
    es = cb.EarlyStopping(rounds=1, min_delta=0.01)
    m = es.before_training(FakeModel())
    assert not es.after_iteration(m, 0, _log(valid__auc=[0.80]))
    assert es.after_iteration(m, 1, _log(valid__auc=[0.80, 0.805]))  # below min_delta
    assert m.attrs["best_iteration"] == "0"
    es = cb.EarlyStopping(rounds=1, metric_name="logloss", data_name="train")
    m = es.before_training(FakeModel())
    es.after_iteration(m, 0, _log(train__logloss=[0.3], valid__auc=[0.5]))
    assert m.attrs["best_score"] == "0.3"
    with pytest.raises(ValueError, match="validation dataset"):
        cb.EarlyStopping(rounds=1).after_iteration(FakeModel(), 0, collections.OrderedDict())
    with pytest.raises(ValueError, match="min_delta"):
        cb.EarlyStopping(rounds=1, min_delta=-1)


def test_evaluation_monitor_period_and_std(capsys):
    mon = cb.EvaluationMonitor(period=2, show_stdv=True)
    for i in range(3):
        mon.after_iteration(None, i, _log(test__rmse=[(1.0 + i, 0.25)] * (i + 1)))
    mon.after_training(None)
    out = capsys.readouterr().out.splitlines()
    assert out == ["[0]\ttest-rmse:1.00000+0.25000", "[2]\ttest-rmse:3.00000+0.25000"]
    mon = cb.EvaluationMonitor(period=5)
    mon.after_iteration(None, 1, _log(v__error=[0.125]))
    mon.after_training(None)
    assert capsys.readouterr().out == "[1]\tv-error:0.12500\n"


def test_fold_aggregation_and_history_layout():
    lines = ["[3]\ttrain-rmse:1\ttest-rmse:2", "[3]\ttrain-rmse:3\ttest-rmse:4"]
    agg = cb.aggregate_cv(lines)
    assert agg == [("train-rmse", 2.0, 1.0), ("test-rmse", 3.0, 1.0)]

    class Packed(FakeModel):
        def eval(self, epoch, feval, output_margin):
            return lines

    container = cb.CallbackContainer([], is_cv=True)
    container.after_iteration(Packed(), 3, None, None)
    assert container.history == {"train": {"rmse": [(2.0, 1.0)]}, "test": {"rmse": [(3.0, 1.0)]}}

    class Single(FakeModel):
        def eval_set(self, evals, epoch, feval, output_margin):
            return "[0]\tvalid-auc:0.75\tvalid-error@0.6:0.125"

    container = cb.CallbackContainer([cb.EarlyStopping(rounds=3)])
    model = container.before_training(Single())
    assert not container.after_iteration(model, 0, None, [(None, "valid")])
    assert container.history == {"valid": {"auc": [0.75], "error@0.6": [0.125]}}
    with pytest.raises(ValueError, match="should not contain"):
        container.after_iteration(model, 1, None, [(None, "va-lid")])
    with pytest.raises(TypeError):
        cb.CallbackContainer([object()])


def test_learning_rate_scheduler():
    m = FakeModel()
    sched = cb.LearningRateScheduler([0.3, 0.2, 0.1])
    sched.after_iteration(m, 2, {})
    assert m.params["learning_rate"] == 0.1
    cb.LearningRateScheduler(lambda e: 1.0 / (e + 1)).after_iteration(m, 3, {})
    assert m.params["learning_rate"] == 0.25
    with pytest.raises(TypeError):
        cb.LearningRateScheduler(3)

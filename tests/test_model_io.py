"""Model files in upstream XGBoost's JSON schema (the reference's
src/model.cpp:28-240): save, load, UBJSON and pickling. The CPU tests build a
model document by hand; a booster loads and saves models without a GPU."""
import json
import os
import pickle

import numpy as np
import pytest

import xgboost as xgb


def _tree(left, right, parents, feat, cond, dl, gain, hess, bw):
    n = len(left)
    return {"base_weights": bw, "categories": [], "categories_nodes": [], "categories_segments": [],
            "categories_sizes": [], "default_left": dl, "id": 0, "left_children": left,
            "loss_changes": gain, "parents": parents, "right_children": right,
            "split_conditions": cond, "split_indices": feat, "split_type": [0] * n,
            "sum_hessian": hess,
            "tree_param": {"num_deleted": "0", "num_feature": "3", "num_nodes": str(n),
                           "size_leaf_vector": "1"}}


def _model(objective="binary:logistic", base="[5E-1]", trees=None, num_class="0"):
    trees = trees or [
        _tree([1, -1, -1], [2, -1, -1], [2147483647, 0, 0], [2, 0, 0], [0.25, -0.125, 0.375],
              [1, 0, 0], [3.5, 0, 0], [10.0, 4.0, 6.0], [0.1, -0.125, 0.375]),
        _tree([1, 3, -1, -1, -1], [2, 4, -1, -1, -1], [2147483647, 0, 0, 1, 1], [0, 1, 0, 0, 0],
              [-1.5, 2.0, 0.5, -0.25, 0.75], [0, 1, 0, 0, 0], [1.0, 0.5, 0, 0, 0],
              [10.0, 7.0, 3.0, 2.0, 5.0], [0.0, 0.1, 0.5, -0.25, 0.75])]
    for i, t in enumerate(trees):
        t["id"] = i
    return {"learner": {
        "attributes": {"best_iteration": "1"}, "feature_names": [], "feature_types": [],
        "gradient_booster": {"model": {
            "gbtree_model_param": {"num_parallel_tree": "1", "num_trees": str(len(trees))},
            "iteration_indptr": list(range(len(trees) + 1)), "tree_info": [0] * len(trees),
            "trees": trees}, "name": "gbtree"},
        "learner_model_param": {"base_score": base, "boost_from_average": "1",
                                "num_class": num_class, "num_feature": "3", "num_target": "1"},
        "objective": {"name": objective, "reg_loss_param": {"scale_pos_weight": "1"}}},
        "version": [3, 5, 0]}


def _canon(raw):
    return json.loads(bytes(raw).decode())


def test_json_round_trip_keeps_every_field():
    doc = _model()
    b = xgb.Booster()
    b.load_model(bytearray(json.dumps(doc).encode()))
    assert b.num_boosted_rounds() == 2
    assert b.num_features() == 3
    assert b.attr("best_iteration") == "1"
    out = _canon(b.save_raw("json"))
    for k, t in enumerate(doc["learner"]["gradient_booster"]["model"]["trees"]):
        got = out["learner"]["gradient_booster"]["model"]["trees"][k]
        for field in ("left_children", "right_children", "parents", "split_indices",
                      "default_left", "split_conditions", "sum_hessian", "base_weights"):
            assert got[field] == t[field], field
        # Leaves carry no split gain.
        assert got["loss_changes"] == [g if l >= 0 else 0 for g, l in zip(t["loss_changes"], t["left_children"])]
    assert out["learner"]["learner_model_param"]["base_score"] == "[0.5]"
    assert out["learner"]["objective"]["name"] == "binary:logistic"
    assert out["learner"]["gradient_booster"]["model"]["iteration_indptr"] == [0, 1, 2]


def test_ubj_and_json_describe_the_same_model(tmp_path):
    b = xgb.Booster()
    b.load_model(bytearray(json.dumps(_model()).encode()))
    text = _canon(b.save_raw("json"))
    b.save_model(os.fspath(tmp_path / "m.ubj"))
    b.save_model(os.fspath(tmp_path / "m.json"))
    assert (tmp_path / "m.json").read_bytes()[:1] == b"{"
    assert (tmp_path / "m.ubj").read_bytes()[:1] == b"{"  # UBJSON objects also open with '{'
    for name in ("m.ubj", "m.json"):
        c = xgb.Booster(model_file=os.fspath(tmp_path / name))
        assert _canon(c.save_raw("json")) == text
    raw = b.save_raw("ubj")
    assert raw[:1] == b"{" and b"$" in raw  # typed numeric arrays
    d = xgb.Booster()
    d.load_model(raw)
    assert _canon(d.save_raw("json")) == text


def test_pickle_and_copy_keep_the_model():
    b = xgb.Booster()
    b.load_model(bytearray(json.dumps(_model("reg:squarederror", "2.5E-1")).encode()))
    text = _canon(b.save_raw("json"))
    assert _canon(pickle.loads(pickle.dumps(b)).save_raw("json")) == text
    assert _canon(b.copy().save_raw("json")) == text
    assert text["learner"]["learner_model_param"]["base_score"] == "[0.25]"


def test_multiclass_model_groups():
    trees = []
    for k in range(3):
        trees.append(_tree([-1], [-1], [2147483647], [0], [0.1 * (k + 1)], [0], [0], [1.0], [0.1]))
    doc = _model("multi:softprob", "[0,0,0]", trees, num_class="3")
    doc["learner"]["gradient_booster"]["model"]["tree_info"] = [0, 1, 2]
    doc["learner"]["gradient_booster"]["model"]["iteration_indptr"] = [0, 3]
    doc["learner"]["objective"] = {"name": "multi:softprob", "softmax_multiclass_param": {"num_class": "3"}}
    b = xgb.Booster()
    b.load_model(bytearray(json.dumps(doc).encode()))
    assert b.num_boosted_rounds() == 1
    out = _canon(b.save_raw("json"))
    assert out["learner"]["learner_model_param"]["num_class"] == "3"
    assert out["learner"]["gradient_booster"]["model"]["tree_info"] == [0, 1, 2]


@pytest.mark.parametrize("mutate,needle", [
    (lambda d: d["learner"]["gradient_booster"].__setitem__("name", "gblinear"), "gbtree"),
    (lambda d: d["learner"]["gradient_booster"]["model"]["trees"][0].update(
        left_children=[1, 0, -1], right_children=[2, 2, -1]), "cyclic"),
    (lambda d: d["learner"]["gradient_booster"]["model"]["trees"][0]["split_indices"].__setitem__(0, 7),
     "out-of-range"),
    (lambda d: d["learner"]["gradient_booster"]["model"]["trees"][0].__setitem__("split_type", [1, 0, 0]),
     "Categorical"),
    (lambda d: d["learner"]["gradient_booster"]["model"].__setitem__("tree_info", [0]), "tree_info"),
])
def test_invalid_models_are_rejected(mutate, needle):
    doc = _model()
    mutate(doc)
    b = xgb.Booster()
    with pytest.raises(xgb.XGBoostError, match=needle):
        b.load_model(bytearray(json.dumps(doc).encode()))


def test_training_without_a_gpu_still_fails_clearly():
    try:
        import torch
        if torch.cuda.is_available():
            pytest.skip("a GPU is present")
    except Exception:  # pragma: no cover
        pass
    b = xgb.Booster()
    b.load_model(bytearray(json.dumps(_model()).encode()))
    with pytest.raises(xgb.XGBoostError, match="CUDA"):
        b.predict(xgb.DMatrix(np.zeros((2, 3), np.float32)))


@pytest.mark.gpu
def test_trained_model_round_trips_through_files(tmp_path):
    """Train, save, load into a fresh booster: identical predictions, and
    continued training from the loaded model gives the same trees as
    training on without saving."""
    rng = np.random.default_rng(3)
    X = rng.normal(size=(5000, 6)).astype(np.float32)
    X[rng.random(X.shape) < 0.1] = np.nan
    y = (np.nan_to_num(X[:, 0]) + rng.normal(size=5000) * 0.3 > 0).astype(np.float32)
    d = xgb.DMatrix(X, label=y)
    params = {"objective": "binary:logistic", "tree_method": "hist", "device": "cuda", "max_depth": 4,
              "eta": 0.3, "max_bin": 64}
    b = xgb.train(params, d, 4)
    want = b.predict(xgb.DMatrix(X), output_margin=True)
    for name in ("m.json", "m.ubj"):
        b.save_model(os.fspath(tmp_path / name))
        c = xgb.Booster(params, model_file=os.fspath(tmp_path / name))
        np.testing.assert_array_equal(c.predict(xgb.DMatrix(X), output_margin=True), want)
    c = pickle.loads(pickle.dumps(b))
    np.testing.assert_array_equal(c.predict(xgb.DMatrix(X), output_margin=True), want)
    full = xgb.train(params, d, 6)
    resumed = xgb.Booster(params, model_file=os.fspath(tmp_path / "m.json"))
    for i in range(4, 6):
        resumed.update(d, i)
    np.testing.assert_array_equal(resumed.predict(xgb.DMatrix(X), output_margin=True),
                                  full.predict(xgb.DMatrix(X), output_margin=True))
    clf = xgb.XGBClassifier(n_estimators=3, max_depth=3, tree_method="hist", device="cuda").fit(X, y)
    clf.save_model(os.fspath(tmp_path / "clf.json"))
    clf2 = xgb.XGBClassifier()
    clf2.load_model(os.fspath(tmp_path / "clf.json"))
    np.testing.assert_array_equal(clf2.predict_proba(X), clf.predict_proba(X))
    assert list(clf2.classes_) == [0.0, 1.0]

"""Model inspection and booster management without a GPU: tree dumps
(text / JSON / dot, the reference's src/model.cpp:334-429), feature importance
(src/c_api.cpp:590-620), round slices (src/model.cpp:430-459), the training
configuration and its round trip (src/model.cpp:245-333), pickling through
XGBoosterSerializeToBuffer, and feature names kept by the native booster."""
import json
import pickle

import numpy as np
import pytest

import xgboost as xgb
from test_model_io import _model, _tree


def _booster(doc=None):
    b = xgb.Booster()
    b.load_model(bytearray(json.dumps(doc or _model()).encode()))
    return b


def _three_rounds():
    """Rounds 0 and 1 of the default model plus a round splitting f2 again."""
    doc = _model("reg:squarederror", "[0.5]")
    trees = doc["learner"]["gradient_booster"]["model"]["trees"]
    trees.append(_tree([1, -1, -1], [2, -1, -1], [2147483647, 0, 0], [2, 0, 0], [1.75, 0.5, -0.5],
                       [0, 0, 0], [1.5, 0, 0], [4.0, 1.0, 3.0], [0.0, 0.5, -0.5]))
    trees[-1]["id"] = 2
    model = doc["learner"]["gradient_booster"]["model"]
    model["tree_info"] = [0, 0, 0]
    model["iteration_indptr"] = [0, 1, 2, 3]
    model["gbtree_model_param"]["num_trees"] = "3"
    return doc


# -- dumps ------------------------------------------------------------------
def test_text_dump_matches_the_reference_layout():
    b = _booster()
    dump = b.get_dump()
    assert dump == [
        "0:[f2<0.25] yes=1,no=2,missing=1\n\t1:leaf=-0.125\n\t2:leaf=0.375\n",
        "0:[f0<-1.5] yes=1,no=2,missing=2\n\t1:[f1<2] yes=3,no=4,missing=3\n"
        "\t\t3:leaf=-0.25\n\t\t4:leaf=0.75\n\t2:leaf=0.5\n"]
    stats = b.get_dump(with_stats=True)
    assert stats[0] == ("0:[f2<0.25] yes=1,no=2,missing=1,gain=3.5,cover=10\n"
                        "\t1:leaf=-0.125,cover=4\n\t2:leaf=0.375,cover=6\n")


def test_text_dump_prints_nine_significant_digits():
    doc = _model()
    doc["learner"]["gradient_booster"]["model"]["trees"][0]["split_conditions"][0] = 0.1
    dump = _booster(doc).get_dump()[0]
    # float32(0.1) printed with setprecision(9)
    assert dump.startswith("0:[f2<0.100000001] ")


def test_json_dump_is_nested_with_sorted_keys():
    b = _booster()
    text = b.get_dump(dump_format="json")[0]
    assert text == """{
  "children": [
    {
      "leaf": -0.125,
      "nodeid": 1
    },
    {
      "leaf": 0.375,
      "nodeid": 2
    }
  ],
  "depth": 0,
  "missing": 1,
  "no": 2,
  "nodeid": 0,
  "split": "f2",
  "split_condition": 0.25,
  "yes": 1
}"""
    tree = json.loads(b.get_dump(dump_format="json", with_stats=True)[1])
    assert tree["gain"] == 1.0 and tree["cover"] == 10.0 and tree["depth"] == 0
    inner = tree["children"][0]
    assert inner["split"] == "f1" and inner["depth"] == 1 and inner["missing"] == 3
    assert [c["leaf"] for c in inner["children"]] == [-0.25, 0.75]
    assert inner["children"][0]["cover"] == 2.0


def test_json_dump_numbers_read_back_exactly():
    doc = _model()
    conds = [0.1, -3.0e-7, 12345678.0]
    doc["learner"]["gradient_booster"]["model"]["trees"][0]["split_conditions"] = conds
    tree = json.loads(_booster(doc).get_dump(dump_format="json")[0])
    # Each value is the binary64 image of the stored float32.
    assert tree["split_condition"] == float(np.float32(0.1))
    assert tree["children"][0]["leaf"] == float(np.float32(-3.0e-7))
    assert tree["children"][1]["leaf"] == 12345678.0


def test_dot_dump():
    dot = _booster().get_dump(dump_format="dot", with_stats=True)[0]
    assert dot == ('digraph {\n    graph [ rankdir=TB ]\n'
                   '    0 [ label="f2<0.25\\ncover=10" ]\n'
                   '    0 -> 1 [ label="yes, missing" ]\n'
                   '    0 -> 2 [ label="no" ]\n'
                   '    1 [ label="leaf=-0.125\\ncover=4" ]\n'
                   '    2 [ label="leaf=0.375\\ncover=6" ]\n}\n')


def test_dump_uses_feature_names_and_rejects_categorical_types(tmp_path):
    b = _booster()
    b.feature_names = ["age", "size", "x y"]
    assert b.get_dump()[0].startswith("0:[x y<0.25]")
    assert json.loads(b.get_dump(dump_format="json")[0])["split"] == "x y"
    b.feature_types = ["q", "q", "c"]
    with pytest.raises(xgb.XGBoostError, match="categorical"):
        b.get_dump()
    b.feature_types = None
    with pytest.raises(xgb.XGBoostError, match="Unknown dump format"):
        b.get_dump(dump_format="xml")
    with pytest.raises(xgb.XGBoostError, match="Feature-map"):
        b.get_dump(fmap=str(tmp_path / "fmap.txt"))
    path = tmp_path / "dump.txt"
    b.dump_model(str(path), with_stats=True)
    text = path.read_text()
    assert text.startswith("booster[0]:\n0:[x y<0.25]") and "booster[1]:\n" in text
    b.dump_model(str(tmp_path / "dump.json"), dump_format="json")
    assert len(json.loads((tmp_path / "dump.json").read_text())) == 2


# -- importance -----------------------------------------------------------------
def test_feature_scores_count_and_average_splits():
    b = _booster(_three_rounds())
    assert b.get_score(importance_type="weight") == {"f0": 1.0, "f1": 1.0, "f2": 2.0}
    assert b.get_fscore() == b.get_score()
    assert b.get_score(importance_type="gain") == {"f0": 1.0, "f1": 0.5, "f2": 2.5}
    assert b.get_score(importance_type="total_gain") == {"f0": 1.0, "f1": 0.5, "f2": 5.0}
    assert b.get_score(importance_type="cover") == {"f0": 10.0, "f1": 7.0, "f2": 7.0}
    assert b.get_score(importance_type="total_cover") == {"f0": 10.0, "f1": 7.0, "f2": 14.0}
    with pytest.raises(xgb.XGBoostError, match="importance"):
        b.get_score(importance_type="shap")


def test_feature_scores_skip_unused_features_and_use_names():
    doc = _model()
    doc["learner"]["gradient_booster"]["model"]["trees"] = \
        doc["learner"]["gradient_booster"]["model"]["trees"][:1]
    doc["learner"]["gradient_booster"]["model"]["tree_info"] = [0]
    doc["learner"]["gradient_booster"]["model"]["iteration_indptr"] = [0, 1]
    doc["learner"]["feature_names"] = ["a", "b", "c"]
    b = _booster(doc)
    assert b.feature_names == ["a", "b", "c"]
    assert b.get_score() == {"c": 1.0}


# -- slices ---------------------------------------------------------------------
def _trees(b):
    return json.loads(bytes(b.save_raw("json")).decode())["learner"]["gradient_booster"]["model"]


def test_slices_select_rounds_and_drop_best_iteration():
    b = _booster(_three_rounds())
    b.set_attr(keep="yes")
    full = _trees(b)["trees"]
    for sel, rounds in ((0, [0]), (slice(1, None), [1, 2]), (slice(0, 3, 2), [0, 2]),
                        (slice(None, 2), [0, 1]), (Ellipsis, [0, 1, 2])):
        s = b[sel]
        assert s.num_boosted_rounds() == len(rounds)
        got = _trees(s)
        assert [t["id"] for t in got["trees"]] == list(range(len(rounds)))
        for t, r in zip(got["trees"], rounds):
            assert t["split_conditions"] == full[r]["split_conditions"]
            assert t["left_children"] == full[r]["left_children"]
        assert got["iteration_indptr"] == list(range(len(rounds) + 1))
        assert s.attr("best_iteration") is None and s.attr("keep") == "yes"
    assert [t.num_boosted_rounds() for t in b] == [1, 1, 1]
    with pytest.raises(IndexError):
        b[5]
    with pytest.raises(IndexError):
        b[1:7]
    with pytest.raises(ValueError):
        b[2:1]
    with pytest.raises(xgb.XGBoostError, match="Invalid model slice"):
        b[0:2:0]


def test_multiclass_slice_keeps_every_class_tree():
    trees = [_tree([-1], [-1], [2147483647], [0], [0.1 * (k + 1)], [0], [0], [1.0], [0.1])
             for k in range(6)]
    doc = _model("multi:softprob", "[0,0,0]", trees, num_class="3")
    doc["learner"]["gradient_booster"]["model"]["tree_info"] = [0, 1, 2, 0, 1, 2]
    doc["learner"]["gradient_booster"]["model"]["iteration_indptr"] = [0, 3, 6]
    doc["learner"]["objective"] = {"name": "multi:softprob",
                                   "softmax_multiclass_param": {"num_class": "3"}}
    s = _booster(doc)[1]
    model = _trees(s)
    assert model["tree_info"] == [0, 1, 2]
    assert [t["split_conditions"][0] for t in model["trees"]] == pytest.approx([0.4, 0.5, 0.6])


# -- configuration and pickling -------------------------------------------------
def test_config_has_the_upstream_layout_and_round_trips():
    b = _booster()
    b.set_param({"max_depth": 8, "eta": 0.1, "lambda": 2, "max_bin": 64, "nthread": 3})
    cfg = json.loads(b.save_config())
    learner = cfg["learner"]
    assert learner["learner_train_param"]["objective"] == "binary:logistic"
    assert learner["learner_train_param"]["booster"] == "gbtree"
    ttp = learner["gradient_booster"]["tree_train_param"]
    assert ttp["max_depth"] == "8" and ttp["eta"] == "0.1" and ttp["learning_rate"] == "0.1"
    assert ttp["reg_lambda"] == "2" and ttp["lambda"] == "2" and ttp["max_bin"] == "64"
    assert learner["generic_param"]["nthread"] == "3"
    assert learner["gradient_booster"]["gbtree_train_param"]["tree_method"] == "hist"
    assert learner["learner_model_param"]["num_feature"] == "3"
    assert learner["objective"]["name"] == "binary:logistic"
    assert cfg["version"] == [3, 5, 0]
    c = _booster()
    c.load_config(b.save_config())
    assert json.loads(c.save_config()) == cfg


def test_load_config_rejects_other_boosters():
    cfg = json.loads(_booster().save_config())
    cfg["learner"]["gradient_booster"]["name"] = "gblinear"
    with pytest.raises(xgb.XGBoostError, match="gbtree"):
        _booster().load_config(json.dumps(cfg))


def test_pickle_keeps_model_parameters_and_names():
    b = _booster()
    b.set_param({"max_depth": 4, "eta": 0.05})
    b.feature_names = ["a", "b", "c"]
    c = pickle.loads(pickle.dumps(b))
    assert bytes(c.save_raw("json")) == bytes(b.save_raw("json"))
    assert json.loads(c.save_config()) == json.loads(b.save_config())
    assert c.feature_names == ["a", "b", "c"]
    assert c.reset() is c


def test_feature_info_is_validated():
    b = _booster()
    with pytest.raises(xgb.XGBoostError, match="length"):
        b.feature_names = ["a", "b"]
    with pytest.raises(xgb.XGBoostError, match="Invalid feature type"):
        b.feature_types = ["q", "q", "z"]
    b.feature_types = ["int", "float", "q"]
    assert b.feature_types == ["int", "float", "q"]
    b.feature_names = None
    assert b.feature_names is None


def test_trees_to_dataframe():
    pytest.importorskip("pandas")
    b = _booster()
    b.feature_names = ["a", "b", "c"]
    df = b.trees_to_dataframe()
    assert list(df.columns) == ["Tree", "Target", "Node", "ID", "Feature", "Split", "Yes", "No",
                                "Missing", "Gain", "Cover", "Category"]
    assert len(df) == 8
    root = df.iloc[0]
    assert (root["Tree"], root["Node"], root["Feature"], root["Split"]) == (0, 0, "c", 0.25)
    assert (root["Yes"], root["No"], root["Missing"], root["Gain"]) == ("0-1", "0-2", "0-1", 3.5)
    leaf = df[(df["Tree"] == 1) & (df["Node"] == 4)].iloc[0]
    assert leaf["Feature"] == "Leaf" and leaf["Gain"] == 0.75 and leaf["Cover"] == 5.0


def test_sklearn_feature_importances(tmp_path):
    b = _booster(_three_rounds())
    path = str(tmp_path / "m.json")
    b.save_model(path)
    reg = xgb.XGBRegressor()
    reg.load_model(path)
    reg.n_features_in_ = 3
    imp = reg.feature_importances_
    np.testing.assert_allclose(imp, np.array([1.0, 0.5, 2.5]) / 4.0, rtol=1e-6)


def test_custom_gradients_are_checked_before_any_device_work():
    from xgboost import core
    b = _booster(_model("reg:squarederror", "[0.5]"))
    d = xgb.DMatrix(np.zeros((4, 3), np.float32), label=np.zeros(4, np.float32))
    with pytest.raises(ValueError, match="shape mismatch"):
        b.boost(d, 0, np.zeros(4), np.zeros(3))
    with pytest.raises(xgb.XGBoostError, match="one row per training sample"):
        b.boost(d, 0, np.zeros(5), np.ones(5))
    with pytest.raises(xgb.XGBoostError, match="shape"):
        b.boost(d, 0, np.zeros((4, 2)), np.ones((4, 2)))
    with pytest.raises(xgb.XGBoostError, match="finite"):
        b.boost(d, 0, np.array([0, np.nan, 0, 0]), np.ones(4))
    with pytest.raises(xgb.XGBoostError, match="finite"):
        b.boost(d, 0, np.zeros(4), np.array([1, 1, np.inf, 1]))
    g = np.zeros(3, np.float32)
    assert core._LIB.XGBoosterBoostOneIter(
        b.handle, d.handle, g.ctypes.data_as(core.ctypes.POINTER(core.ctypes.c_float)),
        g.ctypes.data_as(core.ctypes.POINTER(core.ctypes.c_float)), core.c_bst_ulong(3)) == -1
    assert b"shape" in core._LIB.XGBGetLastError()


def test_concurrent_calls_on_one_booster_are_serialised():
    """Every C call holds the booster's lock (the reference's per-booster
    mutex): threads mutating attributes while others save and dump never see
    a torn model."""
    import threading
    b = _booster(_three_rounds())
    want = b.get_dump()
    errors = []

    def writer(k):
        try:
            for i in range(200):
                b.set_attr(**{"k%d" % k: str(i)})
                b.set_param("max_depth", 3 + (i % 3))
        except Exception as e:  # noqa: BLE001
            errors.append(e)

    def reader():
        try:
            for _ in range(100):
                assert b.get_dump() == want
                doc = json.loads(bytes(b.save_raw("json")).decode())
                assert len(doc["learner"]["gradient_booster"]["model"]["trees"]) == 3
                json.loads(b.save_config())
        except Exception as e:  # noqa: BLE001
            errors.append(e)

    threads = [threading.Thread(target=writer, args=(k,)) for k in range(3)]
    threads += [threading.Thread(target=reader) for _ in range(3)]
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    assert not errors
    assert b.attr("k2") == "199"


def test_device_strings_are_validated():
    b = _booster()
    for good in ("cuda", "gpu", "cuda:0"):
        b.set_param("device", good)
        json.loads(b.save_config())
    for bad, needle in (("cuda:x", "ordinal"), ("cpu", "CUDA devices only"), ("cuda:-1", "ordinal")):
        b.set_param("device", bad)
        with pytest.raises(xgb.XGBoostError, match=needle):
            b.save_config()

"""The package surface of the reference's python-package/xgboost/__init__.py
(no GPU): global configuration through the library, and the entry points
that exist for import compatibility with explicit errors."""
import pytest

import xgboost as xgb


def test_global_config_round_trip_and_context():
    assert xgb.get_config() == {"nthread": 0, "use_rmm": False, "verbosity": 1}
    with xgb.config_context(verbosity=0, nthread=4):
        assert xgb.get_config()["verbosity"] == 0 and xgb.get_config()["nthread"] == 4
    assert xgb.get_config() == {"nthread": 0, "use_rmm": False, "verbosity": 1}
    xgb.set_config(verbosity=2, nthread=None)
    assert xgb.get_config()["verbosity"] == 2
    xgb.set_config(verbosity=1)
    for bad, needle in (({"verbosity": 4}, "verbosity"), ({"use_rmm": True}, "RMM"),
                        ({"colour": 1}, "Unknown global parameter")):
        with pytest.raises(xgb.XGBoostError, match=needle):
            xgb.set_config(**bad)


def test_reference_package_names_exist():
    import xgboost
    for name in ("DMatrix", "QuantileDMatrix", "ExtMemQuantileDMatrix", "Booster", "DataIter", "train",
                 "cv", "build_info", "plot_importance", "plot_tree", "to_graphviz", "set_config",
                 "get_config", "config_context", "XGBModel", "XGBClassifier", "XGBRegressor",
                 "XGBRanker", "XGBRFClassifier", "XGBRFRegressor", "collective"):
        assert hasattr(xgboost, name), name
    with pytest.raises(xgb.XGBoostError, match="Ranking"):
        xgb.XGBRanker().fit([[0.0]], [0.0])
    with pytest.raises(xgb.XGBoostError, match="Random forests"):
        xgb.XGBRFRegressor().fit([[0.0]], [0.0])
    with pytest.raises(TypeError):
        xgb.ExtMemQuantileDMatrix([[1.0]])


def test_dataframe_names_flow_into_matrices_slices_and_boosters():
    pd = pytest.importorskip("pandas")
    import numpy as np
    df = pd.DataFrame({"age": [1.0, 2.0, np.nan], "size": [3.0, 4.0, 5.0]})
    d = xgb.DMatrix(df, label=[0.0, 1.0, 0.0])
    assert d.feature_names == ["age", "size"]
    assert d.slice([2, 0]).feature_names == ["age", "size"]
    b = xgb.Booster({}, [d])
    assert b.feature_names == ["age", "size"]
    d.feature_types = "q"
    assert d.feature_types == ["q", "q"]
    with pytest.raises(ValueError, match="unique"):
        d.feature_names = ["a", "a"]
    d.feature_names = None
    assert d.feature_names is None
    csr = d.get_data()
    assert csr.shape == (3, 2) and csr.nnz == 5


def test_feature_validation_and_split_value_histogram():
    import json

    import numpy as np
    from test_model_io import _model
    b = xgb.Booster()
    b.load_model(bytearray(json.dumps(_model()).encode()))
    b.feature_names = ["a", "b", "c"]
    d = xgb.DMatrix(np.zeros((2, 3), np.float32), feature_names=["a", "x", "c"])
    with pytest.raises(ValueError, match="feature_names mismatch"):
        b.predict(d)
    with pytest.raises(ValueError, match="did not contain feature names"):
        b.predict(xgb.DMatrix(np.zeros((2, 3), np.float32)))
    # One threshold per feature: numpy's single bin spans value +- 0.5, and
    # rows carry each bin's right edge.
    assert b.get_split_value_histogram("c", as_pandas=False).tolist() == [[0.75, 1.0]]
    assert b.get_split_value_histogram("a", as_pandas=False).tolist() == [[-1.0, 1.0]]


def test_estimators_are_scikit_learn_estimators():
    base = pytest.importorskip("sklearn.base")
    r = xgb.XGBRegressor(max_depth=3, learning_rate=0.1, eval_metric="mae")
    c = base.clone(r)
    assert c.get_params()["max_depth"] == 3 and c.get_params()["eval_metric"] == "mae"
    assert base.is_regressor(r) and base.is_classifier(xgb.XGBClassifier())
    assert c.set_params(max_depth=5).max_depth == 5
    assert "XGBRegressor(" in repr(r)


def test_dmatrix_from_text_files(tmp_path):
    import numpy as np
    p = tmp_path / "d.csv"
    p.write_text("0,1.5,2\n1,,3\n")
    d = xgb.DMatrix(str(p) + "?format=csv&label_column=0")
    assert (d.num_row(), d.num_col()) == (2, 2)
    np.testing.assert_array_equal(d.get_label(), [0, 1])
    s = tmp_path / "d.svm"
    s.write_text("1 0:1 2:3\n0 1:2\n")
    d = xgb.DMatrix(str(s) + "?format=libsvm", feature_names=["a", "b", "c"])
    assert d.feature_names == ["a", "b", "c"] and d.num_nonmissing() == 3

"""B200-native XGBoost: histogram tree training (tree_method="hist",
device="cuda") on hand-written sm_100a CUDA kernels, behind the upstream
XGBoost Python API and C ABI."""
from . import callback, collective
from .config import config_context, get_config, set_config
from .core import (Booster, DataIter, DMatrix, ExtMemQuantileDMatrix, QuantileDMatrix, XGBoostError,
                   build_info, synchronize)
from .plotting import plot_importance, plot_tree, to_graphviz
from .sklearn import XGBClassifier, XGBModel, XGBRanker, XGBRegressor, XGBRFClassifier, XGBRFRegressor
from .training import cv, train

__version__ = "3.5.0-dev"

__all__ = ["Booster", "DataIter", "DMatrix", "QuantileDMatrix", "ExtMemQuantileDMatrix", "XGBoostError",
           "XGBModel", "XGBRegressor", "XGBClassifier", "XGBRanker", "XGBRFRegressor", "XGBRFClassifier",
           "train", "cv", "build_info", "callback", "collective", "synchronize", "set_config", "get_config",
           "config_context", "plot_importance", "plot_tree", "to_graphviz"]

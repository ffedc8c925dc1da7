"""B200-native XGBoost: histogram tree training (tree_method="hist",
device="cuda") on hand-written sm_100a CUDA kernels, behind the upstream
XGBoost Python API and C ABI."""
from . import callback, collective
from .core import Booster, DataIter, DMatrix, QuantileDMatrix, XGBoostError, build_info, synchronize
from .sklearn import XGBClassifier, XGBModel, XGBRegressor
from .training import cv, train

__version__ = "3.5.0-dev"

__all__ = ["Booster", "DataIter", "DMatrix", "QuantileDMatrix", "XGBoostError", "XGBModel", "XGBRegressor",
           "XGBClassifier", "train", "cv", "build_info", "callback", "collective", "synchronize"]

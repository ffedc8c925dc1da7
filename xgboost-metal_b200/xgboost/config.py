"""Global configuration (python-package/xgboost/config.py in the reference):
verbosity, use_rmm and nthread, kept per thread by the library
(XGBSetGlobalConfig / XGBGetGlobalConfig)."""
import ctypes
import json
from contextlib import contextmanager

from .core import _LIB, _c_str, _check_call

__all__ = ["set_config", "get_config", "config_context"]


def set_config(**new_config):
    """Sets global parameters; None values are ignored."""
    config = {k: v for k, v in new_config.items() if v is not None}
    _check_call(_LIB.XGBSetGlobalConfig(_c_str(json.dumps(config))))


def get_config():
    out = ctypes.c_char_p()
    _check_call(_LIB.XGBGetGlobalConfig(ctypes.byref(out)))
    return json.loads(out.value.decode())


@contextmanager
def config_context(**new_config):
    """Sets parameters for the duration of a with block; every parameter
    returns to its previous value afterwards."""
    old = get_config().copy()
    set_config(**new_config)
    try:
        yield
    finally:
        set_config(**old)

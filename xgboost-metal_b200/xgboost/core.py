"""ctypes front end over libxgboost.so (the CUDA trainer).

The public classes keep the names, arguments and error behaviour of the
upstream XGBoost Python package (python-package/xgboost/core.py in the
reference): DMatrix, QuantileDMatrix, Booster and XGBoostError, with
device="cuda". The library is loaded from xgboost/lib/ as upstream's
libpath.find_lib_path does (python-package/xgboost/libpath.py:27-58).
"""
import ctypes
import json
import os

import numpy as np

__all__ = ["DMatrix", "QuantileDMatrix", "Booster", "XGBoostError", "build_info"]


class XGBoostError(ValueError):
    """Error raised by the native library (python-package/xgboost/_c_api.py:181-184)."""


def _lib_path():
    here = os.path.dirname(os.path.abspath(__file__))
    path = os.path.join(here, "lib", "libxgboost.so")
    if not os.path.exists(path):
        raise XGBoostError(
            "libxgboost.so not found at %s; build it with xgboost-metal_b200/build.py" % path)
    return path


def _load_lib():
    lib = ctypes.CDLL(_lib_path())
    lib.XGBGetLastError.restype = ctypes.c_char_p
    return lib


_LIB = _load_lib()

c_bst_ulong = ctypes.c_uint64


def _check_call(ret):
    if ret != 0:
        raise XGBoostError(_LIB.XGBGetLastError().decode())


def _c_str(s):
    return ctypes.c_char_p(s.encode())


def build_info():
    out = ctypes.c_char_p()
    _check_call(_LIB.XGBuildInfo(ctypes.byref(out)))
    return json.loads(out.value.decode())


def _array_interface(arr):
    arr = np.asarray(arr)
    inf = arr.__array_interface__
    desc = {"data": [int(inf["data"][0]), True], "shape": list(inf["shape"]),
            "strides": None if inf["strides"] is None else list(inf["strides"]),
            "typestr": inf["typestr"], "version": 3}
    return json.dumps(desc)


def _is_scipy_csr(data):
    return type(data).__name__ in ("csr_matrix", "csr_array")


def _to_2d_float(data):
    if hasattr(data, "to_numpy"):  # pandas
        data = data.to_numpy(dtype=np.float32, na_value=np.nan)
    if hasattr(data, "toarray") and not _is_scipy_csr(data):
        data = data.toarray()
    arr = np.asarray(data)
    if arr.ndim == 1:
        arr = arr.reshape(-1, 1)
    if arr.ndim != 2:
        raise XGBoostError("Data must be 2-dimensional.")
    if arr.dtype.kind not in "fiub":
        arr = arr.astype(np.float32)
    return arr


class DMatrix:
    """Data matrix (python-package/xgboost/core.py DMatrix). Quantisation is
    lazy: it happens on the first training round, as in the reference."""

    def __init__(self, data, label=None, *, weight=None, base_margin=None, missing=None,
                 silent=False, feature_names=None, feature_types=None, nthread=None,
                 group=None, qid=None, label_lower_bound=None, label_upper_bound=None,
                 feature_weights=None, enable_categorical=False, data_split_mode=None):
        if group is not None or qid is not None:
            raise XGBoostError("Ranking groups are not implemented by the CUDA backend.")
        self.handle = ctypes.c_void_p()
        miss = np.nan if missing is None else float(missing)
        config = {"missing": None if np.isnan(miss) else miss, "nthread": nthread or 0}
        if _is_scipy_csr(data):
            csr = data
            _check_call(_LIB.XGDMatrixCreateFromCSR(
                _c_str(_array_interface(csr.indptr)), _c_str(_array_interface(csr.indices)),
                _c_str(_array_interface(np.asarray(csr.data, dtype=np.float32))),
                c_bst_ulong(csr.shape[1]), _c_str(json.dumps(config)), ctypes.byref(self.handle)))
        else:
            arr = _to_2d_float(data)
            # A C-contiguous float32 array with NaN as the missing value is
            # read in place (no host copy); this object keeps it alive. It must
            # not be modified while the DMatrix exists.
            if arr.dtype == np.float32 and arr.flags.c_contiguous and np.isnan(miss):
                config["zero_copy"] = True
                self._data_ref = arr
            _check_call(_LIB.XGDMatrixCreateFromDense(
                _c_str(_array_interface(arr)), _c_str(json.dumps(config)), ctypes.byref(self.handle)))
        self.feature_names = list(feature_names) if feature_names is not None else (
            [str(c) for c in data.columns] if hasattr(data, "columns") else None)
        self.feature_types = feature_types
        if label is not None:
            self.set_label(label)
        if weight is not None:
            self.set_weight(weight)
        if base_margin is not None:
            self.set_base_margin(base_margin)

    def __del__(self):
        # At interpreter exit the module globals may already be gone.
        if _LIB is not None and getattr(self, "handle", None) is not None and self.handle.value:
            _LIB.XGDMatrixFree(self.handle)
            self.handle = None

    def _set_float(self, field, values):
        v = np.ascontiguousarray(np.asarray(values, dtype=np.float32).reshape(-1))
        _check_call(_LIB.XGDMatrixSetInfoFromInterface(
            self.handle, _c_str(field), _c_str(_array_interface(v))))

    def set_label(self, label):
        self._set_float("label", label)

    def set_weight(self, weight):
        self._set_float("weight", weight)

    def set_base_margin(self, margin):
        self._set_float("base_margin", margin)

    def set_float_info(self, field, data):
        self._set_float(field, data)

    def get_float_info(self, field):
        length = c_bst_ulong()
        ptr = ctypes.POINTER(ctypes.c_float)()
        _check_call(_LIB.XGDMatrixGetFloatInfo(self.handle, _c_str(field), ctypes.byref(length),
                                               ctypes.byref(ptr)))
        return np.ctypeslib.as_array(ptr, shape=(length.value,)).copy() if length.value else \
            np.zeros(0, np.float32)

    def get_label(self):
        return self.get_float_info("label")

    def get_weight(self):
        return self.get_float_info("weight")

    def num_row(self):
        out = c_bst_ulong()
        _check_call(_LIB.XGDMatrixNumRow(self.handle, ctypes.byref(out)))
        return out.value

    def num_col(self):
        out = c_bst_ulong()
        _check_call(_LIB.XGDMatrixNumCol(self.handle, ctypes.byref(out)))
        return out.value

    def num_nonmissing(self):
        out = c_bst_ulong()
        _check_call(_LIB.XGDMatrixNumNonMissing(self.handle, ctypes.byref(out)))
        return out.value


class QuantileDMatrix(DMatrix):
    """A DMatrix quantised at construction (python-package/xgboost/core.py
    QuantileDMatrix): its cuts come from `ref` when given, so a validation or
    sharded matrix shares the training matrix's bins."""

    def __init__(self, data, label=None, *, weight=None, base_margin=None, missing=None,
                 silent=False, feature_names=None, feature_types=None, nthread=None,
                 max_bin=None, ref=None, group=None, qid=None, label_lower_bound=None,
                 label_upper_bound=None, feature_weights=None, enable_categorical=False,
                 max_quantile_batches=None, data_split_mode=None):
        super().__init__(data, label, weight=weight, base_margin=base_margin, missing=missing,
                         feature_names=feature_names, feature_types=feature_types, nthread=nthread,
                         group=group, qid=qid)
        self.max_bin = 256 if max_bin is None else int(max_bin)
        _check_call(_LIB.XGDMatrixQuantise(self.handle, ctypes.c_int(self.max_bin),
                                           ref.handle if ref is not None else None))


class Booster:
    """A gradient-boosted tree model trained on the GPU
    (python-package/xgboost/core.py Booster)."""

    def __init__(self, params=None, cache=None, model_file=None):
        cache = list(cache or [])
        arr = (ctypes.c_void_p * len(cache))(*[d.handle for d in cache])
        self.handle = ctypes.c_void_p()
        _check_call(_LIB.XGBoosterCreate(arr, c_bst_ulong(len(cache)), ctypes.byref(self.handle)))
        self._cache = cache
        self.feature_names = cache[0].feature_names if cache else None
        self.feature_types = None
        params = params or {}
        if isinstance(params, dict):
            items = list(params.items())
        else:
            items = list(params)
        for k, v in items:
            if k == "eval_metric":
                continue
            self.set_param(k, v)
        if model_file is not None:
            self.load_model(model_file)

    def __del__(self):
        if _LIB is not None and getattr(self, "handle", None) is not None and self.handle.value:
            _LIB.XGBoosterFree(self.handle)
            self.handle = None

    def set_param(self, params, value=None):
        if isinstance(params, dict):
            items = params.items()
        elif isinstance(params, str):
            items = [(params, value)]
        else:
            items = params
        for k, v in items:
            if v is None:
                continue
            if isinstance(v, bool):
                v = int(v)
            _check_call(_LIB.XGBoosterSetParam(self.handle, _c_str(str(k)), _c_str(str(v))))

    def update(self, dtrain, iteration, fobj=None):
        if fobj is not None:
            raise XGBoostError("Custom objectives are not implemented by the CUDA backend yet.")
        _check_call(_LIB.XGBoosterUpdateOneIter(self.handle, ctypes.c_int(iteration), dtrain.handle))

    def num_boosted_rounds(self):
        out = ctypes.c_int()
        _check_call(_LIB.XGBoosterBoostedRounds(self.handle, ctypes.byref(out)))
        return out.value

    def num_features(self):
        out = c_bst_ulong()
        _check_call(_LIB.XGBoosterGetNumFeature(self.handle, ctypes.byref(out)))
        return out.value

    def predict(self, data, output_margin=False, pred_leaf=False, pred_contribs=False,
                approx_contribs=False, pred_interactions=False, validate_features=True,
                training=False, iteration_range=(0, 0), strict_shape=False):
        if pred_leaf or pred_contribs or pred_interactions:
            raise XGBoostError("Leaf and contribution predictions are not implemented by the CUDA backend.")
        config = json.dumps({"type": 1 if output_margin else 0, "training": bool(training),
                             "iteration_begin": int(iteration_range[0]),
                             "iteration_end": int(iteration_range[1]),
                             "strict_shape": bool(strict_shape)})
        shape = ctypes.POINTER(c_bst_ulong)()
        dims = c_bst_ulong()
        result = ctypes.POINTER(ctypes.c_float)()
        _check_call(_LIB.XGBoosterPredictFromDMatrix(
            self.handle, data.handle, _c_str(config), ctypes.byref(shape), ctypes.byref(dims),
            ctypes.byref(result)))
        dims_list = [shape[i] for i in range(dims.value)]
        n = int(np.prod(dims_list)) if dims_list else 0
        if n == 0:
            return np.zeros(dims_list, np.float32)
        return np.ctypeslib.as_array(result, shape=(n,)).copy().reshape(dims_list)

    def inplace_predict(self, data, iteration_range=(0, 0), predict_type="value", missing=np.nan,
                        validate_features=True, base_margin=None, strict_shape=False):
        dm = DMatrix(data, missing=missing, base_margin=base_margin)
        return self.predict(dm, output_margin=predict_type == "margin",
                            iteration_range=iteration_range, strict_shape=strict_shape)

    def attr(self, key):
        out = ctypes.c_char_p()
        success = ctypes.c_int()
        _check_call(_LIB.XGBoosterGetAttr(self.handle, _c_str(key), ctypes.byref(out),
                                          ctypes.byref(success)))
        return out.value.decode() if success.value else None

    def set_attr(self, **kwargs):
        for k, v in kwargs.items():
            _check_call(_LIB.XGBoosterSetAttr(self.handle, _c_str(k),
                                              None if v is None else _c_str(str(v))))

    def attributes(self):
        length = c_bst_ulong()
        names = ctypes.POINTER(ctypes.c_char_p)()
        _check_call(_LIB.XGBoosterGetAttrNames(self.handle, ctypes.byref(length), ctypes.byref(names)))
        keys = [names[i].decode() for i in range(length.value)]
        return {k: self.attr(k) for k in keys}

    def save_config(self):
        length = c_bst_ulong()
        out = ctypes.c_char_p()
        _check_call(_LIB.XGBoosterSaveJsonConfig(self.handle, ctypes.byref(length), ctypes.byref(out)))
        return out.value.decode()

    def cuda_profile(self):
        """Device timings of the histogram kernels (set cuda_profile=1)."""
        out = ctypes.c_char_p()
        _check_call(_LIB.XGBoosterGetCudaProfile(self.handle, ctypes.byref(out)))
        return json.loads(out.value.decode())

    def reset_cuda_profile(self):
        _check_call(_LIB.XGBoosterResetCudaProfile(self.handle))

    def record_event(self, slot):
        """Records CUDA event `slot` on the booster's stream (device timing)."""
        _check_call(_LIB.XGBoosterRecordEvent(self.handle, ctypes.c_int(int(slot))))

    def event_elapsed(self, a, b):
        """Device milliseconds between two recorded events."""
        ms = ctypes.c_float()
        _check_call(_LIB.XGBoosterEventElapsed(self.handle, ctypes.c_int(a), ctypes.c_int(b),
                                               ctypes.byref(ms)))
        return ms.value

    # -- model files (python-package/xgboost/core.py save_model / load_model /
    # save_raw in the reference): upstream XGBoost's JSON schema, as text or
    # as Universal Binary JSON.
    def save_model(self, fname):
        """Saves the model: JSON when the file name ends in ".json", else UBJSON."""
        _check_call(_LIB.XGBoosterSaveModel(self.handle, _c_str(os.fspath(fname))))

    def save_raw(self, raw_format="ubj"):
        """The model as bytes ("json" or "ubj")."""
        length = c_bst_ulong()
        out = ctypes.c_char_p()
        _check_call(_LIB.XGBoosterSaveModelToBuffer(
            self.handle, _c_str(json.dumps({"format": raw_format})), ctypes.byref(length),
            ctypes.byref(out)))
        return bytearray(ctypes.string_at(out, length.value))

    def load_model(self, fname):
        """Loads a model from a file name or from the bytes of save_raw."""
        if isinstance(fname, (bytes, bytearray, memoryview)):
            buf = bytes(fname)
            _check_call(_LIB.XGBoosterLoadModelFromBuffer(self.handle, ctypes.c_char_p(buf),
                                                          c_bst_ulong(len(buf))))
        else:
            _check_call(_LIB.XGBoosterLoadModel(self.handle, _c_str(os.fspath(fname))))

    def __getstate__(self):
        return {"raw": bytes(self.save_raw("ubj")), "feature_names": self.feature_names,
                "feature_types": self.feature_types}

    def __setstate__(self, state):
        self.handle = ctypes.c_void_p()
        _check_call(_LIB.XGBoosterCreate(None, c_bst_ulong(0), ctypes.byref(self.handle)))
        self._cache = []
        self.feature_names = state.get("feature_names")
        self.feature_types = state.get("feature_types")
        self.load_model(state["raw"])

    def copy(self):
        return Booster(model_file=self.save_raw("ubj"))

    def __copy__(self):
        return self.copy()

    def __deepcopy__(self, memo):
        return self.copy()


def synchronize():
    """Waits for all work on the current device (used by timing code)."""
    _check_call(_LIB.XGBBSynchronize())


def set_device(ordinal):
    _check_call(_LIB.XGBBSetDevice(ctypes.c_int(int(ordinal))))

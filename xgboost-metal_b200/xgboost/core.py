"""ctypes front end over libxgboost.so (the CUDA trainer).

The public classes keep the names, arguments and error behaviour of the
upstream XGBoost Python package (python-package/xgboost/core.py in the
reference): DMatrix, QuantileDMatrix, Booster and XGBoostError, with
device="cuda". The library is loaded from xgboost/lib/ as upstream's
libpath.find_lib_path does (python-package/xgboost/libpath.py:27-58).
"""
import ctypes
import json
import math
import os

import numpy as np

__all__ = ["DMatrix", "QuantileDMatrix", "ExtMemQuantileDMatrix", "DataIter", "Booster", "XGBoostError",
           "build_info"]


class XGBoostError(ValueError):
    """Error raised by the native library (python-package/xgboost/_c_api.py:181-184)."""


def _lib_path():
    here = os.path.dirname(os.path.abspath(__file__))
    path = os.path.join(here, "lib", "libxgboost.so")
    if not os.path.exists(path):
        raise XGBoostError(
            "libxgboost.so not found at %s; build it with xgboost-metal_b200/build.py" % path)
    return path


_VERSION = (3, 5, 0)
_LOG_CALLBACK = ctypes.CFUNCTYPE(None, ctypes.c_char_p)


def _log(msg):
    print(msg.decode("utf-8", "replace"), flush=True)


def _load_lib():
    """Loads the library, routes its log messages to stdout and checks that
    it is the version this package belongs to (python-package/xgboost/
    _c_api.py:90-174 in the reference)."""
    lib = ctypes.CDLL(_lib_path())
    lib.XGBGetLastError.restype = ctypes.c_char_p
    lib.callback = _LOG_CALLBACK(_log)
    if lib.XGBRegisterLogCallback(lib.callback) != 0:
        raise XGBoostError(lib.XGBGetLastError().decode("utf-8", "replace"))
    major, minor, patch = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
    lib.XGBoostVersion(ctypes.byref(major), ctypes.byref(minor), ctypes.byref(patch))
    libver = (major.value, minor.value, patch.value)
    if libver != _VERSION:
        raise ValueError("Mismatched version between the Python package (%s) and the native shared object "
                         "(%s) loaded from %s." % (".".join(map(str, _VERSION)), ".".join(map(str, libver)),
                                                   _lib_path()))
    return lib


_LIB = _load_lib()

c_bst_ulong = ctypes.c_uint64


def _check_call(ret):
    if ret != 0:
        raise XGBoostError(_LIB.XGBGetLastError().decode("utf-8", "replace"))


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


def _set_str_info(fn, handle, field, values):
    """Feature names or types through Set*StrFeatureInfo (None clears them)."""
    if values is None:
        _check_call(fn(handle, _c_str(field), None, c_bst_ulong(0)))
        return
    values = [str(v) for v in values]
    arr = (ctypes.c_char_p * len(values))(*[v.encode() for v in values])
    _check_call(fn(handle, _c_str(field), arr, c_bst_ulong(len(values))))


def _get_str_info(fn, handle, field):
    length = c_bst_ulong()
    sarr = ctypes.POINTER(ctypes.c_char_p)()
    _check_call(fn(handle, _c_str(field), ctypes.byref(length), ctypes.byref(sarr)))
    values = [sarr[i].decode() for i in range(length.value)]
    return values if values else None


_NEXT_CALLBACK = ctypes.CFUNCTYPE(ctypes.c_int, ctypes.c_void_p)
_RESET_CALLBACK = ctypes.CFUNCTYPE(None, ctypes.c_void_p)


class DataIter:
    """Batches for DMatrix / QuantileDMatrix (python-package/xgboost/core.py
    DataIter): subclasses define reset() and next(input_data), where next
    calls input_data(data=..., label=..., weight=..., base_margin=...) once
    per batch and returns False after the last one. The batches are
    concatenated on the host before quantisation."""

    def __init__(self, cache_prefix=None, release_data=True, *, on_host=True,
                 min_cache_page_bytes=None):
        self.cache_prefix = cache_prefix
        self._release = release_data
        self._exception = None
        self._proxy = None
        self._batch = None
        self._feature_names = None
        self._feature_types = None

    def reset(self):
        raise NotImplementedError()

    def next(self, input_data):
        raise NotImplementedError()

    # An exception inside a ctypes callback cannot cross the C frames: it is
    # kept, the iteration stops, and it is raised after the C call returns.
    def _handle_exception(self, fn, default):
        if self._exception is not None:
            return default
        try:
            return fn()
        except Exception as e:  # noqa: BLE001
            self._exception = e
        return default

    def reraise(self):
        self._batch = None
        if self._exception is not None:
            exc, self._exception = self._exception, None
            raise exc

    def _reset_wrapper(self, _this):
        if self._release:
            self._batch = None
        self._handle_exception(self.reset, None)

    def _input_data(self, *, data, label=None, weight=None, base_margin=None, feature_names=None,
                    feature_types=None, **kwargs):
        proxy = self._proxy
        if _is_scipy_csr(data):
            values = np.asarray(data.data, dtype=np.float32)
            keep = (data.indptr, data.indices, values)
            _check_call(_LIB.XGProxyDMatrixSetDataCSR(
                proxy, _c_str(_array_interface(data.indptr)), _c_str(_array_interface(data.indices)),
                _c_str(_array_interface(values)), c_bst_ulong(data.shape[1])))
        else:
            arr = _to_2d_float(data)
            keep = (arr,)
            _check_call(_LIB.XGProxyDMatrixSetDataDense(proxy, _c_str(_array_interface(arr))))
        # Every field is written for every batch (empty when absent), so no
        # field of an earlier batch survives into this one.
        for field, values in (("label", label), ("weight", weight), ("base_margin", base_margin)):
            v = np.zeros(0, np.float32) if values is None else \
                np.ascontiguousarray(np.asarray(values, dtype=np.float32).reshape(-1))
            keep = keep + (v,)
            _check_call(_LIB.XGDMatrixSetInfoFromInterface(proxy, _c_str(field),
                                                           _c_str(_array_interface(v))))
        if feature_names is not None:
            self._feature_names = list(feature_names)
        elif hasattr(data, "columns"):
            self._feature_names = [str(c) for c in data.columns]
        if feature_types is not None:
            self._feature_types = list(feature_types)
        for field, values in (("feature_name", self._feature_names), ("feature_type", self._feature_types)):
            if values is not None:
                _set_str_info(_LIB.XGDMatrixSetStrFeatureInfo, proxy, field, values)
        self._batch = keep

    def _next_wrapper(self, _this):
        return self._handle_exception(lambda: int(bool(self.next(self._input_data))), 0)

    def _create(self, config, ref=None, quantile=False):
        """Runs the iterator through the C callbacks and returns the handle."""
        proxy = ctypes.c_void_p()
        _check_call(_LIB.XGProxyDMatrixCreate(ctypes.byref(proxy)))
        self._proxy = proxy
        reset = _RESET_CALLBACK(self._reset_wrapper)
        nxt = _NEXT_CALLBACK(self._next_wrapper)
        handle = ctypes.c_void_p()
        try:
            if quantile:
                ret = _LIB.XGQuantileDMatrixCreateFromCallback(
                    None, proxy, ref, reset, nxt, _c_str(json.dumps(config)), ctypes.byref(handle))
            else:
                ret = _LIB.XGDMatrixCreateFromCallback(
                    None, proxy, reset, nxt, _c_str(json.dumps(config)), ctypes.byref(handle))
            self.reraise()
            _check_call(ret)
        finally:
            _LIB.XGDMatrixFree(proxy)
            self._proxy = None
            self._batch = None
        return handle


class DMatrix:
    """Data matrix (python-package/xgboost/core.py DMatrix). Quantisation is
    lazy: it happens on the first training round, as in the reference. A
    DataIter is read batch by batch and concatenated."""

    def __init__(self, data, label=None, *, weight=None, base_margin=None, missing=None,
                 silent=False, feature_names=None, feature_types=None, nthread=None,
                 group=None, qid=None, label_lower_bound=None, label_upper_bound=None,
                 feature_weights=None, enable_categorical=False, data_split_mode=None):
        if group is not None or qid is not None:
            raise XGBoostError("Ranking groups are not implemented by the CUDA backend.")
        self.handle = ctypes.c_void_p()
        miss = np.nan if missing is None else float(missing)
        config = {"missing": None if np.isnan(miss) else miss, "nthread": nthread or 0}
        if isinstance(data, DataIter):
            self.handle = data._create(config)
            self.feature_names = list(feature_names) if feature_names is not None else \
                data._feature_names
            self.feature_types = feature_types if feature_types is not None else data._feature_types
            return
        if isinstance(data, (str, os.PathLike)):
            # A text file: "path?format=csv" (label_column=K) or
            # "path?format=libsvm" (XGDMatrixCreateFromURI).
            uri = os.fspath(data)
            _check_call(_LIB.XGDMatrixCreateFromURI(_c_str(json.dumps({"uri": uri, "silent": int(silent)})),
                                                    ctypes.byref(self.handle)))
            if feature_names is not None:
                self.feature_names = feature_names
            if feature_types is not None:
                self.feature_types = feature_types
            for setter, values in ((self.set_label, label), (self.set_weight, weight),
                                   (self.set_base_margin, base_margin)):
                if values is not None:
                    setter(values)
            return
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

    @classmethod
    def _from_handle(cls, handle):
        d = cls.__new__(cls)
        d.handle = handle if isinstance(handle, ctypes.c_void_p) else ctypes.c_void_p(handle)
        return d

    # Feature names and types are kept by the native matrix, so slices, folds
    # and boosters created from it see them (python-package/xgboost/core.py
    # DMatrix.feature_names).
    @property
    def feature_names(self):
        return _get_str_info(_LIB.XGDMatrixGetStrFeatureInfo, self.handle, "feature_name")

    @feature_names.setter
    def feature_names(self, names):
        if names is not None:
            names = list(names)
            if len(names) != len(set(names)):
                raise ValueError("feature_names must be unique")
        _set_str_info(_LIB.XGDMatrixSetStrFeatureInfo, self.handle, "feature_name", names)

    @property
    def feature_types(self):
        return _get_str_info(_LIB.XGDMatrixGetStrFeatureInfo, self.handle, "feature_type")

    @feature_types.setter
    def feature_types(self, types):
        if isinstance(types, str):
            types = [types] * self.num_col()
        _set_str_info(_LIB.XGDMatrixSetStrFeatureInfo, self.handle, "feature_type", types)

    def slice(self, rindex, allow_groups=False):
        """The rows `rindex` as a new DMatrix (labels, weights, margins and
        feature names follow)."""
        idx = np.ascontiguousarray(np.asarray(rindex, dtype=np.int32).reshape(-1))
        handle = ctypes.c_void_p()
        _check_call(_LIB.XGDMatrixSliceDMatrixEx(self.handle, idx.ctypes.data_as(ctypes.POINTER(ctypes.c_int)),
                                                 c_bst_ulong(idx.size), ctypes.byref(handle),
                                                 ctypes.c_int(int(allow_groups))))
        return DMatrix._from_handle(handle)

    def get_data(self):
        """The present entries as a scipy CSR matrix."""
        from scipy.sparse import csr_matrix
        rows, cols, nnz = self.num_row(), self.num_col(), self.num_nonmissing()
        indptr = np.zeros(rows + 1, np.uint64)
        indices = np.zeros(max(nnz, 1), np.uint32)
        data = np.zeros(max(nnz, 1), np.float32)
        _check_call(_LIB.XGDMatrixGetDataAsCSR(self.handle, _c_str("{}"),
                                               indptr.ctypes.data_as(ctypes.POINTER(c_bst_ulong)),
                                               indices.ctypes.data_as(ctypes.POINTER(ctypes.c_uint)),
                                               data.ctypes.data_as(ctypes.POINTER(ctypes.c_float))))
        return csr_matrix((data[:nnz], indices[:nnz], indptr), shape=(rows, cols))

    def get_quantile_cut(self):
        """(indptr, values) of the histogram cuts: per feature -inf and then
        its cut values."""
        ip, vals = ctypes.c_char_p(), ctypes.c_char_p()
        _check_call(_LIB.XGDMatrixGetQuantileCut(self.handle, _c_str("{}"), ctypes.byref(ip),
                                                 ctypes.byref(vals)))
        ip_ai, v_ai = json.loads(ip.value.decode()), json.loads(vals.value.decode())
        indptr = np.ctypeslib.as_array(ctypes.cast(ip_ai["data"][0], ctypes.POINTER(c_bst_ulong)),
                                       (ip_ai["shape"][0],)).copy()
        n = v_ai["shape"][0]
        values = np.ctypeslib.as_array(ctypes.cast(v_ai["data"][0], ctypes.POINTER(ctypes.c_float)),
                                       (n,)).copy() if n else np.zeros(0, np.float32)
        return indptr, values

    def save_binary(self, fname, silent=True):
        _check_call(_LIB.XGDMatrixSaveBinary(self.handle, _c_str(os.fspath(fname)), ctypes.c_int(silent)))

    def set_info(self, *, label=None, weight=None, base_margin=None, feature_names=None,
                 feature_types=None, **kwargs):
        if label is not None:
            self.set_label(label)
        if weight is not None:
            self.set_weight(weight)
        if base_margin is not None:
            self.set_base_margin(base_margin)
        if feature_names is not None:
            self.feature_names = feature_names
        if feature_types is not None:
            self.feature_types = feature_types
        unknown = [k for k, v in kwargs.items() if v is not None]
        if unknown:
            raise XGBoostError("Unsupported metadata: %s" % ", ".join(unknown))

    def get_base_margin(self):
        return self.get_float_info("base_margin")

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
        self.max_bin = 256 if max_bin is None else int(max_bin)
        if isinstance(data, DataIter):
            if group is not None or qid is not None:
                raise XGBoostError("Ranking groups are not implemented by the CUDA backend.")
            miss = np.nan if missing is None else float(missing)
            config = {"missing": None if np.isnan(miss) else miss, "nthread": nthread or 0,
                      "max_bin": self.max_bin}
            self.handle = data._create(config, ref.handle if ref is not None else None,
                                       quantile=True)
            self.feature_names = list(feature_names) if feature_names is not None else \
                data._feature_names
            self.feature_types = feature_types if feature_types is not None else data._feature_types
            return
        super().__init__(data, label, weight=weight, base_margin=base_margin, missing=missing,
                         feature_names=feature_names, feature_types=feature_types, nthread=nthread,
                         group=group, qid=qid)
        _check_call(_LIB.XGDMatrixQuantise(self.handle, ctypes.c_int(self.max_bin),
                                           ref.handle if ref is not None else None))


class ExtMemQuantileDMatrix(QuantileDMatrix):
    """QuantileDMatrix from a DataIter for data that is streamed in batches
    (python-package/xgboost/core.py ExtMemQuantileDMatrix). The batches are
    concatenated in host memory (XGExtMemQuantileDMatrixCreateFromCallback);
    nothing is paged to disk."""

    def __init__(self, data, *, missing=None, nthread=None, max_bin=None, ref=None,
                 enable_categorical=False, max_quantile_batches=None, cache_host_ratio=None):
        if not isinstance(data, DataIter):
            raise TypeError("ExtMemQuantileDMatrix takes a DataIter.")
        self.max_bin = 256 if max_bin is None else int(max_bin)
        miss = np.nan if missing is None else float(missing)
        config = {"missing": None if np.isnan(miss) else miss, "nthread": nthread or 0,
                  "max_bin": self.max_bin}
        self.handle = data._create(config, ref.handle if ref is not None else None, quantile=True)
        if data._feature_names is not None:
            self.feature_names = data._feature_names
        if data._feature_types is not None:
            self.feature_types = data._feature_types


class Booster:
    """A gradient-boosted tree model trained on the GPU
    (python-package/xgboost/core.py Booster)."""

    def __init__(self, params=None, cache=None, model_file=None):
        cache = list(cache or [])
        arr = (ctypes.c_void_p * len(cache))(*[d.handle for d in cache])
        self.handle = ctypes.c_void_p()
        _check_call(_LIB.XGBoosterCreate(arr, c_bst_ulong(len(cache)), ctypes.byref(self.handle)))
        self._cache = cache
        if cache:
            self.feature_names = cache[0].feature_names
            self.feature_types = cache[0].feature_types
        if isinstance(model_file, Booster):
            # Model and configuration of another booster, as pickling copies them.
            buf = model_file.__getstate__()["handle"]
            _check_call(_LIB.XGBoosterUnserializeFromBuffer(self.handle, ctypes.c_char_p(buf),
                                                            c_bst_ulong(len(buf))))
        elif model_file is not None:
            self.load_model(model_file)
        # Parameters given here override those of a loaded model, as upstream.
        params = params or {}
        if isinstance(params, dict):
            items = list(params.items())
        else:
            items = list(params)
        for k, v in items:
            if k == "eval_metric" and isinstance(v, (list, tuple)):
                for m in v:  # each setting adds one metric
                    self.set_param(k, m)
                continue
            self.set_param(k, v)

    def __del__(self):
        if _LIB is not None and getattr(self, "handle", None) is not None and self.handle.value:
            _LIB.XGBoosterFree(self.handle)
            self.handle = None

    # Feature names and types live in the native booster, so that model files,
    # dumps and importance scores carry them (python-package/xgboost/core.py
    # Booster.feature_names).
    def _get_feature_info(self, field):
        length = c_bst_ulong()
        sarr = ctypes.POINTER(ctypes.c_char_p)()
        _check_call(_LIB.XGBoosterGetStrFeatureInfo(self.handle, _c_str(field), ctypes.byref(length),
                                                    ctypes.byref(sarr)))
        values = [sarr[i].decode() for i in range(length.value)]
        return values if values else None

    def _set_feature_info(self, field, values):
        if values is None:
            _check_call(_LIB.XGBoosterSetStrFeatureInfo(self.handle, _c_str(field), None,
                                                        c_bst_ulong(0)))
            return
        values = [str(v) for v in values]
        arr = (ctypes.c_char_p * len(values))(*[v.encode() for v in values])
        _check_call(_LIB.XGBoosterSetStrFeatureInfo(self.handle, _c_str(field), arr,
                                                    c_bst_ulong(len(values))))

    @property
    def feature_names(self):
        return self._get_feature_info("feature_name")

    @feature_names.setter
    def feature_names(self, names):
        self._set_feature_info("feature_name", names)

    @property
    def feature_types(self):
        return self._get_feature_info("feature_type")

    @feature_types.setter
    def feature_types(self, types):
        self._set_feature_info("feature_type", types)

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

    def _validate_features(self, feature_names):
        """Raises ValueError when the data's feature names differ from the
        model's (python-package/xgboost/core.py Booster._validate_features)."""
        mine = self.feature_names
        if mine is None:
            return
        if feature_names is None:
            raise ValueError("data did not contain feature names, but the following fields are expected: "
                             + ", ".join(mine))
        if list(mine) != list(feature_names):
            msg = "feature_names mismatch: {0} {1}".format(mine, feature_names)
            dat_missing = set(mine) - set(feature_names)
            my_missing = set(feature_names) - set(mine)
            if dat_missing:
                msg += "\nexpected " + ", ".join(str(s) for s in dat_missing) + " in input data"
            if my_missing:
                msg += "\ntraining data did not have the following fields: " + ", ".join(str(s) for s in my_missing)
            raise ValueError(msg)

    def get_split_value_histogram(self, feature, fmap="", bins=None, as_pandas=True):
        """Histogram of the thresholds the model splits `feature` at: rows of
        (SplitValue, Count) for the non-empty bins."""
        import re
        names = self.feature_names
        if names is not None and feature in names:
            types = self.feature_types
            if types is not None and types[names.index(feature)] == "c":
                raise ValueError("Split value histogram doesn't support categorical split.")
        pattern = re.compile(r"\[{0}<([\d.Ee+-]+)\]".format(re.escape(str(feature))))
        values = [float(x) for tree in self.get_dump(fmap=fmap) for x in pattern.findall(tree)]
        n_unique = len(np.unique(values))
        nbins = max(min(n_unique, bins) if bins is not None else n_unique, 1)
        counts, edges = np.histogram(values, bins=nbins)
        stacked = np.column_stack((edges[1:], counts))
        stacked = stacked[stacked[:, 1] > 0]
        if as_pandas:
            try:
                from pandas import DataFrame
                return DataFrame(stacked, columns=["SplitValue", "Count"])
            except ImportError:
                pass
        return stacked

    def update(self, dtrain, iteration, fobj=None):
        """One boosting round; with `fobj(margins, dtrain) -> (grad, hess)` the
        round trains on a custom objective's gradients."""
        if self.feature_names is None and dtrain.num_row():
            names, types = dtrain.feature_names, dtrain.feature_types
            if names is not None:
                self.feature_names = names
            if types is not None:
                self.feature_types = types
        else:
            self._validate_features(dtrain.feature_names)
        if fobj is None:
            _check_call(_LIB.XGBoosterUpdateOneIter(self.handle, ctypes.c_int(iteration),
                                                    dtrain.handle))
            return
        pred = self.predict(dtrain, output_margin=True, training=True)
        grad, hess = fobj(pred, dtrain)
        self.boost(dtrain, iteration, grad, hess)

    def boost(self, dtrain, iteration, grad, hess):
        """One round from gradients and Hessians of shape (rows,) or
        (rows, groups) (XGBoosterTrainOneIter)."""
        g = np.ascontiguousarray(np.asarray(grad, dtype=np.float32))
        h = np.ascontiguousarray(np.asarray(hess, dtype=np.float32))
        if g.shape != h.shape:
            raise ValueError("grad / hess shape mismatch: %s / %s" % (g.shape, h.shape))
        if g.ndim == 2 and g.shape[1] == 1:
            g, h = g.reshape(-1), h.reshape(-1)
        _check_call(_LIB.XGBoosterTrainOneIter(self.handle, dtrain.handle, ctypes.c_int(iteration),
                                               _c_str(_array_interface(g)),
                                               _c_str(_array_interface(h))))

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
        if pred_contribs or pred_interactions:
            raise XGBoostError("Contribution predictions are not implemented by the CUDA backend.")
        if validate_features:
            self._validate_features(data.feature_names)
        config = json.dumps({"type": 6 if pred_leaf else (1 if output_margin else 0), "training": bool(training),
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
        """Prediction straight from an array (XGBoosterPredictFromDense); CSR
        input goes through a DMatrix."""
        if predict_type not in ("value", "margin"):
            raise XGBoostError("predict_type must be 'value' or 'margin'.")
        if validate_features:
            if hasattr(data, "columns"):
                self._validate_features([str(c) for c in data.columns])
            shape = getattr(data, "shape", None)
            if shape is not None and len(shape) == 2 and shape[1] != self.num_features():
                raise ValueError("Feature shape mismatch, expected: %d, got %d" % (self.num_features(), shape[1]))
        if _is_scipy_csr(data):
            dm = DMatrix(data, missing=missing, base_margin=base_margin)
            return self.predict(dm, output_margin=predict_type == "margin",
                                iteration_range=iteration_range, strict_shape=strict_shape)
        arr = _to_2d_float(data)
        miss = float(missing) if missing is not None else np.nan
        config = json.dumps({"type": 1 if predict_type == "margin" else 0, "training": False,
                             "iteration_begin": int(iteration_range[0]),
                             "iteration_end": int(iteration_range[1]),
                             "strict_shape": bool(strict_shape),
                             "missing": None if np.isnan(miss) else miss})
        proxy = None
        if base_margin is not None:
            proxy = ctypes.c_void_p()
            _check_call(_LIB.XGProxyDMatrixCreate(ctypes.byref(proxy)))
        try:
            if proxy is not None:
                bm = np.ascontiguousarray(np.asarray(base_margin, dtype=np.float32).reshape(-1))
                _check_call(_LIB.XGDMatrixSetInfoFromInterface(proxy, _c_str("base_margin"),
                                                               _c_str(_array_interface(bm))))
            shape = ctypes.POINTER(c_bst_ulong)()
            dims = c_bst_ulong()
            result = ctypes.POINTER(ctypes.c_float)()
            _check_call(_LIB.XGBoosterPredictFromDense(
                self.handle, _c_str(_array_interface(arr)), _c_str(config), proxy,
                ctypes.byref(shape), ctypes.byref(dims), ctypes.byref(result)))
            dims_t = tuple(shape[i] for i in range(dims.value))
            n = int(np.prod(dims_t)) if dims_t else 0
            return np.ctypeslib.as_array(result, shape=(n,)).copy().reshape(dims_t) if n else \
                np.zeros(dims_t, np.float32)
        finally:
            if proxy is not None:
                _LIB.XGDMatrixFree(proxy)

    # -- evaluation (python-package/xgboost/core.py eval_set / eval) ---------
    def eval_set(self, evals, iteration=0, feval=None, output_margin=True):
        """"[iteration]\tname-metric:value..." for every (DMatrix, name) pair
        (XGBoosterEvalOneIter), plus feval(predictions, dmatrix) -> (name,
        value) or a list of them."""
        for d, name in evals:
            if not isinstance(d, DMatrix) or not isinstance(name, str):
                raise TypeError("evals must be a list of (DMatrix, str) pairs")
        dmats = (ctypes.c_void_p * len(evals))(*[d.handle.value for d, _ in evals])
        names = (ctypes.c_char_p * len(evals))(*[n.encode() for _, n in evals])
        msg = ctypes.c_char_p()
        _check_call(_LIB.XGBoosterEvalOneIter(self.handle, ctypes.c_int(iteration), dmats, names,
                                              c_bst_ulong(len(evals)), ctypes.byref(msg)))
        res = msg.value.decode()
        if feval is not None:
            for d, evname in evals:
                ret = feval(self.predict(d, training=False, output_margin=output_margin), d)
                for name, val in (ret if isinstance(ret, list) else [ret]):
                    res += "\t%s-%s:%f" % (evname, name, val)
        return res

    def eval(self, data, name="eval", iteration=0):
        return self.eval_set([(data, name)], iteration)

    @property
    def best_iteration(self):
        v = self.attr("best_iteration")
        if v is None:
            raise AttributeError("`best_iteration` is only defined when early stopping is used.")
        return int(v)

    @property
    def best_score(self):
        v = self.attr("best_score")
        if v is None:
            raise AttributeError("`best_score` is only defined when early stopping is used.")
        return float(v)

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

    # Pickling keeps the model and the training configuration
    # (XGBoosterSerializeToBuffer: {"Config", "Model"} as UBJSON).
    def __getstate__(self):
        length = c_bst_ulong()
        out = ctypes.c_char_p()
        _check_call(_LIB.XGBoosterSerializeToBuffer(self.handle, ctypes.byref(length),
                                                    ctypes.byref(out)))
        state = {k: v for k, v in self.__dict__.items() if k not in ("handle", "_cache")}
        state["handle"] = bytes(ctypes.string_at(out, length.value))
        return state

    def __setstate__(self, state):
        state = dict(state)
        buf = state.pop("handle")
        handle = ctypes.c_void_p()
        _check_call(_LIB.XGBoosterCreate(None, c_bst_ulong(0), ctypes.byref(handle)))
        _check_call(_LIB.XGBoosterUnserializeFromBuffer(handle, ctypes.c_char_p(buf),
                                                        c_bst_ulong(len(buf))))
        self.__dict__.update(state)
        self.handle = handle
        self._cache = []

    def load_config(self, config):
        """Restores the parameters written by save_config."""
        _check_call(_LIB.XGBoosterLoadJsonConfig(self.handle, _c_str(config)))

    def reset(self):
        """Releases the training state on the device; the model stays."""
        _check_call(_LIB.XGBoosterReset(self.handle))
        return self

    def copy(self):
        return Booster(model_file=self.save_raw("ubj"))

    def __copy__(self):
        return self.copy()

    def __deepcopy__(self, memo):
        return self.copy()

    # -- slicing (python-package/xgboost/core.py Booster.__getitem__) --------
    def __getitem__(self, val):
        """A booster of the rounds selected by an int or a slice; the
        best_iteration and best_score attributes are dropped."""
        if isinstance(val, (int, np.integer)) and not isinstance(val, bool):
            val = slice(int(val), int(val) + 1)
        if val is Ellipsis:
            val = slice(0, 0)
        if isinstance(val, tuple):
            raise ValueError("Only supports slicing through 1 dimension.")
        if not isinstance(val, slice):
            raise TypeError("Expected an int, a slice or an ellipsis, got %s" % type(val).__name__)
        start = 0 if val.start is None or val.start is Ellipsis else val.start
        stop = 0 if val.stop is None or val.stop is Ellipsis else val.stop
        if val.stop is not None and val.stop is not Ellipsis and stop < start:
            raise ValueError("Invalid slice", val)
        step = 1 if val.step is None else val.step
        handle = ctypes.c_void_p()
        status = _LIB.XGBoosterSlice(self.handle, ctypes.c_int(start), ctypes.c_int(stop),
                                     ctypes.c_int(step), ctypes.byref(handle))
        if status == -2:
            raise IndexError("Layer index out of range")
        _check_call(status)
        sliced = Booster.__new__(Booster)
        sliced.handle = handle
        sliced._cache = []
        return sliced

    def __iter__(self):
        for i in range(self.num_boosted_rounds()):
            yield self[i]

    # -- model inspection (python-package/xgboost/core.py get_dump,
    # dump_model, get_score, get_fscore, trees_to_dataframe) ----------------
    def get_dump(self, fmap="", with_stats=False, dump_format="text"):
        """One string per tree: "text", "json" or "dot"."""
        length = c_bst_ulong()
        sarr = ctypes.POINTER(ctypes.c_char_p)()
        _check_call(_LIB.XGBoosterDumpModelEx(self.handle, _c_str(os.fspath(fmap)),
                                              ctypes.c_int(int(with_stats)), _c_str(dump_format),
                                              ctypes.byref(length), ctypes.byref(sarr)))
        return [sarr[i].decode() for i in range(length.value)]

    def dump_model(self, fout, fmap="", with_stats=False, dump_format="text"):
        """Writes get_dump to a file name or an open text file."""
        close = isinstance(fout, (str, os.PathLike))
        f = open(os.fspath(os.path.expanduser(fout)), "w", encoding="utf-8") if close else fout
        try:
            trees = self.get_dump(fmap, with_stats, dump_format)
            if dump_format == "json":
                f.write("[\n")
                f.write(",\n".join(trees))
                f.write("\n]")
            else:
                for i, tree in enumerate(trees):
                    f.write("booster[%d]:\n" % i)
                    f.write(tree)
        finally:
            if close:
                f.close()

    def get_score(self, fmap="", importance_type="weight"):
        """Importance of each feature used by a split: "weight", "gain",
        "cover", "total_gain" or "total_cover"."""
        features = ctypes.POINTER(ctypes.c_char_p)()
        scores = ctypes.POINTER(ctypes.c_float)()
        n = c_bst_ulong()
        dim = c_bst_ulong()
        shape = ctypes.POINTER(c_bst_ulong)()
        config = json.dumps({"importance_type": importance_type, "feature_map": os.fspath(fmap)})
        _check_call(_LIB.XGBoosterFeatureScore(self.handle, _c_str(config), ctypes.byref(n),
                                               ctypes.byref(features), ctypes.byref(dim),
                                               ctypes.byref(shape), ctypes.byref(scores)))
        return {features[i].decode(): float(scores[i]) for i in range(n.value)}

    def get_fscore(self, fmap=""):
        return self.get_score(fmap, importance_type="weight")

    def trees_to_dataframe(self, fmap=""):
        """One row per node: Tree, Target, Node, ID, Feature, Split, Yes, No,
        Missing, Gain (leaf value for leaves), Cover, Category."""
        from pandas import DataFrame
        model = json.loads(self.save_raw(raw_format="json"))
        gbm = model["learner"]["gradient_booster"]
        trees = gbm["model"]["trees"]
        tree_info = gbm["model"]["tree_info"]
        fnames = dict(enumerate(self.feature_names or []))
        ftypes = dict(enumerate(self.feature_types or []))
        cols = {k: [] for k in ("Tree", "Target", "Node", "ID", "Feature", "Split", "Yes", "No",
                                "Missing", "Gain", "Cover", "Category")}

        def row(**kw):
            for k in cols:
                cols[k].append(kw.get(k))

        for tid, tree in enumerate(trees):
            left, right = tree["left_children"], tree["right_children"]
            target = int(tree_info[tid])
            stack = [0]
            while stack:
                nid = stack.pop()
                if left[nid] == -1:
                    row(Tree=tid, Target=target, Node=nid, ID="%d-%d" % (tid, nid), Feature="Leaf",
                        Gain=float(tree["split_conditions"][nid]), Cover=tree["sum_hessian"][nid])
                    continue
                stack.append(left[nid])
                stack.append(right[nid])
                fidx = tree["split_indices"][nid]
                dft = left[nid] if tree["default_left"][nid] else right[nid]
                yes, no = left[nid], right[nid]
                split = tree["split_conditions"][nid]
                if ftypes.get(fidx, "q") == "i":
                    yes, no = (right[nid] if tree["default_left"][nid] else left[nid]), dft
                    split = None
                elif ftypes.get(fidx, "q") == "int":
                    split = float(math.ceil(split))
                row(Tree=tid, Target=target, Node=nid, ID="%d-%d" % (tid, nid),
                    Feature=fnames.get(fidx, "f%d" % fidx), Split=split, Yes="%d-%d" % (tid, yes),
                    No="%d-%d" % (tid, no), Missing="%d-%d" % (tid, dft),
                    Gain=tree["loss_changes"][nid], Cover=tree["sum_hessian"][nid])
        df = DataFrame(cols).astype({"Tree": "Int64", "Target": "Int64", "Node": "Int64",
                                     "ID": "string", "Feature": "string", "Split": "Float64",
                                     "Yes": "string", "No": "string", "Missing": "string",
                                     "Gain": "Float64", "Cover": "Float64"})
        return df.sort_values(["Tree", "Node", "Target"]).reset_index(drop=True)


def synchronize():
    """Waits for all work on the current device (used by timing code)."""
    _check_call(_LIB.XGBBSynchronize())


def set_device(ordinal):
    _check_call(_LIB.XGBBSetDevice(ctypes.c_int(int(ordinal))))

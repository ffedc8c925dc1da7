"""The drop-in boundary without a GPU: the library loads, exports every entry
point the headers declare, and reports errors the upstream way."""
import ctypes
import os
import re

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB = os.path.join(ROOT, "xgboost-metal_b200", "xgboost", "lib", "libxgboost.so")
HEADERS = [os.path.join(ROOT, "include", "xgboost", "c_api.h"), os.path.join(ROOT, "include", "xgb_b200.h")]


def declared_symbols():
    names = []
    for h in HEADERS:
        text = open(h).read()
        names += re.findall(r"^XGB_DLL\s+[\w\s\*]+?\b(\w+)\s*\(", text, flags=re.M)
    return sorted(set(names))


def test_headers_declare_the_training_path():
    names = declared_symbols()
    for must in ("XGDMatrixCreateFromDense", "XGBoosterCreate", "XGBoosterSetParam",
                 "XGBoosterUpdateOneIter", "XGBoosterPredictFromDMatrix", "XGBoosterPredict",
                 "XGBGetLastError", "XGCommunicatorInit", "XGBBTrainHost"):
        assert must in names


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(LIB)
    missing = [n for n in declared_symbols() if not hasattr(lib, n)]
    assert not missing, missing


def test_version_and_build_info():
    lib = ctypes.CDLL(LIB)
    v = [ctypes.c_int() for _ in range(3)]
    lib.XGBoostVersion(*[ctypes.byref(x) for x in v])
    assert [x.value for x in v] == [3, 5, 0]
    import xgboost
    info = xgboost.build_info()
    assert info["USE_CUDA"] and info["USE_NCCL"]


def test_dmatrix_round_trip_on_host():
    import xgboost as xgb
    X = np.arange(12, dtype=np.float32).reshape(4, 3)
    X[1, 2] = -999.0
    d = xgb.DMatrix(X, label=[0, 1, 0, 1], weight=[1, 2, 3, 4], missing=-999.0)
    assert d.num_row() == 4 and d.num_col() == 3
    assert d.num_nonmissing() == 11
    np.testing.assert_array_equal(d.get_label(), [0, 1, 0, 1])
    np.testing.assert_array_equal(d.get_weight(), [1, 2, 3, 4])


def test_csr_input_densifies_absent_entries_as_missing():
    import scipy.sparse as sp
    import xgboost as xgb
    m = sp.csr_matrix(np.array([[1.0, 0, 2.0], [0, 0, 3.0]], np.float32))
    d = xgb.DMatrix(m)
    assert d.num_row() == 2 and d.num_col() == 3 and d.num_nonmissing() == 3


def test_errors_are_reported_not_raised_through_the_abi():
    import xgboost as xgb
    X = np.ones((3, 2), np.float32)
    X[0, 0] = np.inf
    # A non-NaN missing sentinel takes the copying path, validated on the host
    # at construction; zero-copy input is validated when it reaches the GPU.
    with pytest.raises(xgb.XGBoostError, match="infinity"):
        xgb.DMatrix(X, missing=-999.0)
    with pytest.raises(xgb.XGBoostError, match="Label"):
        xgb.DMatrix(np.ones((2, 2), np.float32), label=[np.nan, 1])
    lib = ctypes.CDLL(LIB)
    lib.XGBGetLastError.restype = ctypes.c_char_p
    assert lib.XGDMatrixFree(None) == -1
    assert b"null" in lib.XGBGetLastError()


def test_no_gpu_means_a_clear_error_not_a_fallback():
    import xgboost as xgb
    try:
        import torch
        has_gpu = torch.cuda.is_available()
    except Exception:  # pragma: no cover
        has_gpu = False
    if has_gpu:
        pytest.skip("a GPU is present")
    d = xgb.DMatrix(np.ones((4, 2), np.float32), label=[0, 1, 0, 1])
    with pytest.raises(xgb.XGBoostError, match="CUDA"):
        xgb.train({"tree_method": "hist", "device": "cuda"}, d, 1)


def test_nccl_is_not_a_load_time_dependency():
    # NCCL is opened only when a communicator is created, so importing the
    # library never pins an NCCL build into the process.
    import subprocess
    out = subprocess.run(["ldd", LIB], capture_output=True, text=True).stdout
    assert "libnccl" not in out
    code = ("import sys; sys.path.insert(0, %r); import xgboost; import torch; print('ok')"
            % os.path.join(ROOT, "xgboost-metal_b200"))
    res = subprocess.run([__import__("sys").executable, "-c", code], capture_output=True, text=True)
    assert res.stdout.strip().endswith("ok"), res.stderr[-2000:]

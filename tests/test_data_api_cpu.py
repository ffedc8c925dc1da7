"""Host-side DMatrix entry points of the C ABI (no GPU): sparse and columnar
construction, text files, DLPack host tensors, metadata setters and getters,
feature names, data export, row slices, cross-validation folds, and the
single-rank collective entry points. Results are compared with dense numpy
equivalents read back through XGDMatrixGetDataAsCSR."""
import ctypes
import json
import socket

import numpy as np
import pytest

import xgboost as xgb
from xgboost import core

L = core._LIB
fp = ctypes.POINTER(ctypes.c_float)


def _ai(a):
    return core._c_str(core._array_interface(a))


def _handle(fn, *args):
    h = ctypes.c_void_p()
    core._check_call(fn(*args, ctypes.byref(h)))
    return h


def _dense(h):
    """The matrix's values (NaN = missing) through XGDMatrixGetDataAsCSR."""
    rows, cols, nnz = core.c_bst_ulong(), core.c_bst_ulong(), core.c_bst_ulong()
    core._check_call(L.XGDMatrixNumRow(h, ctypes.byref(rows)))
    core._check_call(L.XGDMatrixNumCol(h, ctypes.byref(cols)))
    core._check_call(L.XGDMatrixNumNonMissing(h, ctypes.byref(nnz)))
    indptr = np.zeros(rows.value + 1, np.uint64)
    indices = np.zeros(max(nnz.value, 1), np.uint32)
    data = np.zeros(max(nnz.value, 1), np.float32)
    core._check_call(L.XGDMatrixGetDataAsCSR(h, b"{}", indptr.ctypes.data_as(ctypes.POINTER(ctypes.c_uint64)),
                                             indices.ctypes.data_as(ctypes.POINTER(ctypes.c_uint)),
                                             data.ctypes.data_as(fp)))
    out = np.full((rows.value, cols.value), np.nan, np.float32)
    for r in range(rows.value):
        for k in range(int(indptr[r]), int(indptr[r + 1])):
            out[r, indices[k]] = data[k]
    return out


def _free(h):
    L.XGDMatrixFree(h)


@pytest.fixture
def dense():
    rng = np.random.default_rng(31)
    X = rng.normal(size=(9, 5)).astype(np.float32)
    X[rng.random(X.shape) < 0.3] = np.nan
    return X


def test_sparse_layouts_densify_like_numpy(dense):
    sp = pytest.importorskip("scipy.sparse")
    zeros_absent = np.nan_to_num(dense, nan=0.0)
    expect = np.where(zeros_absent == 0, np.nan, zeros_absent)
    csr = sp.csr_matrix(zeros_absent)
    h = _handle(L.XGDMatrixCreateFromCSR, _ai(csr.indptr), _ai(csr.indices), _ai(csr.data),
                core.c_bst_ulong(5), b"{}")
    np.testing.assert_array_equal(_dense(h), expect)
    _free(h)
    csc = sp.csc_matrix(zeros_absent)
    h = _handle(L.XGDMatrixCreateFromCSC, _ai(csc.indptr), _ai(csc.indices), _ai(csc.data),
                core.c_bst_ulong(9), b"{}")
    np.testing.assert_array_equal(_dense(h), expect)
    _free(h)
    coo = sp.coo_matrix(zeros_absent)
    ri, ci = coo.row.astype(np.int64), coo.col.astype(np.int64)  # kept alive: the JSON holds raw pointers
    h = _handle(L.XGDMatrixCreateFromCOO, _ai(ri), _ai(ci), _ai(coo.data), core.c_bst_ulong(9),
                core.c_bst_ulong(5), b"{}")
    np.testing.assert_array_equal(_dense(h), expect)
    _free(h)
    # An explicit entry equal to `missing` is missing too.
    h = _handle(L.XGDMatrixCreateFromCSR, _ai(csr.indptr), _ai(csr.indices), _ai(csr.data),
                core.c_bst_ulong(5), json.dumps({"missing": float(csr.data[0])}).encode())
    got = _dense(h)
    _free(h)
    assert np.isnan(got).sum() == np.isnan(expect).sum() + 1
    bad_ptr = csr.indptr.copy()
    bad_ptr[-1] += 3
    assert L.XGDMatrixCreateFromCSR(_ai(bad_ptr), _ai(csr.indices), _ai(csr.data), core.c_bst_ulong(5), b"{}",
                                    ctypes.byref(ctypes.c_void_p())) == -1
    assert b"span" in L.XGBGetLastError()


def test_columnar_inputs_with_validity_masks(dense):
    cols = [np.ascontiguousarray(dense[:, c]) for c in range(5)]
    valid = np.array([1, 0, 1, 1, 1, 1, 0, 1, 1], np.uint8)
    bits = np.packbits(valid, bitorder="little")
    ifaces = []
    for c, col in enumerate(cols):
        d = json.loads(core._array_interface(col))
        if c == 2:
            d["mask"] = {"data": [bits.ctypes.data, True], "shape": [9], "typestr": "<t1", "version": 3}
        ifaces.append(d)
    h = _handle(L.XGDMatrixCreateFromColumnar, json.dumps(ifaces).encode(), b"{}")
    expect = dense.copy()
    expect[valid == 0, 2] = np.nan
    np.testing.assert_array_equal(_dense(h), expect)
    _free(h)
    ifaces[1]["shape"] = [8]
    assert L.XGDMatrixCreateFromColumnar(json.dumps(ifaces).encode(), b"{}", ctypes.byref(ctypes.c_void_p())) == -1
    assert b"same length" in L.XGBGetLastError()


def test_text_files(tmp_path):
    csv = tmp_path / "d.csv"
    csv.write_text("1.5,0,2\n,3,-1\n4,1,0.25\n")
    h = _handle(L.XGDMatrixCreateFromURI, json.dumps({"uri": str(csv) + "?format=csv&label_column=1"}).encode())
    np.testing.assert_array_equal(_dense(h), np.array([[1.5, 2], [np.nan, -1], [4, 0.25]], np.float32))
    n = core.c_bst_ulong()
    p = fp()
    core._check_call(L.XGDMatrixGetFloatInfo(h, b"label", ctypes.byref(n), ctypes.byref(p)))
    np.testing.assert_array_equal(np.ctypeslib.as_array(p, (n.value,)), [0, 3, 1])
    _free(h)
    svm = tmp_path / "d.svm"
    svm.write_text("1 0:1.5 3:2\n0 1:-1 # comment\n1\n")
    h = _handle(L.XGDMatrixCreateFromURI, json.dumps({"uri": str(svm) + "?format=libsvm"}).encode())
    np.testing.assert_array_equal(_dense(h), np.array([[1.5, np.nan, np.nan, 2], [np.nan, -1, np.nan, np.nan],
                                                       [np.nan] * 4], np.float32))
    _free(h)
    svm.write_text("1 qid:3 0:1\n")
    assert L.XGDMatrixCreateFromURI(json.dumps({"uri": str(svm) + "?format=libsvm"}).encode(),
                                    ctypes.byref(ctypes.c_void_p())) == -1
    assert b"qid" in L.XGBGetLastError()
    assert L.XGDMatrixCreateFromURI(json.dumps({"uri": str(svm)}).encode(), ctypes.byref(ctypes.c_void_p())) == -1
    assert b"explicit format" in L.XGBGetLastError()


def test_dlpack_host_tensor_is_copied_and_released(dense):
    capsule_get = ctypes.pythonapi.PyCapsule_GetPointer
    capsule_get.restype = ctypes.c_void_p
    capsule_get.argtypes = [ctypes.py_object, ctypes.c_char_p]
    capsule_rename = ctypes.pythonapi.PyCapsule_SetName
    capsule_rename.argtypes = [ctypes.py_object, ctypes.c_char_p]
    src = np.ascontiguousarray(dense[:, ::2].astype(np.float64))  # strided source copied first
    cap = src.__dlpack__()
    ptr = capsule_get(cap, b"dltensor")
    capsule_rename(cap, b"used_dltensor")  # the library now owns the tensor
    h = _handle(L.XGDMatrixCreateFromDLPack, ctypes.c_void_p(ptr), ctypes.c_int(0), ctypes.c_float(np.nan))
    np.testing.assert_array_equal(_dense(h), src.astype(np.float32))
    _free(h)


def test_metadata_names_and_references(dense):
    d = xgb.DMatrix(dense)
    w64 = np.linspace(0.5, 1.5, 9)
    core._check_call(L.XGDMatrixSetDenseInfo(d.handle, b"weight", w64.ctypes.data_as(ctypes.c_void_p),
                                             core.c_bst_ulong(9), ctypes.c_int(2)))
    np.testing.assert_array_equal(d.get_weight(), w64.astype(np.float32))
    labels = np.arange(9, dtype=np.uint32)
    core._check_call(L.XGDMatrixSetUIntInfo(d.handle, b"label", labels.ctypes.data_as(ctypes.POINTER(ctypes.c_uint)),
                                            core.c_bst_ulong(9)))
    out = ctypes.c_char_p()
    core._check_call(L.XGDMatrixGetInfoRef(d.handle, b"label", ctypes.byref(out)))
    ref = json.loads(out.value.decode())
    assert ref["shape"] == [9] and ref["typestr"] == "<f4"
    view = np.ctypeslib.as_array(ctypes.cast(ref["data"][0], fp), (9,))
    np.testing.assert_array_equal(view, labels.astype(np.float32))
    assert L.XGDMatrixSetUIntInfo(d.handle, b"group", labels.ctypes.data_as(ctypes.POINTER(ctypes.c_uint)),
                                  core.c_bst_ulong(9)) == -1
    n = core.c_bst_ulong(7)
    up = ctypes.POINTER(ctypes.c_uint)()
    core._check_call(L.XGDMatrixGetUIntInfo(d.handle, b"group_ptr", ctypes.byref(n), ctypes.byref(up)))
    assert n.value == 0
    names = (ctypes.c_char_p * 5)(*[b"a", b"b", b"c", b"d", b"e"])
    core._check_call(L.XGDMatrixSetStrFeatureInfo(d.handle, b"feature_name", names, core.c_bst_ulong(5)))
    sarr = ctypes.POINTER(ctypes.c_char_p)()
    core._check_call(L.XGDMatrixGetStrFeatureInfo(d.handle, b"feature_name", ctypes.byref(n), ctypes.byref(sarr)))
    assert [sarr[i] for i in range(n.value)] == [b"a", b"b", b"c", b"d", b"e"]
    assert L.XGDMatrixSetStrFeatureInfo(d.handle, b"feature_name", names, core.c_bst_ulong(4)) == -1
    flag = ctypes.c_int(-1)
    core._check_call(L.XGDMatrixWasZeroCopied(d.handle, ctypes.byref(flag)))
    assert flag.value == 1  # float32 C-contiguous NaN-missing input is read in place
    copied = xgb.DMatrix(dense.astype(np.float64))
    core._check_call(L.XGDMatrixWasZeroCopied(copied.handle, ctypes.byref(flag)))
    assert flag.value == 0
    mode = core.c_bst_ulong(9)
    core._check_call(L.XGDMatrixDataSplitMode(d.handle, ctypes.byref(mode)))
    assert mode.value == 0


def test_slices_and_cv_folds(dense):
    d = xgb.DMatrix(dense, label=np.arange(9, dtype=np.float32), weight=np.linspace(1, 2, 9))
    names = (ctypes.c_char_p * 5)(*[b"a", b"b", b"c", b"d", b"e"])
    core._check_call(L.XGDMatrixSetStrFeatureInfo(d.handle, b"feature_name", names, core.c_bst_ulong(5)))
    idx = np.array([7, 0, 7, 3], np.int32)
    h = _handle(L.XGDMatrixSliceDMatrix, d.handle, idx.ctypes.data_as(ctypes.POINTER(ctypes.c_int)),
                core.c_bst_ulong(4))
    np.testing.assert_array_equal(_dense(h), dense[idx])
    s = xgb.DMatrix.__new__(xgb.DMatrix)
    s.handle = h
    np.testing.assert_array_equal(s.get_label(), idx.astype(np.float32))
    np.testing.assert_array_equal(s.get_weight(), np.linspace(1, 2, 9).astype(np.float32)[idx])
    n = core.c_bst_ulong()
    sarr = ctypes.POINTER(ctypes.c_char_p)()
    core._check_call(L.XGDMatrixGetStrFeatureInfo(h, b"feature_name", ctypes.byref(n), ctypes.byref(sarr)))
    assert n.value == 5
    bad = np.array([9], np.int32)
    assert L.XGDMatrixSliceDMatrix(d.handle, bad.ctypes.data_as(ctypes.POINTER(ctypes.c_int)), core.c_bst_ulong(1),
                                   ctypes.byref(ctypes.c_void_p())) == -1
    for shuffle, stratified in ((0, 0), (1, 0), (1, 1)):
        tr = (ctypes.c_void_p * 3)()
        te = (ctypes.c_void_p * 3)()
        core._check_call(L.XGDMatrixBuildCVFolds(d.handle, ctypes.c_int(3), ctypes.c_uint(5), ctypes.c_int(shuffle),
                                                 ctypes.c_int(stratified), tr, te))
        seen = []
        for k in range(3):
            test_labels = xgb.DMatrix.__new__(xgb.DMatrix)
            test_labels.handle = ctypes.c_void_p(te[k])
            train_labels = xgb.DMatrix.__new__(xgb.DMatrix)
            train_labels.handle = ctypes.c_void_p(tr[k])
            a, b = test_labels.get_label(), train_labels.get_label()
            assert len(a) == 3 and len(b) == 6 and not set(a) & set(b)
            seen += list(a)
        assert sorted(seen) == list(range(9))
        if not shuffle:
            assert [int(x) for x in seen] == list(range(9))  # contiguous chunks


def test_single_rank_collective_and_trackers(capfd):
    assert L.XGCommunicatorIsDistributed() == 0
    buf = np.array([1.5, 2.5], np.float32)
    core._check_call(L.XGCommunicatorAllreduce(buf.ctypes.data_as(ctypes.c_void_p), ctypes.c_size_t(2),
                                               ctypes.c_int(1), ctypes.c_int(2)))
    np.testing.assert_array_equal(buf, [1.5, 2.5])
    core._check_call(L.XGCommunicatorBroadcast(buf.ctypes.data_as(ctypes.c_void_p), ctypes.c_size_t(8),
                                               ctypes.c_int(0)))
    assert L.XGCommunicatorAllreduce(buf.ctypes.data_as(ctypes.c_void_p), ctypes.c_size_t(2), ctypes.c_int(12),
                                     ctypes.c_int(2)) == -1
    name = ctypes.c_char_p()
    core._check_call(L.XGCommunicatorGetProcessorName(ctypes.byref(name)))
    assert name.value.decode() == socket.gethostname()
    core._check_call(L.XGCommunicatorPrint(b"hello from the communicator"))
    assert "hello from the communicator" in capfd.readouterr().out
    assert L.XGTrackerCreate(b"{}", ctypes.byref(ctypes.c_void_p())) == -1
    assert b"NCCL" in L.XGBGetLastError()
    assert L.XGTrackerFree(None) == 0
    cat = ctypes.c_void_p(1)
    bst = xgb.Booster()
    core._check_call(L.XGBoosterGetCategories(bst.handle, b"{}", ctypes.byref(cat)))
    assert cat.value is None
    assert L.XGBCategoriesFree(None) == 0


def test_arrow_record_batch():
    pa = pytest.importorskip("pyarrow")
    batch = pa.record_batch({"a": pa.array([1.5, None, 3.0], pa.float64()),
                             "b": pa.array([1, 2, None], pa.int32()),
                             "c": pa.array([True, False, None])}).slice(0, 3)
    schema_buf = (ctypes.c_byte * 128)()
    array_buf = (ctypes.c_byte * 128)()
    batch._export_to_c(ctypes.addressof(array_buf), ctypes.addressof(schema_buf))
    h = _handle(L.XGDMatrixCreateFromArrow, ctypes.byref(schema_buf), ctypes.byref(array_buf),
                ctypes.c_float(np.nan))
    np.testing.assert_array_equal(_dense(h), np.array([[1.5, 1, 1], [np.nan, 2, 0], [3, np.nan, np.nan]],
                                                      np.float32))
    n = core.c_bst_ulong()
    sarr = ctypes.POINTER(ctypes.c_char_p)()
    core._check_call(L.XGDMatrixGetStrFeatureInfo(h, b"feature_name", ctypes.byref(n), ctypes.byref(sarr)))
    assert [sarr[i] for i in range(n.value)] == [b"a", b"b", b"c"]
    core._check_call(L.XGDMatrixGetStrFeatureInfo(h, b"feature_type", ctypes.byref(n), ctypes.byref(sarr)))
    assert [sarr[i] for i in range(n.value)] == [b"float", b"int", b"i"]
    _free(h)
    # An offset slice keeps its rows.
    sliced = batch.slice(1, 2)
    sliced._export_to_c(ctypes.addressof(array_buf), ctypes.addressof(schema_buf))
    h = _handle(L.XGDMatrixCreateFromArrow, ctypes.byref(schema_buf), ctypes.byref(array_buf),
                ctypes.c_float(np.nan))
    np.testing.assert_array_equal(_dense(h), np.array([[np.nan, 2, 0], [3, np.nan, np.nan]], np.float32))
    _free(h)


class BatchCSR(ctypes.Structure):
    _fields_ = [("size", ctypes.c_size_t), ("columns", ctypes.c_size_t), ("offset", ctypes.POINTER(ctypes.c_int64)),
                ("label", fp), ("weight", fp), ("index", ctypes.POINTER(ctypes.c_int)), ("value", fp)]


SET_DATA = ctypes.CFUNCTYPE(ctypes.c_int, ctypes.c_void_p, BatchCSR)
NEXT = ctypes.CFUNCTYPE(ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p)


def test_legacy_batch_iterator():
    batches = [  # (offsets, index, value, label)
        (np.array([0, 2, 3], np.int64), np.array([0, 2, 1], np.int32), np.array([1, 2, 3], np.float32),
         np.array([0, 1], np.float32)),
        (np.array([3, 4], np.int64), np.array([3], np.int32), np.array([4], np.float32), np.array([1], np.float32)),
    ]
    state = {"i": 0}

    def nxt(_handle, set_fn, holder):
        if state["i"] == len(batches):
            return 0
        off, idx, val, lab = batches[state["i"]]
        state["i"] += 1
        b = BatchCSR(len(off) - 1, 4, off.ctypes.data_as(ctypes.POINTER(ctypes.c_int64)),
                     lab.ctypes.data_as(fp), None, idx.ctypes.data_as(ctypes.POINTER(ctypes.c_int)),
                     val.ctypes.data_as(fp))
        return 1 if SET_DATA(set_fn)(holder, b) == 0 else 0

    cb = NEXT(nxt)
    h = _handle(L.XGDMatrixCreateFromDataIter, None, cb, None, ctypes.c_float(np.nan))
    np.testing.assert_array_equal(_dense(h), np.array([[1, np.nan, 2, np.nan], [np.nan, 3, np.nan, np.nan],
                                                       [np.nan, np.nan, np.nan, 4]], np.float32))
    n = core.c_bst_ulong()
    p = fp()
    core._check_call(L.XGDMatrixGetFloatInfo(h, b"label", ctypes.byref(n), ctypes.byref(p)))
    np.testing.assert_array_equal(np.ctypeslib.as_array(p, (n.value,)), [0, 1, 1])
    _free(h)

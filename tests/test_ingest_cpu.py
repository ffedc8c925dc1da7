"""Host ingestion paths of the C ABI that need no GPU: buffer descriptors
(the reference's spec_from_descriptor and ingest_strided_typed,
src/c_api.cpp:657-690, kernels/boost.metal:256-306) and batch iterators
through a proxy matrix (src/c_api.cpp:140-157, 214-224)."""
import ctypes

import numpy as np
import pytest

import xgboost as xgb
from xgboost import core


class Desc(ctypes.Structure):
    _fields_ = [("data", ctypes.c_void_p), ("shape", ctypes.c_uint64 * 2),
                ("strides", ctypes.c_int64 * 2), ("ndim", ctypes.c_uint32),
                ("dtype_code", ctypes.c_uint32), ("mask_data", ctypes.c_void_p),
                ("mask_bit_offset", ctypes.c_int64), ("mask_mode", ctypes.c_uint32),
                ("flags", ctypes.c_uint32)]


CODES = {np.dtype(np.float32): 1, np.dtype(np.float64): 2, np.dtype(np.float16): 3,
         np.dtype(np.int8): 5, np.dtype(np.int16): 6, np.dtype(np.int32): 7, np.dtype(np.int64): 8,
         np.dtype(np.uint8): 9, np.dtype(np.uint16): 10, np.dtype(np.uint32): 11,
         np.dtype(np.uint64): 12, np.dtype(np.bool_): 13}


def desc_of(a, code=None, mask=None, mask_mode=0, mask_offset=0, flags=0):
    d = Desc()
    d.data = a.ctypes.data
    d.ndim = a.ndim
    for i in range(a.ndim):
        d.shape[i] = a.shape[i]
        d.strides[i] = a.strides[i]
    d.dtype_code = CODES[a.dtype] if code is None else code
    d.mask_data = None if mask is None else mask.ctypes.data
    d.mask_mode = mask_mode
    d.mask_bit_offset = mask_offset
    d.flags = flags
    return d


def _label_through(d):
    """Decodes a 1-D descriptor through the label field and reads it back."""
    h = ctypes.c_void_p()
    x = np.zeros((4, 1), np.float32)
    core._check_call(core._LIB.XGDMatrixCreateFromMat(x.ctypes.data_as(ctypes.POINTER(ctypes.c_float)),
                                                      core.c_bst_ulong(4), core.c_bst_ulong(1),
                                                      ctypes.c_float(np.nan), ctypes.byref(h)))
    try:
        ret = core._LIB.XGDMatrixSetInfoFromBufferDescriptor(h, b"base_margin", ctypes.byref(d))
        core._check_call(ret)
        n = core.c_bst_ulong()
        p = ctypes.POINTER(ctypes.c_float)()
        core._check_call(core._LIB.XGDMatrixGetFloatInfo(h, b"base_margin", ctypes.byref(n),
                                                         ctypes.byref(p)))
        return np.ctypeslib.as_array(p, shape=(n.value,)).copy()
    finally:
        core._LIB.XGDMatrixFree(h)


@pytest.mark.parametrize("dtype", sorted(CODES, key=str))
def test_descriptor_dtypes_decode_like_numpy(dtype):
    a = np.array([0, 1, 2, 3, 7, 100], dtype=np.float64)
    if dtype.kind == "i":
        a = -a
    src = a.astype(dtype)
    got = _label_through(desc_of(src))
    np.testing.assert_array_equal(got, src.astype(np.float32))


def test_descriptor_bfloat16_strides_and_contiguous_flag():
    v = np.array([1.5, -2.25, 3.0e-3, 65504.0], np.float32)
    bf = (v.view(np.uint32) >> 16).astype(np.uint16)
    got = _label_through(desc_of(bf, code=4))
    np.testing.assert_array_equal(got, (bf.astype(np.uint32) << 16).view(np.float32))
    # Every other element through a negative-free stride.
    wide = np.arange(12, dtype=np.float64)
    np.testing.assert_array_equal(_label_through(desc_of(wide[::3])), [0, 3, 6, 9])
    # Bit 0 of flags: strides ignored, C-contiguous assumed.
    ints = np.arange(4, dtype=np.int32)
    d = desc_of(ints)
    d.strides[0] = 999
    d.flags = 1
    np.testing.assert_array_equal(_label_through(d), [0, 1, 2, 3])


def test_descriptor_bits_and_row_masks():
    bits = np.array([0b10110010, 0b00000001], np.uint8)
    d = desc_of(bits, code=14)
    d.shape[0] = 9
    d.flags = 4
    d.strides[0] = 1  # start at bit 1
    # Bits 1..9 of the LSB-first stream.
    stream = [(int(bits[i // 8]) >> (i % 8)) & 1 for i in range(16)]
    np.testing.assert_array_equal(_label_through(d), stream[1:10])
    vals = np.array([1.0, 2.0, 3.0, 4.0], np.float32)
    valid_bits = np.array([0b1011 << 2], np.uint8)
    out = _label_through(desc_of(vals, mask=valid_bits, mask_mode=1, mask_offset=2))
    np.testing.assert_array_equal(np.isnan(out), [False, False, True, False])
    valid_bytes = np.array([0, 1, 1, 0], np.uint8)
    out = _label_through(desc_of(vals, mask=valid_bytes, mask_mode=2))
    np.testing.assert_array_equal(np.isnan(out), [True, False, False, True])
    out = _label_through(desc_of(vals, mask=valid_bytes, mask_mode=3))
    np.testing.assert_array_equal(np.isnan(out), [False, True, True, False])


def test_descriptor_matrix_counts_missing_and_rejects_bad_input():
    X = np.arange(12, dtype=np.float64).reshape(4, 3)
    X[1, 2] = -1
    mask = np.array([1, 1, 0, 1], np.uint8)
    d = desc_of(X, mask=mask, mask_mode=2)
    h = ctypes.c_void_p()
    core._check_call(core._LIB.XGDMatrixCreateFromBufferDescriptor(ctypes.byref(d), ctypes.c_float(-1),
                                                                   ctypes.byref(h)))
    rows, cols, nnz = core.c_bst_ulong(), core.c_bst_ulong(), core.c_bst_ulong()
    core._check_call(core._LIB.XGDMatrixNumRow(h, ctypes.byref(rows)))
    core._check_call(core._LIB.XGDMatrixNumCol(h, ctypes.byref(cols)))
    core._check_call(core._LIB.XGDMatrixNumNonMissing(h, ctypes.byref(nnz)))
    core._LIB.XGDMatrixFree(h)
    # Row 2 is masked out (3 values) and -1 is the missing value (1 value).
    assert (rows.value, cols.value, nnz.value) == (4, 3, 8)
    # Zero copy of a float32 C-contiguous matrix.
    Y = np.ones((5, 2), np.float32)
    d = desc_of(Y, flags=2)
    core._check_call(core._LIB.XGDMatrixCreateFromBufferDescriptor(ctypes.byref(d), ctypes.c_float(np.nan),
                                                                   ctypes.byref(h)))
    core._LIB.XGDMatrixFree(h)
    for mutate, needle in ((lambda d: setattr(d, "ndim", 1), b"two dimensional"),
                           (lambda d: setattr(d, "dtype_code", 99), b"dtype"),
                           (lambda d: setattr(d, "mask_mode", 7), b"mask mode"),
                           (lambda d: setattr(d, "data", None), b"Null data")):
        d = desc_of(Y)
        mutate(d)
        assert core._LIB.XGDMatrixCreateFromBufferDescriptor(ctypes.byref(d), ctypes.c_float(np.nan),
                                                             ctypes.byref(h)) == -1
        assert needle in core._LIB.XGBGetLastError()
    inf = np.array([[1.0, np.inf]], np.float32)
    assert core._LIB.XGDMatrixCreateFromBufferDescriptor(ctypes.byref(desc_of(inf)), ctypes.c_float(np.nan),
                                                         ctypes.byref(h)) == -1
    assert b"infinity" in core._LIB.XGBGetLastError()


class Batches(xgb.DataIter):
    def __init__(self, parts, fail_at=None):
        super().__init__()
        self.parts = parts
        self.i = 0
        self.fail_at = fail_at
        self.resets = 0

    def reset(self):
        self.i = 0
        self.resets += 1

    def next(self, input_data):
        if self.i == len(self.parts):
            return False
        if self.fail_at == self.i:
            raise KeyError("batch %d is broken" % self.i)
        input_data(**self.parts[self.i])
        self.i += 1
        return True


def _parts(rng, sizes, cols=4, weights=True):
    out = []
    for n in sizes:
        X = rng.normal(size=(n, cols)).astype(np.float32)
        X[rng.random(X.shape) < 0.2] = np.nan
        part = {"data": X, "label": rng.normal(size=n).astype(np.float32)}
        if weights:
            part["weight"] = rng.random(n).astype(np.float32)
        out.append(part)
    return out


def test_iterator_concatenates_batches_and_metadata():
    rng = np.random.default_rng(5)
    parts = _parts(rng, [7, 1, 12])
    it = Batches(parts)
    d = xgb.DMatrix(it)
    assert it.resets == 2
    assert (d.num_row(), d.num_col()) == (20, 4)
    X = np.concatenate([p["data"] for p in parts])
    assert d.num_nonmissing() == int(np.sum(~np.isnan(X)))
    np.testing.assert_array_equal(d.get_label(), np.concatenate([p["label"] for p in parts]))
    np.testing.assert_array_equal(d.get_weight(), np.concatenate([p["weight"] for p in parts]))


def test_iterator_missing_value_csr_and_feature_names():
    sp = pytest.importorskip("scipy.sparse")
    a = np.array([[1.0, -9.0], [-9.0, 4.0]], np.float32)
    csr = sp.csr_matrix(np.array([[0.0, 5.0], [6.0, 0.0]], np.float32))
    it = Batches([{"data": a, "label": [0, 1], "feature_names": ["u", "v"]},
                  {"data": csr, "label": [1, 0]}])
    d = xgb.DMatrix(it, missing=-9.0)
    assert d.num_row() == 4 and d.num_col() == 2
    assert d.num_nonmissing() == 4  # two -9 entries, two absent CSR entries
    assert d.feature_names == ["u", "v"]


def test_iterator_errors():
    rng = np.random.default_rng(6)
    with pytest.raises(KeyError, match="broken"):
        xgb.DMatrix(Batches(_parts(rng, [3, 3]), fail_at=1))
    bad = _parts(rng, [3, 3])
    bad[1]["data"] = bad[1]["data"][:, :3]
    with pytest.raises(xgb.XGBoostError, match="same number of features"):
        xgb.DMatrix(Batches(bad))
    mixed = _parts(rng, [3, 3])
    del mixed[1]["weight"]
    with pytest.raises(xgb.XGBoostError, match="weights"):
        xgb.DMatrix(Batches(mixed))
    with pytest.raises(xgb.XGBoostError, match="no feature data"):
        xgb.DMatrix(Batches([]))

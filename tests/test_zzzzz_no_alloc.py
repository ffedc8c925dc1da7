"""XGBBGradientsDeviceNoAlloc: the device-pointer gradient entry point whose
scale accumulators live in a fixed device array. It must give the same pairs
and scales as XGBBGradientsHost (which sizes its buffers per call), also when
called twice in a row on one stream, since each call must clear the array
before accumulating into it. Collected last so that it also runs after every
other test has used the device."""
import ctypes

import numpy as np
import pytest

from product import _ptr, check, lib

OBJECTIVES = {"reg:squarederror": 0, "binary:logistic": 1, "multi:softprob": 3}


def _inputs(objective, rows, groups, seed, weighted):
    rng = np.random.default_rng(seed)
    margins = (rng.standard_normal((rows, groups)) * 3).astype(np.float32)
    if objective == "multi:softprob":
        labels = rng.integers(0, groups, rows).astype(np.float32)
    elif objective == "binary:logistic":
        labels = (rng.random(rows) < 0.3).astype(np.float32)
    else:
        labels = (rng.standard_normal(rows) * 10).astype(np.float32)
    weights = rng.uniform(0.1, 4.0, rows).astype(np.float32) if weighted else None
    return margins, labels, weights


def _host(objective, margins, labels, weights, spw):
    rows, groups = margins.shape
    pairs = np.zeros((groups, rows, 2), np.float32)
    scales = np.zeros((groups, 2), np.float32)
    check(lib().XGBBGradientsHost(ctypes.c_int(OBJECTIVES[objective]), _ptr(margins), _ptr(labels),
                                  _ptr(weights), ctypes.c_uint64(rows), ctypes.c_uint32(groups),
                                  ctypes.c_float(spw), _ptr(pairs), _ptr(scales)))
    return pairs, scales


def _upload(torch, margins, labels, weights):
    """Device copies of one case plus output buffers filled with NaN."""
    rows, groups = margins.shape
    dev = torch.device("cuda", 0)
    return (torch.from_numpy(margins).to(dev), torch.from_numpy(labels).to(dev),
            None if weights is None else torch.from_numpy(weights).to(dev),
            torch.full((groups, rows, 2), float("nan"), dtype=torch.float32, device=dev),
            torch.full((groups, 2), float("nan"), dtype=torch.float32, device=dev))


def _enqueue(stream, objective, bufs, spw):
    """Enqueues the no-allocation call on `stream` without waiting for it."""
    dm, dl, dw, pairs, scales = bufs
    rows, groups = dm.shape
    check(lib().XGBBGradientsDeviceNoAlloc(
        ctypes.c_int(OBJECTIVES[objective]), ctypes.c_void_p(dm.data_ptr()),
        ctypes.c_void_p(dl.data_ptr()), None if dw is None else ctypes.c_void_p(dw.data_ptr()),
        ctypes.c_uint64(rows), ctypes.c_uint32(groups), ctypes.c_float(spw),
        ctypes.c_void_p(pairs.data_ptr()), ctypes.c_void_p(scales.data_ptr()),
        ctypes.c_void_p(stream.cuda_stream)))


@pytest.mark.gpu
def test_two_calls_in_a_row_match_the_allocating_entry_point():
    import torch
    cases = [("binary:logistic", 100_003, 1, 11, True, 2.5),
             ("multi:softprob", 7_777, 5, 12, False, 1.0),
             ("reg:squarederror", 65_536, 1, 13, True, 1.0)]
    stream = torch.cuda.Stream(device=0)
    inputs = [_inputs(obj, rows, groups, seed, w) for obj, rows, groups, seed, w, _ in cases]
    bufs = [_upload(torch, *inp) for inp in inputs]
    torch.cuda.synchronize()
    # All calls back to back on one stream, with no wait in between: each one
    # must clear the accumulators the previous one left behind.
    for (obj, _, _, _, _, spw), b in zip(cases, bufs):
        _enqueue(stream, obj, b, spw)
    stream.synchronize()
    for (obj, _, _, _, _, spw), inp, b in zip(cases, inputs, bufs):
        want_pairs, want_scales = _host(obj, *inp, spw)
        assert b[3].cpu().numpy().tobytes() == want_pairs.tobytes(), obj
        assert b[4].cpu().numpy().tobytes() == want_scales.tobytes(), obj


@pytest.mark.gpu
def test_repeated_call_is_identical():
    import torch
    stream = torch.cuda.Stream(device=0)
    inp = _inputs("multi:softprob", 30_000, 3, 21, True)
    first, second = _upload(torch, *inp), _upload(torch, *inp)
    torch.cuda.synchronize()
    _enqueue(stream, "multi:softprob", first, 1.0)
    _enqueue(stream, "multi:softprob", second, 1.0)
    stream.synchronize()
    want_pairs, want_scales = _host("multi:softprob", *inp, 1.0)
    for b in (first, second):
        assert b[3].cpu().numpy().tobytes() == want_pairs.tobytes()
        assert b[4].cpu().numpy().tobytes() == want_scales.tobytes()


@pytest.mark.parametrize("groups,rows,needle", [(65, 10, "exceeds the 64 output groups"),
                                                (0, 10, "groups must be at least 1"),
                                                (1, 0, "rows must be between")])
def test_sizes_beyond_the_fixed_scratch_are_rejected(groups, rows, needle):
    # Rejected before anything touches the device: runs without a GPU too.
    dummy = ctypes.c_void_p(16)
    ret = lib().XGBBGradientsDeviceNoAlloc(ctypes.c_int(1), dummy, dummy, None, ctypes.c_uint64(rows),
                                           ctypes.c_uint32(groups), ctypes.c_float(1.0), dummy, dummy,
                                           None)
    assert ret == -1
    assert needle in lib().XGBGetLastError().decode()

"""lrs_matvec_noalloc -- the matvec for callers that cannot allocate device memory.

Some host engines give the library a fixed device-memory budget at start-up
and forbid allocation afterwards, or must not let a call trigger cudaMalloc's
device-wide synchronization.  lrs_matvec stages its host vectors through
device buffers it allocates on first use; lrs_matvec_noalloc stages them
through a fixed array built into the library instead.  This test calls it
through the C ABI and checks it against lrs_matvec on two calls in a row (the
second call reuses the array the first one left behind), with the tolerance
the other GEMV tests use.  It lives in its own file, collected last, so a run
that stops at the first failure has already run every other test.
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
TOL = 1e-3  # |got - ref| <= TOL * max(|ref|, 1), as in test_gpu_gemv.py


def _call_noalloc(lrs, backend, t, x):
    lib = lrs.library()
    handle = backend.upload(t)
    y = np.empty(t.rows(), dtype=np.float32)
    code = lib.lrs_matvec_noalloc(backend.handle, handle,
                                  x.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), x.size,
                                  y.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), y.size)
    if code:
        raise lrs.LrsError(code, lib.lrs_last_error().decode())
    return y


def _close(got, ref):
    return np.all(np.abs(got - ref) <= TOL * np.maximum(np.abs(ref), 1.0))


@pytest.mark.parametrize("qt", ["Q4_K", "Q8_0", "Q6_K"])
def test_noalloc_matches_matvec_on_two_calls(lrs, backend, qt):
    rng = np.random.default_rng(42)
    shapes = [(1000, 2048), (333, 512)]  # the second call is smaller than the first
    for rows, cols in shapes:
        v = (rng.standard_normal(rows * cols) * 0.02).astype(np.float32)
        t = lrs.QuantTensor.quantize(v, rows, cols, lrs.QuantType[qt])
        x = rng.standard_normal(cols).astype(np.float32)
        ref = np.empty(rows, dtype=np.float32)
        backend.matvec(t, x, ref)
        got = _call_noalloc(lrs, backend, t, x)
        assert _close(got, ref), float(np.abs(got - ref).max())
        backend.release(t)


def test_noalloc_rejects_matrices_beyond_its_scratch(lrs, backend):
    cols = 65536 + 256
    t = lrs.QuantTensor.quantize(np.zeros(cols, np.float32), 1, cols, lrs.QuantType.Q8_0)
    with pytest.raises(lrs.LrsError, match="exceeds the fixed scratch"):
        _call_noalloc(lrs, backend, t, np.zeros(cols, np.float32))
    backend.release(t)

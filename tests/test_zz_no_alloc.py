"""lrs_matvec_noalloc -- the matvec for callers that cannot allocate device memory.

Some host engines give the library a fixed device-memory budget at start-up
and forbid allocation afterwards, or must not let a call trigger cudaMalloc's
device-wide synchronization.  lrs_matvec stages its host vectors through
device buffers it allocates on first use; lrs_matvec_noalloc stages them
through a fixed array built into the library instead.

This test calls it through the C ABI on two calls in a row (the second call
reuses the array the first one left behind) and checks every row against the
oracle's scalar dot (dot_row_scalar, src/quant.rs:458-648) within the row bar
of the other GEMV tests, and bit for bit against lrs_matvec, which runs the
same kernel.  One case sits at the column limit.  It lives in its own file,
collected last, so a run that stops at the first failure has already run every
other test.
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
TOL = 1e-3  # |got - ref| <= TOL * max(|ref|, 1), as in test_gpu_gemv.py
MAX_COLS = 65536
MAX_ROWS = 262144


def _call_noalloc(lrs, backend, t, x, n_out=None):
    lib = lrs.library()
    handle = backend.upload(t)
    y = np.empty(t.rows() if n_out is None else n_out, dtype=np.float32)
    code = lib.lrs_matvec_noalloc(backend.handle, handle,
                                  x.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), x.size,
                                  y.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), y.size)
    if code:
        raise lrs.LrsError(code, lib.lrs_last_error().decode())
    return y


def _check_rows(got, ref):
    err = np.abs(got.astype(np.float64) - ref.astype(np.float64))
    bound = TOL * np.maximum(np.abs(ref.astype(np.float64)), 1.0)
    assert np.all(err <= bound), f"{int((err > bound).sum())} rows off; worst err {err.max():.3e}"


@pytest.mark.parametrize("qt", ["Q4_K", "Q8_0", "Q6_K"])
def test_noalloc_matches_oracle_on_two_calls(lrs, orc, backend, qt):
    rng = np.random.default_rng(42)
    shapes = [(1000, 2048), (333, 512)]  # the second call is smaller than the first
    for rows, cols in shapes:
        v = (rng.standard_normal(rows * cols) * 0.02).astype(np.float32)
        t = lrs.QuantTensor.quantize(v, rows, cols, lrs.QuantType[qt])
        x = rng.standard_normal(cols).astype(np.float32)
        got = _call_noalloc(lrs, backend, t, x)
        ref = orc.matvec(orc.SCALAR, t.data, int(t.quant_type), rows, cols, x)
        _check_rows(got, ref)
        same = np.empty(rows, dtype=np.float32)
        backend.matvec(t, x, same)
        assert np.array_equal(got.view(np.uint32), same.view(np.uint32))
        backend.release(t)


def test_noalloc_at_the_column_limit(lrs, orc, backend):
    rows, cols = 40, MAX_COLS
    rng = np.random.default_rng(5)
    v = (rng.standard_normal(rows * cols) * 0.02).astype(np.float32)
    t = lrs.QuantTensor.quantize(v, rows, cols, lrs.QuantType.Q4_K)
    x = rng.standard_normal(cols).astype(np.float32)
    for _ in range(2):
        got = _call_noalloc(lrs, backend, t, x)
        _check_rows(got, orc.matvec(orc.SCALAR, t.data, int(t.quant_type), rows, cols, x))
    backend.release(t)


def test_noalloc_rejects_matrices_beyond_its_scratch(lrs, backend):
    cols = MAX_COLS + 256
    t = lrs.QuantTensor.quantize(np.zeros(cols, np.float32), 1, cols, lrs.QuantType.Q8_0)
    with pytest.raises(lrs.LrsError, match="exceeds the fixed scratch"):
        _call_noalloc(lrs, backend, t, np.zeros(cols, np.float32))
    backend.release(t)
    rows = MAX_ROWS + 1  # rejected on the host before any device work
    t = lrs.QuantTensor.quantize(np.zeros(rows * 32, np.float32), rows, 32, lrs.QuantType.Q8_0)
    with pytest.raises(lrs.LrsError, match="exceeds the fixed scratch"):
        _call_noalloc(lrs, backend, t, np.zeros(32, np.float32))
    backend.release(t)

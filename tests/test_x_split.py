"""The activation splits of the CUDA dot products, restated on the CPU.

The kernels never round the weights (they are decoded exactly from their
GGML blocks) but feed x to the integer / tensor-core units split in two:

* batch 1 (gemv_fast.cuh prep_x, gemv5_kernel): per 8-column run,
  s = max|x| / 127, q = x / s, xh = rint(q), xl = clamp(rint((q - xh) * 256),
  -127, 127); x ~= s * (xh + xl / 256), products summed exactly in int32 by
  dp4a;
* batched (gemm_mma.cu xsplit_kernel, gemm_tc.cu xsplit_tc_kernel): per item,
  s = 2^(e - 14) with max|x| = f * 2^e, f in [0.5, 1); xh = f16(x / s),
  xl = f16(x / s - xh); f16 x f16 products are exact in the f32 accumulators.

This test restates both splits in numpy and bounds the dot-product error
they cause against the f64 dot, for the row bar the GPU tests use
(1e-3 * max(|dot|, |w| |x| / sqrt(n))), on the x the models produce and on
adversarial x (one outlier per run, values spanning 30 binary orders,
mostly zeros, values near 1e-30).  It documents how much of the bar the split uses;
the kernels themselves are checked against the oracle by the GPU tests.
"""
import numpy as np
import pytest

BAR = 1e-3


def split_b1(x):
    """Batch-1 split: returns the reconstructed x (what the dp4a sums see)."""
    v = x.astype(np.float32).reshape(-1, 8)
    mx = np.abs(v).max(axis=1, keepdims=True)
    sc = np.where(mx > 0, mx / np.float32(127.0), np.float32(1.0)).astype(np.float32)
    inv = (np.float32(1.0) / sc).astype(np.float32)
    q = (v * inv).astype(np.float32)
    h = np.rint(q)
    lo = np.clip(np.rint((q - h) * np.float32(256.0)), -127, 127)
    assert np.abs(h).max() <= 127
    # the kernel sums (h << 8) + l in int32 and multiplies by s / 256
    return ((h * 256 + lo) * (sc / np.float32(256.0))).reshape(-1).astype(np.float64)


def split_batched(x):
    """Batched split (one item): reconstructed x = s * (xh + xl)."""
    x = x.astype(np.float32)
    mx = float(np.abs(x).max())
    e = 14
    if mx > 0 and np.isfinite(mx):
        e = np.frexp(mx)[1]
    s = np.float32(np.ldexp(1.0, e - 14))
    y = (x / s).astype(np.float32)
    hi = y.astype(np.float16)
    lo = (y - hi.astype(np.float32)).astype(np.float16)
    assert np.isfinite(hi).all() and np.abs(hi.astype(np.float32)).max() < 2 ** 14
    return (hi.astype(np.float64) + lo.astype(np.float64)) * float(s)


def bar_share(w, x, xr):
    """Largest |dot error| / row bar over the rows of w."""
    exact = w.astype(np.float64) @ x.astype(np.float64)
    got = w.astype(np.float64) @ xr
    floor = (np.linalg.norm(w.astype(np.float64), axis=1) * np.linalg.norm(x.astype(np.float64))
             / np.sqrt(x.size))
    return float((np.abs(got - exact) / (BAR * np.maximum(np.abs(exact), floor))).max())


def xs(kind, n, rng):
    if kind == "normal":
        return rng.standard_normal(n).astype(np.float32)
    if kind == "rmsnormed":  # post-RMSNorm activations: unit RMS
        x = rng.standard_normal(n) * rng.lognormal(0, 1, n)
        return (x / np.sqrt((x * x).mean())).astype(np.float32)
    if kind == "outlier_per_run":  # one value per 8-column run 1000x the rest
        x = rng.standard_normal(n).astype(np.float32)
        x[::8] *= 1000
        return x
    if kind == "wide_range":  # magnitudes over 30 binary orders
        return (rng.standard_normal(n) * 2.0 ** rng.integers(-20, 10, n)).astype(np.float32)
    if kind == "sparse":
        x = rng.standard_normal(n).astype(np.float32)
        x[rng.random(n) < 0.9] = 0
        return x
    if kind == "tiny":
        return (rng.standard_normal(n) * 1e-30).astype(np.float32)
    raise ValueError(kind)


KINDS = ["normal", "rmsnormed", "outlier_per_run", "wide_range", "sparse", "tiny"]


@pytest.mark.parametrize("kind", KINDS)
@pytest.mark.parametrize("n", [896, 3584, 18944])
def test_splits_stay_inside_the_row_bar(kind, n):
    rng = np.random.default_rng(n + len(kind))
    w = (rng.standard_normal((64, n)) * 0.02).astype(np.float32)
    x = xs(kind, n, rng)
    b1 = bar_share(w, x, split_b1(x))
    bt = bar_share(w, x, split_batched(x))
    print(f"{kind} n={n}: batch-1 split uses {b1:.2e} of the bar, batched split {bt:.2e}")
    assert b1 < 0.2 and bt < 1e-2


def test_split_bits():
    """Relative error of one reconstructed element: batch 1 about 2^-15 of
    its run's max, batched about 2^-22 of the item's max."""
    rng = np.random.default_rng(5)
    x = rng.standard_normal(1 << 16).astype(np.float32)
    runmax = np.abs(x.reshape(-1, 8)).max(axis=1).repeat(8)
    e1 = np.abs(split_b1(x) - x) / runmax
    e2 = np.abs(split_batched(x) - x) / np.abs(x).max()
    assert e1.max() < 2.0 ** -14.9
    assert e2.max() < 2.0 ** -21


def _f16_exact(v):
    v = np.asarray(v, np.float64)
    return np.array_equal(v.astype(np.float16).astype(np.float64), v)


def test_tensor_core_operands_are_exact_in_f16():
    """Every A value the tensor-core matmuls build from the GGML codes is an
    exact f16, so each product with an f16 x half is exact in f32 (11 x 11
    significant bits) and only the f32 accumulation rounds."""
    q4 = np.arange(16)
    sc6 = np.arange(64)
    # gemm_tc Q4_K: A = sc * q (6-bit scale, 4-bit code); A_min = 32 * m
    assert _f16_exact(np.outer(sc6, q4)) and _f16_exact(32 * sc6)
    # gemm_tc Q6_K: (q - 32) * (sc & 15) and (q - 32) * (sc - (sc & 15)), sc int8
    q6 = np.arange(64) - 32
    sc8 = np.arange(-128, 128)
    assert _f16_exact(np.outer(q6, sc8 & 15))
    assert _f16_exact(np.outer(q6, sc8 - (sc8 & 15)))
    # gemm_mma: q - z for every type (Q8_0 signed codes; 5-bit codes minus 16)
    assert _f16_exact(np.arange(-128, 128)) and _f16_exact(np.arange(32) - 16)
    # the x halves: |x / s| < 2^14 with s a power of two, so hi and lo are
    # finite f16 and hi * A < 2^14 * 2^12 stays far below the f32 range
    rng = np.random.default_rng(9)
    x = rng.standard_normal(4096).astype(np.float32) * np.float32(1e3)
    mx = float(np.abs(x).max())
    s = np.ldexp(1.0, np.frexp(mx)[1] - 14)
    hi = (x / np.float32(s)).astype(np.float16)
    assert np.isfinite(hi).all() and np.abs(hi.astype(np.float64)).max() < 2 ** 14
    a = np.float64(4096)
    prod = hi.astype(np.float64) * a
    assert np.array_equal(prod.astype(np.float32).astype(np.float64), prod)

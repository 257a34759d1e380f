"""CPU tests of the oracle (the C restatement of llama.rs's scalar path) and of
the product's load-time encoders.

* Known-answer blocks (tests/golden/kat_blocks.json) pin value_at and
  dot_row_scalar of every GGML type bit for bit.
* The reference's own unit tests (src/quant.rs:973-1063) are restated as-is:
  they are the only parity pins the reference ships.
"""
import json
import math
import os

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))


def _kat():
    with open(os.path.join(HERE, "golden", "kat_blocks.json")) as f:
        return json.load(f)["cases"]


@pytest.mark.parametrize("case", _kat(), ids=lambda c: c["name"])
def test_oracle_matches_known_answer_blocks(orc, case):
    t, rows, cols = case["type"], case["rows"], case["cols"]
    data = np.frombuffer(bytes.fromhex(case["data"]), dtype=np.uint8)
    rb = len(data) // rows
    x = np.array([math.sin(i * 0.037) for i in range(cols)], dtype=np.float32)
    for r in range(rows):
        row = data[r * rb:(r + 1) * rb]
        got = orc.dequantize_row(row, t, cols).view(np.uint32)
        assert got.tolist() == case["value_bits"][r]
        dot = np.float32(orc.dot_row(orc.SCALAR, row, t, x)).view(np.uint32)
        assert int(dot) == case["dot_bits"][r]


def _sin_cos_values(n):
    return np.array([(math.sin(i * 0.17) + math.cos(i * 0.03)) * 0.3 for i in range(n)],
                    dtype=np.float32)


def test_q4k_roundtrip_and_dot_are_consistent(lrs, orc):
    # src/quant.rs:973-995
    values = np.array([(np.float32(math.sin(np.float32(i) * np.float32(0.17))) +
                        np.float32(math.cos(np.float32(i) * np.float32(0.03)))) * np.float32(0.3)
                       for i in range(512)], dtype=np.float32)
    t = lrs.QuantTensor.quantize_q4k(values, 2, 256)
    assert t.quant_type == lrs.QuantType.Q4_K
    row = orc.dequantize_row(t.row_data(1), int(t.quant_type), 256)
    mae = float(np.abs(row - values[256:]).sum() / 256)
    assert mae < 0.06, mae
    inp = np.array([math.cos(i * 0.11) for i in range(256)], dtype=np.float32)
    expected = np.float32(0)
    for a, b in zip(row, inp):
        expected = np.float32(expected + a * b)
    out = orc.matvec(orc.SCALAR, t.data, int(t.quant_type), 2, 256, inp)
    assert abs(out[1] - expected) < 1e-4


def test_q4k_shape_falls_back_like_llama_cpp(lrs):
    # src/quant.rs:997-1001
    t = lrs.QuantTensor.quantize_q4k(np.zeros(896, np.float32), 1, 896)
    assert t.quant_type == lrs.QuantType.Q5_0


def _synthetic_q5k_block(lrs):
    # src/quant.rs:1016-1023
    data = bytearray(176)
    data[0:2] = np.array([0.003], dtype="<f2").tobytes()
    data[2:4] = np.array([0.001], dtype="<f2").tobytes()
    for i in range(4, 176):
        data[i] = ((i - 4) * 73 + 19) & 0xFF
    return lrs.QuantTensor(bytes(data), (1, 256), lrs.QuantType.Q5_K)


def test_avx2_quant_kernels_match_scalar(lrs, orc):
    # src/quant.rs:1003-1037
    if not orc.avx2_available():
        pytest.skip("no AVX2+FMA on this host")
    inp = np.array([math.sin(i * 0.037) for i in range(256)], dtype=np.float32)
    values = np.array([(math.sin(i * 0.071) - math.cos(i * 0.19)) * 0.2 for i in range(256)],
                      dtype=np.float32)
    tensors = [lrs.QuantTensor.quantize_q4k(values, 1, 256),
               lrs.QuantTensor.quantize_q5_0(values, 1, 256),
               _synthetic_q5k_block(lrs),
               lrs.QuantTensor.quantize_q6k(values, 1, 256),
               lrs.QuantTensor.quantize_q8_0(values, 1, 256)]
    for t in tensors:
        row = t.row_data(0)
        scalar = orc.dot_row(orc.SCALAR, row, int(t.quant_type), inp)
        simd = orc.dot_row(orc.AVX2, row, int(t.quant_type), inp)
        assert abs(scalar - simd) <= 2e-4 * max(abs(scalar), 1.0), t.quant_type


def test_q6k_and_q8_roundtrip(lrs, orc):
    # src/quant.rs:1039-1063
    values = np.array([(math.sin(i * 0.071) - math.cos(i * 0.19)) * 0.2 for i in range(512)],
                      dtype=np.float32)
    for t, max_mae in [(lrs.QuantTensor.quantize_q6k(values, 2, 256), 0.008),
                       (lrs.QuantTensor.quantize_q8_0(values, 2, 256), 0.003)]:
        decoded = orc.dequantize(t.data, int(t.quant_type), 2, 256)
        mae = float(np.abs(decoded.reshape(-1) - values).sum() / values.size)
        assert mae < max_mae, (t.quant_type, mae)
        inp = np.array([math.sin(i * 0.13) for i in range(256)], dtype=np.float32)
        expected = np.float32(0)
        for a, b in zip(decoded[0], inp):
            expected = np.float32(expected + a * b)
        out = orc.matvec(orc.SCALAR, t.data, int(t.quant_type), 2, 256, inp)
        assert abs(out[0] - expected) < 1e-4


@pytest.mark.parametrize("qt", ["F16", "BF16", "Q4_0", "Q4_1", "Q5_0", "Q5_1", "Q8_0", "Q4_K",
                                "Q5_K", "Q6_K"])
def test_encoders_roundtrip_quality(lrs, orc, qt):
    """Every encoder produces blocks value_at decodes close to the input."""
    rng = np.random.default_rng(3)
    values = (rng.standard_normal(4 * 512) * 0.02).astype(np.float32)
    t = lrs.QuantTensor.quantize(values, 4, 512, lrs.QuantType[qt])
    assert t.quant_type == lrs.QuantType[qt]
    dec = orc.dequantize(t.data, int(t.quant_type), 4, 512).reshape(-1)
    rel = float(np.abs(dec - values).mean() / np.abs(values).mean())
    limit = {"F16": 1e-3, "BF16": 1e-2, "Q8_0": 0.02, "Q6_K": 0.05}.get(qt, 0.2)
    assert rel < limit, rel


def test_scalar_matvec_is_thread_count_invariant(lrs, orc):
    rng = np.random.default_rng(0)
    values = (rng.standard_normal(512 * 1024) * 0.02).astype(np.float32)
    t = lrs.QuantTensor.quantize_q4k(values, 512, 1024)
    x = rng.standard_normal(1024).astype(np.float32)
    a = orc.matvec(orc.SCALAR, t.data, int(t.quant_type), 512, 1024, x, threads=1)
    b = orc.matvec(orc.SCALAR, t.data, int(t.quant_type), 512, 1024, x, threads=4)
    assert np.array_equal(a, b)


def test_oracle_argmax_takes_last_maximum(orc):
    # argmax_current_logits, src/engine.rs:233-241 (max_by keeps the last max)
    assert orc.argmax(np.array([1.0, 3.0, 2.0, 3.0, 0.5], np.float32)) == 3
    assert orc.argmax(np.array([-0.0, 0.0], np.float32)) == 1
    assert orc.argmax(np.array([0.0, -0.0], np.float32)) == 0  # total_cmp: -0 < +0
    assert orc.argmax(np.array([np.inf, np.nan], np.float32)) == 1  # +NaN ranks above +inf

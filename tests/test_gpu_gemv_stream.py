"""GPU parity of the bulk-copy batch-1 GEMV (gemv_stream.cu, LRS_GEMV_STREAM=1).

Same bars as the direct-load kernel: every row dot within 1e-3 relative of
dot_row_scalar (src/quant.rs:458-648), and a whole model's logits within 2e-2
and greedy tokens identical to the oracle's.  The cases cover every block
type, ragged row tiles, rows split into several K-chunks, rows whose bytes do
not start on a 16-byte boundary (Q6_K/Q5_0/Q8_0 row sizes), a segment run
(q/k/v) and all epilogues (bias, residual add, SwiGLU pair, argmax, fused
RMSNorm) through the model.

The kernel is selected per launch by LRS_GEMV_STREAM=1; these tests run when
LRS_TEST_NEW_KERNELS=1 is set as well.
"""
import os

import numpy as np
import pytest

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(os.environ.get("LRS_TEST_NEW_KERNELS") != "1",
                       reason="stream GEMV parity runs with LRS_TEST_NEW_KERNELS=1"),
]
TOL = 1e-3
LOGIT_TOL = 2e-2
ALL_TYPES = ["F16", "BF16", "Q4_0", "Q4_1", "Q5_0", "Q5_1", "Q8_0", "Q4_K", "Q5_K", "Q6_K"]


@pytest.fixture(autouse=True)
def stream_on(monkeypatch):
    monkeypatch.setenv("LRS_GEMV_STREAM", "1")


def _check_rows(got, ref):
    err = np.abs(got.astype(np.float64) - ref.astype(np.float64))
    bound = TOL * np.maximum(np.abs(ref.astype(np.float64)), 1.0)
    bad = np.nonzero(err > bound)
    assert bad[0].size == 0, f"{bad[0].size} rows off; worst err {err.max():.3e}"


_MATS = {}


def _matrix(lrs, qt, rows, cols, seed):
    """Quantized once per module (the host encoders are the slow part)."""
    key = (qt, rows, cols, seed)
    if key not in _MATS:
        v = (np.random.default_rng(seed).standard_normal(rows * cols) * 0.02).astype(np.float32)
        _MATS[key] = lrs.QuantTensor.quantize(v, rows, cols, lrs.QuantType[qt])
    return _MATS[key]


def _matvec_case(lrs, orc, backend, qt, rows, cols, seed):
    t = _matrix(lrs, qt, rows, cols, seed)
    assert t.quant_type == lrs.QuantType[qt]
    x = np.random.default_rng(seed + 1).standard_normal((1, cols)).astype(np.float32)
    got = backend.matvec_batched(t, x)[0]
    ref = orc.matvec(orc.SCALAR, t.data, int(t.quant_type), rows, cols, x[0])
    _check_rows(got, ref)
    y = np.empty(rows, dtype=np.float32)
    backend.matvec(t, x[0], y)
    assert np.array_equal(y, got)
    backend.release(t)


@pytest.mark.parametrize("qt", ALL_TYPES)
@pytest.mark.parametrize("shape", [(333, 1024), (7, 768), (1, 256)], ids=str)
def test_stream_matvec_every_type(lrs, orc, backend, qt, shape):
    # 333 rows: ragged last tile; 768 = 3 super-blocks: K-quant rows of 3 blocks
    # (Q6_K 630 bytes: rows off the 16-byte grid); 1 row: a single tile
    _matvec_case(lrs, orc, backend, qt, *shape, 21)


@pytest.mark.parametrize("qt,shape", [
    ("Q6_K", (3584, 18944)),    # c3 down: two K-chunks per row, 15540-byte rows
    ("Q4_K", (18944, 3584)),    # c3 gate/up shape
    ("Q4_K", (3584, 3584)),     # c3 q/o
    ("Q8_0", (512, 3584)),      # c3 v: few rows
    ("Q8_0", (152064, 3584)),   # c3 LM head under q4km
    ("Q5_0", (4864, 896)),      # c0 widths
    ("F16", (896, 4864)),
], ids=lambda v: str(v))
def test_stream_matvec_sweep_shapes(lrs, orc, backend, qt, shape):
    _matvec_case(lrs, orc, backend, qt, *shape, 23)


def _cfg(lrs, hidden, inter, heads, kv, layers, vocab, hd, tied):
    return lrs.LlamaConfig(hidden, inter, heads, kv, layers, vocab, 1e-6, 1e6, 32768, hd, tied)


@pytest.mark.parametrize("recipe", ["NONE", "Q4K", "Q4KM"])
def test_stream_tiny_model_greedy(lrs, orc, backend, recipe):
    cfg = _cfg(lrs, 512, 1024, 4, 2, 3, 2000, 128, False)
    sm = lrs.SynthModel(cfg, 5, lrs.LoadQuantization[recipe])
    prompt = lrs.prompt_tokens(5, 40, cfg.vocab_size)
    n_decode = 32
    ref = orc.OracleModel(sm.desc(), 256, orc.SCALAR, 0).benchmark_tokens(
        prompt, n_decode, keep_logits=True)
    model = lrs.CudaQwen2Model(backend, sm.desc(), max_seq_len=256)
    logits, first = model.prefill(prompt, 0)
    assert np.abs(logits - ref["logits"][0]).max() < LOGIT_TOL
    produced = model.decode_greedy([first], [len(prompt)], n_decode)[:, 0]
    toks = np.concatenate([[first], produced[:-1]])
    assert np.array_equal(ref["tokens"], toks)


def test_stream_c3_width_greedy(lrs, orc, backend):
    # 7B widths (q4km: Q4_K q/k/o/gate/up, Q8_0 v and head, Q6_K down), 2 layers
    cfg = lrs.config_c3()
    cfg.num_hidden_layers = 2
    sm = lrs.SynthModel(cfg, 2, lrs.LoadQuantization.Q4KM)
    prompt = lrs.prompt_tokens(2, 24, cfg.vocab_size)
    n_decode = 24
    ref = orc.OracleModel(sm.desc(), 128, orc.SCALAR, 0).benchmark_tokens(
        prompt, n_decode, keep_logits=True)
    model = lrs.CudaQwen2Model(backend, sm.desc(), max_seq_len=128)
    logits, first = model.prefill(prompt, 0)
    assert np.abs(logits - ref["logits"][0]).max() < LOGIT_TOL
    produced = model.decode_greedy([first], [len(prompt)], n_decode)[:, 0]
    toks = np.concatenate([[first], produced[:-1]])
    assert np.array_equal(ref["tokens"], toks)

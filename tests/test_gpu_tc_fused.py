"""GPU parity of the tcgen05 matmul with its output step fused (LRS_TC_FUSED=1)
and with Q4_K rows streamed through a shared-memory ring (LRS_TC_RAW=1).

The fused kernel adds the K-group partials in the order of the separate
epilogue kernel (in the CTA that finishes last for its row block) and applies
bias / residual add / SwiGLU / argmax itself, overlapping the x preparation by
programmatic dependent launch.  Bars: every row within 1e-3 relative of
dot_row_scalar (src/quant.rs:458-648); whole-model logits within 2e-2 and
greedy tokens equal to the oracle's.  The cases cover 16/32/64-item tiles,
one and several K-groups, Q4_K and Q6_K, every epilogue through the model
(q4k recipe: Q4_K LM head with the argmax in the matmul), and the backend's
own scratch (matvec_batched).

Selected per launch by LRS_TC_FUSED=1 / LRS_TC_RAW=1; runs when
LRS_TEST_NEW_KERNELS=1.
"""
import os

import numpy as np
import pytest

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(os.environ.get("LRS_TEST_NEW_KERNELS") != "1",
                       reason="fused tcgen05 parity runs with LRS_TEST_NEW_KERNELS=1"),
]
TOL = 1e-3
LOGIT_TOL = 2e-2


@pytest.fixture(autouse=True, params=["fused", "fused+raw", "raw"])
def fused_on(monkeypatch, request):
    # the fused output step, the raw-row ring for Q4_K (LRS_TC_RAW=1), and both
    if "fused" in request.param:
        monkeypatch.setenv("LRS_TC_FUSED", "1")
    if "raw" in request.param:
        monkeypatch.setenv("LRS_TC_RAW", "1")


def _check_rows(got, ref):
    err = np.abs(got.astype(np.float64) - ref.astype(np.float64))
    bound = TOL * np.maximum(np.abs(ref.astype(np.float64)), 1.0)
    bad = np.nonzero(err > bound)
    assert bad[0].size == 0, f"{bad[0].size} rows off; worst err {err.max():.3e}"


_MATS = {}


def _matrix(lrs, qt, rows, cols):
    """Quantized once per module (the host encoders are the slow part)."""
    key = (qt, rows, cols)
    if key not in _MATS:
        v = (np.random.default_rng(31).standard_normal(rows * cols) * 0.02).astype(np.float32)
        _MATS[key] = lrs.QuantTensor.quantize(v, rows, cols, lrs.QuantType[qt])
    return _MATS[key]


@pytest.mark.parametrize("shape", [(1000, 512), (300, 3584), (4864, 896 * 2), (18944, 3584)],
                         ids=str)
@pytest.mark.parametrize("batch", [5, 17, 33, 64])
@pytest.mark.parametrize("qt", ["Q4_K", "Q6_K"])
def test_fused_tc_matvec_batched(lrs, orc, backend, qt, shape, batch):
    rows, cols = shape
    t = _matrix(lrs, qt, rows, cols)
    x = np.random.default_rng(32).standard_normal((batch, cols)).astype(np.float32)
    got = backend.matvec_batched(t, x)
    for b in sorted({0, batch // 2, batch - 1}):
        ref = orc.matvec(orc.SCALAR, t.data, int(t.quant_type), rows, cols, x[b])
        _check_rows(got[b], ref)
    again = backend.matvec_batched(t, x)  # counters were left at zero
    assert np.array_equal(got, again)


def _cfg(lrs, hidden, inter, heads, kv, layers, vocab, hd, tied):
    return lrs.LlamaConfig(hidden, inter, heads, kv, layers, vocab, 1e-6, 1e6, 32768, hd, tied)


@pytest.mark.parametrize("recipe", ["Q4K", "Q4KM"])
@pytest.mark.parametrize("B", [5, 20, 64])
def test_fused_tc_batched_model(lrs, orc, backend, recipe, B):
    cfg = _cfg(lrs, 512, 1536, 4, 2, 2, 3000, 128, recipe == "Q4K")
    sm = lrs.SynthModel(cfg, 12, lrs.LoadQuantization[recipe])
    n_dec = 12
    m = lrs.CudaQwen2Model(backend, sm.desc(), max_seq_len=256, max_sequences=B)
    prompts = [lrs.prompt_tokens(400 + s, 20 + s % 7, cfg.vocab_size) for s in range(B)]
    firsts = [m.prefill(p, 0, seq=s)[1] for s, p in enumerate(prompts)]
    produced = m.decode_greedy(firsts, [len(p) for p in prompts], n_dec, list(range(B)))
    fed = np.concatenate([np.array(firsts, np.uint32)[None, :], produced[:-1]], axis=0)
    for s in sorted({0, B // 2, B - 1}):
        ref = orc.OracleModel(sm.desc(), 256).benchmark_tokens(prompts[s], n_dec)
        assert np.array_equal(ref["tokens"], fed[:, s]), f"sequence {s}"


def test_fused_tc_prefill_logits(lrs, orc, backend):
    # a 70-token prefill runs the batched matmuls on 64 + 6 token chunks
    cfg = _cfg(lrs, 512, 1024, 4, 2, 3, 2000, 128, False)
    sm = lrs.SynthModel(cfg, 5, lrs.LoadQuantization.Q4K)
    prompt = lrs.prompt_tokens(5, 70, cfg.vocab_size)
    ref = orc.OracleModel(sm.desc(), 256, orc.SCALAR, 0).benchmark_tokens(prompt, 4, keep_logits=True)
    model = lrs.CudaQwen2Model(backend, sm.desc(), max_seq_len=256)
    logits, first = model.prefill(prompt, 0)
    assert np.abs(logits - ref["logits"][0]).max() < LOGIT_TOL
    assert first == orc.argmax(ref["logits"][0])

"""GPU parity of the streamed decode attention (attn3_kernel, LRS_ATTN_V3=1).

Bars as for the whole model: logits within 2e-2 of the oracle's scalar path and
identical greedy tokens.  The cases cover head_dim 64 and 128, f32 and bf16 KV,
one 32-position block per split (many splits, the in-kernel combine), many
blocks per split (the three-stage ring wraps around), ragged last blocks, a
single split (direct output), and the streamed batch-1 GEMV together with it.

The kernel is selected per launch by LRS_ATTN_V3=1; these tests run when
LRS_TEST_NEW_KERNELS=1 is set as well.
"""
import os

import numpy as np
import pytest

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(os.environ.get("LRS_TEST_NEW_KERNELS") != "1",
                       reason="attention v3 parity runs with LRS_TEST_NEW_KERNELS=1"),
]
LOGIT_TOL = 2e-2


@pytest.fixture(autouse=True)
def attn3_on(monkeypatch):
    monkeypatch.setenv("LRS_ATTN_V3", "1")


def _cfg(lrs, hidden, inter, heads, kv, layers, vocab, hd, tied):
    return lrs.LlamaConfig(hidden, inter, heads, kv, layers, vocab, 1e-6, 1e6, 32768, hd, tied)


def _greedy_pair(lrs, orc, backend, cfg, seed, n_prompt, n_decode, max_seq, kv_bf16=False):
    sm = lrs.SynthModel(cfg, seed, lrs.LoadQuantization.Q4KM)
    prompt = lrs.prompt_tokens(seed, n_prompt, cfg.vocab_size)
    ref = orc.OracleModel(sm.desc(), max_seq, orc.SCALAR, 0).benchmark_tokens(
        prompt, n_decode, keep_logits=True)
    model = lrs.CudaQwen2Model(backend, sm.desc(), max_seq_len=max_seq, kv_bf16=kv_bf16)
    logits, first = model.prefill(prompt, 0)
    produced = model.decode_greedy([first], [n_prompt], n_decode)[:, 0]
    toks = np.concatenate([[first], produced[:-1]])
    return ref, logits, toks


@pytest.mark.parametrize("hd", [64, 128])
def test_attn3_tiny_model_greedy(lrs, orc, backend, hd):
    # 70 + 40 positions at batch 1: many single-block splits and the combine
    cfg = _cfg(lrs, 512, 1024, 512 // hd, 2, 3, 2000, hd, hd == 64)
    ref, logits, toks = _greedy_pair(lrs, orc, backend, cfg, 5, 70, 40, 1024)
    assert np.abs(logits - ref["logits"][0]).max() < LOGIT_TOL
    assert np.array_equal(ref["tokens"], toks)


@pytest.mark.parametrize("hd", [64, 128])
def test_attn3_bf16_kv(lrs, orc, backend, hd):
    cfg = _cfg(lrs, 512, 1024, 512 // hd, 2, 2, 2000, hd, True)
    ref, logits, toks = _greedy_pair(lrs, orc, backend, cfg, 6, 40, 8, 512, kv_bf16=True)
    assert np.abs(logits - ref["logits"][0]).max() < LOGIT_TOL


def test_attn3_long_context_batch1(lrs, orc, backend):
    # 700 prompt positions + 48 decode steps, GQA group of 7 (c0's 14 / 2 heads)
    cfg = _cfg(lrs, 896, 1024, 14, 2, 2, 3000, 64, True)
    ref, logits, toks = _greedy_pair(lrs, orc, backend, cfg, 7, 700, 48, 1024)
    assert np.abs(logits - ref["logits"][0]).max() < LOGIT_TOL
    assert np.array_equal(ref["tokens"], toks)


def test_attn3_many_blocks_per_split(lrs, orc, backend):
    # 64 sequences of ~600 positions: few splits per (item, kv head), so each
    # split streams ~10 blocks through the 3-stage ring; ragged ends differ per item
    cfg = _cfg(lrs, 512, 1024, 4, 2, 2, 3000, 128, False)
    sm = lrs.SynthModel(cfg, 8, lrs.LoadQuantization.Q4KM)
    B, n_dec = 64, 12
    m = lrs.CudaQwen2Model(backend, sm.desc(), max_seq_len=1024, max_sequences=B)
    prompts = [lrs.prompt_tokens(300 + s, 580 + 7 * (s % 9), cfg.vocab_size) for s in range(B)]
    firsts = [m.prefill(p, 0, seq=s)[1] for s, p in enumerate(prompts)]
    produced = m.decode_greedy(firsts, [len(p) for p in prompts], n_dec, list(range(B)))
    fed = np.concatenate([np.array(firsts, np.uint32)[None, :], produced[:-1]], axis=0)
    for s in (0, 17, 63):
        ref = orc.OracleModel(sm.desc(), 1024).benchmark_tokens(prompts[s], n_dec)
        assert np.array_equal(ref["tokens"], fed[:, s]), f"sequence {s}"


def test_attn3_with_stream_gemv_c3_width(lrs, orc, backend, monkeypatch):
    monkeypatch.setenv("LRS_GEMV_STREAM", "1")
    cfg = lrs.config_c3()
    cfg.num_hidden_layers = 2
    ref, logits, toks = _greedy_pair(lrs, orc, backend, cfg, 2, 40, 32, 256)
    assert np.abs(logits - ref["logits"][0]).max() < LOGIT_TOL
    assert np.array_equal(ref["tokens"], toks)

"""GPU parity of the whole Qwen2 token loop against the oracle.

Bars (from the task statement): final logits within 2e-2 max-abs of the
reference scalar path, and identical greedy token sequences (the oracle's
per-step top-1/top-2 margin is reported when a token differs).
"""
import numpy as np

from conftest import assert_greedy
import pytest

pytestmark = pytest.mark.gpu
LOGIT_TOL = 2e-2


def _cfg(lrs, hidden, inter, heads, kv, layers, vocab, hd, tied):
    return lrs.LlamaConfig(hidden, inter, heads, kv, layers, vocab, 1e-6, 1e6, 32768, hd, tied)


def _run_pair(lrs, orc, backend, cfg, recipe, seed, n_prompt, n_decode, max_seq=1024,
              threads=0, kv_bf16=False):
    sm = lrs.SynthModel(cfg, seed, recipe)
    prompt = lrs.prompt_tokens(seed, n_prompt, cfg.vocab_size)
    ref = orc.OracleModel(sm.desc(), max_seq, orc.SCALAR, threads).benchmark_tokens(
        prompt, n_decode, keep_logits=True)
    model = lrs.CudaQwen2Model(backend, sm.desc(), max_seq_len=max_seq, kv_bf16=kv_bf16)
    logits, first = model.prefill(prompt, 0)
    toks = []
    if n_decode:  # tokens fed to each decode step: the prefill argmax, then each step's argmax
        produced = model.decode_greedy([first], [n_prompt], n_decode)[:, 0]
        toks = np.concatenate([[first], produced[:-1]])
    return sm, model, prompt, ref, logits, first, np.asarray(toks)


def _assert_tokens(ref, toks):
    i = assert_greedy(ref, toks)
    if i is not None:
        print(f"greedy tokens equal up to the near-tie at step {i} "
              f"(oracle margin {ref['margins'][i]:.2e})")


@pytest.mark.parametrize("recipe", ["NONE", "Q4K", "Q4KM"])
@pytest.mark.parametrize("hd", [64, 128])
def test_tiny_model_prefill_and_greedy(lrs, orc, backend, recipe, hd):
    cfg = _cfg(lrs, 512, 1024, 512 // hd, 2 if hd == 128 else 4, 3, 2000, hd, hd == 64)
    sm, model, prompt, ref, logits, first, toks = _run_pair(
        lrs, orc, backend, cfg, lrs.LoadQuantization[recipe], 5, 70, 40)
    assert np.abs(logits - ref["logits"][0]).max() < LOGIT_TOL
    assert first == orc.argmax(ref["logits"][0])
    _assert_tokens(ref, toks)


def test_forward_token_matches_prefill(lrs, backend):
    cfg = _cfg(lrs, 256, 512, 4, 2, 2, 500, 64, True)
    sm = lrs.SynthModel(cfg, 9, lrs.LoadQuantization.Q4KM)
    prompt = lrs.prompt_tokens(9, 20, cfg.vocab_size)
    m = lrs.CudaQwen2Model(backend, sm.desc(), max_seq_len=256, max_sequences=2)
    la, aa = m.prefill(prompt, 0, seq=0)
    for i, t in enumerate(prompt[:-1]):
        assert m.forward_token(int(t), i, lrs.LogitsMode.SKIP, seq=1) is None
    lb, ab = m.forward_token(int(prompt[-1]), len(prompt) - 1, lrs.LogitsMode.COMPUTE, seq=1)
    assert np.abs(la - lb).max() < 1e-4 and aa == ab


def test_batched_sequences_match_single(lrs, orc, backend):
    """Data-parallel decode: B independent sequences in one step == each alone."""
    cfg = _cfg(lrs, 512, 1024, 8, 2, 2, 3000, 64, False)
    sm = lrs.SynthModel(cfg, 4, lrs.LoadQuantization.Q4KM)
    B, n_prompt, n_dec = 5, 33, 24
    m = lrs.CudaQwen2Model(backend, sm.desc(), max_seq_len=512, max_sequences=B)
    firsts, refs = [], []
    for s in range(B):
        prompt = lrs.prompt_tokens(100 + s, n_prompt + s, cfg.vocab_size)
        _, f = m.prefill(prompt, 0, seq=s)
        firsts.append(f)
        refs.append(orc.OracleModel(sm.desc(), 512).benchmark_tokens(prompt, n_dec))
    produced = m.decode_greedy(firsts, [n_prompt + s for s in range(B)], n_dec, list(range(B)))
    fed = np.concatenate([np.array(firsts, np.uint32)[None, :], produced[:-1]], axis=0)
    for s in range(B):
        _assert_tokens(refs[s], fed[:, s])


def test_kv_bf16_option_runs(lrs, orc, backend):
    cfg = _cfg(lrs, 512, 1024, 4, 2, 2, 2000, 128, True)
    sm, model, prompt, ref, logits, first, toks = _run_pair(
        lrs, orc, backend, cfg, lrs.LoadQuantization.Q4KM, 6, 40, 8, kv_bf16=True)
    assert np.abs(logits - ref["logits"][0]).max() < LOGIT_TOL


@pytest.mark.parametrize("case", ["c0", "c3_2layers"])
def test_kv_bf16_greedy_128_steps(lrs, orc, backend, case):
    """The paged bf16 KV cache against the reference's f32 cache over 128
    greedy steps.  bf16 rounds K and V to 8 bits of mantissa, so a step whose
    top-1/top-2 logit margin is within that rounding may pick the other token:
    the tokens must match up to the first step where the oracle's margin is
    below 5e-3.  The prompt's logits are held to 5e-2 max-abs: the KV rows of
    a whole 64-token prompt are rounded, and on the c3 widths that moves a
    logit by up to ~3e-2, past the 2e-2 bar of the f32 cache."""
    if case == "c0":
        cfg, seed, n_prompt = lrs.config_c0(), 0, 128
    else:
        cfg, seed, n_prompt = lrs.config_c3(), 2, 64
        cfg.num_hidden_layers = 2
    sm, model, prompt, ref, logits, first, toks = _run_pair(
        lrs, orc, backend, cfg, lrs.LoadQuantization.Q4KM, seed, n_prompt, 128, max_seq=512,
        kv_bf16=True)
    err = float(np.abs(logits - ref["logits"][0]).max())
    print(f"bf16 KV {case}: prompt logits max-abs error {err:.3e}")
    assert err < 5e-2
    want = ref["tokens"]
    diff = np.nonzero(want != toks)[0]
    close = np.nonzero(ref["margins"][:len(want)] < 5e-3)[0]
    first_close = int(close[0]) if close.size else len(want)
    if diff.size:
        i = int(diff[0])
        print(f"bf16 KV {case}: tokens diverge at step {i} (oracle margin {ref['margins'][i]:.2e})")
        assert i >= first_close, (f"bf16 KV: tokens diverge at step {i} with oracle margin "
                                  f"{ref['margins'][i]:.2e}")
    else:
        print(f"bf16 KV {case}: 128 tokens match")


def test_errors_like_reference(lrs, backend):
    cfg = _cfg(lrs, 256, 512, 4, 2, 1, 300, 64, True)
    sm = lrs.SynthModel(cfg, 1, lrs.LoadQuantization.Q4K)
    m = lrs.CudaQwen2Model(backend, sm.desc(), max_seq_len=64)
    with pytest.raises(lrs.LrsError, match="outside vocabulary"):
        m.forward_token(300, 0)
    with pytest.raises(lrs.LrsError, match="exceeds configured context"):
        m.forward_token(1, 64)
    with pytest.raises(lrs.LrsError, match="at least one token"):
        m.prefill([], 0)


def test_c0_shape_benchmark_workload(lrs, orc, backend):
    """benchmark config 0: Qwen2.5-0.5B shape, seed 0, q4km, prompt 128 + 32 greedy tokens."""
    sm, model, prompt, ref, logits, first, toks = _run_pair(
        lrs, orc, backend, lrs.config_c0(), lrs.LoadQuantization.Q4KM, 0, 128, 32, max_seq=4096)
    assert np.abs(logits - ref["logits"][0]).max() < LOGIT_TOL
    _assert_tokens(ref, toks)


def test_c3_width_two_layers(lrs, orc, backend):
    """Qwen2.5-7B widths (q4km: Q4_K / Q8_0 / Q6_K, untied head) with 2 layers, 128 greedy steps."""
    cfg = lrs.config_c3()
    cfg.num_hidden_layers = 2
    sm, model, prompt, ref, logits, first, toks = _run_pair(
        lrs, orc, backend, cfg, lrs.LoadQuantization.Q4KM, 2, 16, 128, max_seq=4096)
    assert np.abs(logits - ref["logits"][0]).max() < LOGIT_TOL
    _assert_tokens(ref, toks)


def test_c3_width_64_sequences(lrs, orc, backend):
    """The c3 data-parallel decode shape: 64 sequences per step at Qwen2.5-7B widths
    (2 layers); sequences 0, 31 and 63 are checked against the oracle."""
    cfg = lrs.config_c3()
    cfg.num_hidden_layers = 2
    sm = lrs.SynthModel(cfg, 3, lrs.LoadQuantization.Q4KM)
    B, n_dec = 64, 16
    m = lrs.CudaQwen2Model(backend, sm.desc(), max_seq_len=256, max_sequences=B)
    prompts = [lrs.prompt_tokens(200 + s, 8 + s % 5, cfg.vocab_size) for s in range(B)]
    firsts = [m.prefill(p, 0, seq=s)[1] for s, p in enumerate(prompts)]
    produced = m.decode_greedy(firsts, [len(p) for p in prompts], n_dec, list(range(B)))
    fed = np.concatenate([np.array(firsts, np.uint32)[None, :], produced[:-1]], axis=0)
    for s in (0, 31, 63):
        ref = orc.OracleModel(sm.desc(), 256).benchmark_tokens(prompts[s], n_dec)
        _assert_tokens(ref, fed[:, s])


def test_model_from_gguf_file(lrs, orc, backend, tmp_path):
    """A q4km model written as GGUF and loaded through lrs_gguf_qwen2_desc
    (tensors uploaded straight from the mapped file) decodes like the oracle."""
    cfg = _cfg(lrs, 512, 1024, 8, 2, 2, 2000, 64, False)
    sm = lrs.SynthModel(cfg, 12, lrs.LoadQuantization.Q4KM)
    path = str(tmp_path / "m.gguf")
    lrs.write_qwen2_gguf(path, sm.desc())
    g = lrs.GgufFile(path)
    model = lrs.CudaQwen2Model(backend, g.qwen2_desc(lrs.LoadQuantization.Q4KM), max_seq_len=256)
    prompt = lrs.prompt_tokens(12, 30, cfg.vocab_size)
    ref = orc.OracleModel(sm.desc(), 256).benchmark_tokens(prompt, 16, keep_logits=True)
    logits, first = model.prefill(prompt, 0)
    produced = model.decode_greedy([first], [len(prompt)], 16)[:, 0]
    assert np.abs(logits - ref["logits"][0]).max() < LOGIT_TOL
    _assert_tokens(ref, np.concatenate([[first], produced[:-1]]))
    model.close()


def test_c2_width_two_layers(lrs, orc, backend):
    """Qwen2.5-1.5B widths under q4k: every matrix Q4_K, including the tied
    151936-row head (benchmark config 2), 2 layers, batch 1."""
    cfg = lrs.config_c2()
    cfg.num_hidden_layers = 2
    sm, model, prompt, ref, logits, first, toks = _run_pair(
        lrs, orc, backend, cfg, lrs.LoadQuantization.Q4K, 1, 24, 32, max_seq=512)
    assert np.abs(logits - ref["logits"][0]).max() < LOGIT_TOL
    _assert_tokens(ref, toks)


def test_c4_width_batch16(lrs, orc, backend):
    """Qwen2.5-32B widths (hidden 5120, 40/8 heads, intermediate 27648, q4k),
    2 layers: batch 1 and 16 sequences (the tcgen05 path at 16 items)."""
    cfg = lrs.config_c4()
    cfg.num_hidden_layers = 2
    sm, model, prompt, ref, logits, first, toks = _run_pair(
        lrs, orc, backend, cfg, lrs.LoadQuantization.Q4K, 3, 20, 12, max_seq=256)
    assert np.abs(logits - ref["logits"][0]).max() < LOGIT_TOL
    _assert_tokens(ref, toks)
    B, n_dec = 16, 8
    m = lrs.CudaQwen2Model(backend, sm.desc(), max_seq_len=256, max_sequences=B)
    prompts = [lrs.prompt_tokens(600 + s, 10 + s, cfg.vocab_size) for s in range(B)]
    firsts = [m.prefill(p, 0, seq=s)[1] for s, p in enumerate(prompts)]
    produced = m.decode_greedy(firsts, [len(p) for p in prompts], n_dec, list(range(B)))
    fed = np.concatenate([np.array(firsts, np.uint32)[None, :], produced[:-1]], axis=0)
    for s in (0, B - 1):
        r = orc.OracleModel(sm.desc(), 256).benchmark_tokens(prompts[s], n_dec)
        _assert_tokens(r, fed[:, s])

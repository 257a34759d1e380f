"""The stochastic sampler (InferenceEngine::sample_current_logits,
src/engine.rs:253-325) on the device, against the oracle's restatement.

The reference draws u from rand::thread_rng(); both sides take u here, so a
token is a deterministic function of (logits, window, parameters, u).  Equal
values, left unordered by the reference's sort_unstable_by, are ordered
larger index first on both sides.  The reference has no sampler tests: the
oracle (oracle.cpp orc_sample) is checked against a second, pure-Python
restatement below.  Device and oracle agree on every token unless the
oracle's decision lies within 1e-5 (probability units) of its boundary,
where the last-ulp differences of the device expf may flip it.

CPU: Python restatement vs oracle, edge cases, validate_sampling's messages.
GPU: device vs
oracle on full-vocabulary logits, and the model's forward_sample.
"""
import math
import os

import numpy as np
import pytest

F = np.float32


def _total_key(v):
    b = int(np.array([v], F).view(np.int32)[0])
    return b ^ ((b >> 31) & 0x7FFFFFFF)


def py_sample(logits, recent, temperature, top_p, top_k, penalty, u):
    """src/engine.rs:253-325, line by line, in float32 scalars."""
    seen = set(int(t) for t in recent if t < len(logits))
    cand = []
    for t, raw in enumerate(logits):
        value = F(raw)
        if penalty != 1.0 and t in seen:
            value = F(value / F(penalty)) if value > 0 else F(value * F(penalty))
        if temperature > 0.0:
            value = F(value / F(temperature))
        if not np.isfinite(value):
            value = F(-np.inf)
        cand.append((t, value))
    cand.sort(key=lambda c: (_total_key(c[1]), c[0]), reverse=True)
    if temperature <= 0.0:
        return cand[0][0]
    if 0 < top_k < len(cand):
        cand = cand[:top_k]
    mx = cand[0][1]
    vals = [F(np.exp(F(v - mx))) for _, v in cand]
    s = F(0)
    for v in vals:
        s = F(s + v)
    if not np.isfinite(s) or s <= 0:
        return cand[0][0]
    probs = [F(v / s) for v in vals]
    cum, cutoff = F(0), len(cand)
    for i, p in enumerate(probs):
        cum = F(cum + p)
        if cum >= F(top_p):
            cutoff = i + 1
            break
    kept = F(0)
    for p in probs[:cutoff]:
        kept = F(kept + p)
    r = F(F(u) * kept)
    for i in range(cutoff):
        r = F(r - probs[i])
        if r <= 0:
            return cand[i][0]
    return cand[cutoff - 1][0]


def _cases(rng, n_cases, vocab):
    for _ in range(n_cases):
        logits = (rng.standard_normal(vocab) * rng.choice([0.5, 2.0, 6.0])).astype(F)
        recent = rng.integers(0, vocab, size=rng.integers(0, 65)).astype(np.uint32)
        yield dict(logits=logits, recent=recent,
                   temperature=float(rng.choice([0.0, 0.3, 0.7, 1.0, 1.7])),
                   top_p=float(rng.choice([0.05, 0.5, 0.9, 1.0])),
                   top_k=int(rng.choice([1, 2, 40, 333, 0])),
                   penalty=float(rng.choice([1.0, 1.1, 0.8, 2.5])),
                   u=float(rng.random()))


def test_oracle_matches_python_restatement(orc):
    rng = np.random.default_rng(0)
    for c in _cases(rng, 300, 500):
        want = py_sample(c["logits"], c["recent"], c["temperature"], c["top_p"], c["top_k"],
                         c["penalty"], c["u"])
        got, margin = orc.sample(c["logits"], c["recent"], c["temperature"], c["top_p"],
                                 c["top_k"], c["penalty"], c["u"])
        assert got == want or margin < 1e-5, c


def test_oracle_edge_cases(orc):
    l = np.array([1.0, 3.0, 3.0, -2.0, 0.5], F)
    # greedy: the first candidate = last of the equal maxima
    assert orc.sample(l, [], 0.0, 0.9, 40, 1.1, 0.3)[0] == 2
    # repetition penalty divides positive values, multiplies negative ones
    assert orc.sample(l, [2], 0.0, 0.9, 40, 1.5, 0.3)[0] == 1
    assert orc.sample(np.array([-1.0, -1.2], F), [0], 0.0, 0.9, 40, 1.5, 0.0)[0] == 1
    # top_k = 1 and a tiny top_p keep only the first candidate
    assert orc.sample(l, [], 1.0, 0.9, 1, 1.0, 0.99)[0] == 2
    assert orc.sample(l, [], 1.0, 1e-6, 0, 1.0, 0.99)[0] == 2
    # u = 0 takes the first kept candidate
    assert orc.sample(l, [], 1.0, 1.0, 0, 1.0, 0.0)[0] == 2
    # non-finite values become -inf; all -inf: the first candidate (last index)
    nan = np.array([np.nan, 1.0, np.inf], F)
    assert orc.sample(nan, [], 1.0, 1.0, 0, 1.0, 0.99)[0] == 1
    assert orc.sample(np.full(4, -np.inf, F), [], 1.0, 1.0, 0, 1.0, 0.5)[0] == 3


def test_validation_messages(lrs):
    S = lrs.Sampler
    lrs.sampler_check(S(), 151936)
    for bad, msg in [(S(temperature=-0.1), "temperature must be finite and non-negative"),
                     (S(temperature=math.inf), "temperature must be finite and non-negative"),
                     (S(top_p=0.0), r"top_p must be in \(0, 1\]"),
                     (S(top_p=1.5), r"top_p must be in \(0, 1\]"),
                     (S(repetition_penalty=0.0), "repetition_penalty must be finite and positive")]:
        with pytest.raises(lrs.LrsError, match=msg):
            lrs.sampler_check(bad, 151936)
    with pytest.raises(lrs.LrsError, match="top_k must be in 1..4096") as e:
        lrs.sampler_check(S(top_k=0), 151936)
    assert e.value.code == 2  # LRS_ERR_UNSUPPORTED
    lrs.sampler_check(S(top_k=0), 3000)      # the vocabulary itself is small enough
    lrs.sampler_check(S(temperature=0.0, top_k=0), 151936)  # greedy: top_k unused
    # the seen bitmap of the device sampler is in shared memory
    lrs.sampler_check(S(temperature=0.0), 1 << 20)
    with pytest.raises(lrs.LrsError, match="vocabulary too large") as e:
        lrs.sampler_check(S(temperature=0.0), 1 << 22)
    assert e.value.code == 2




@pytest.mark.gpu
@pytest.mark.parametrize("vocab", [151936, 4000, 37])
def test_device_sampler_matches_oracle(lrs, orc, backend, vocab):
    import torch
    rng = np.random.default_rng(vocab)
    n_flip = 0
    for c in _cases(rng, 60, vocab):
        k = c["top_k"]
        if c["temperature"] > 0 and (k == 0 or k >= vocab) and vocab > lrs.SAMPLE_MAX_TOP_K:
            k = 40
        p = lrs.Sampler(c["temperature"], c["top_p"], k, c["penalty"])
        d = torch.from_numpy(c["logits"]).cuda()
        torch.cuda.synchronize()
        got = backend.sample_logits(d.data_ptr(), vocab, p, c["recent"], c["u"])
        want, margin = orc.sample(c["logits"], c["recent"], c["temperature"], c["top_p"], k,
                                  c["penalty"], c["u"])
        if got != want:
            assert margin < 1e-5, (c, got, want, margin)
            n_flip += 1
    assert n_flip <= 2


@pytest.mark.gpu
def test_model_forward_sample_matches_oracle(lrs, orc, backend):
    cfg = lrs.LlamaConfig(512, 1024, 4, 2, 2, 3000, 1e-6, 1e6, 32768, 128, False)
    sm = lrs.SynthModel(cfg, 9, lrs.LoadQuantization.Q4KM)
    prompt = [int(t) for t in lrs.prompt_tokens(9, 20, cfg.vocab_size)]
    model = lrs.CudaQwen2Model(backend, sm.desc(), max_seq_len=256)
    om = orc.OracleModel(sm.desc(), 256)
    logits = om.prefill(np.array(prompt, np.uint32))
    model.prefill(prompt, 0)
    params = lrs.Sampler(0.7, 0.9, 40, 1.1)
    rng = np.random.default_rng(1)
    recent = prompt[-64:]
    tok = prompt[-1]
    pos = len(prompt) - 1
    # the first sampled token comes from the prefill logits on both sides
    u = float(rng.random())
    want, _ = orc.sample(logits, recent, 0.7, 0.9, 40, 1.1, u)
    tok = want
    for step in range(16):
        recent = (recent + [tok])[-64:]
        pos += 1
        u = float(rng.random())
        got = model.forward_sample(tok, pos, params, recent, u)
        want, margin = orc.sample(om.forward_token(tok, pos), recent, 0.7, 0.9, 40, 1.1, u)
        assert got == want or margin < 1e-5, (step, got, want, margin)
        tok = want

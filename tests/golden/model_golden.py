"""Full-depth model fixtures: the reference scalar path (the oracle) run once on
the benchmark configurations, stored as golden outputs for the GPU tests.

The synthetic models are deterministic (counter-based N(0, 0.02) weights,
the reference's encoders), so a GPU box rebuilds the same bytes; the fixture
holds a SHA-256 of every tensor byte of the model it was made from, and the
test checks it before comparing.

Stored per configuration (tests/golden/model_<name>.json):
* the tokens fed to each of the `decode` greedy steps (benchmark_tokens,
  src/engine.rs:189-241) and the oracle's top-1/top-2 margin at each step;
* the logits after the prompt and after the last decode step, at the top 64
  indices of the oracle's logits and at 1024 seeded random indices.

Generation (slow: the literal per-token scalar path, all host cores):
    python tests/golden/model_golden.py c3 c2
"""
import hashlib
import json
import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))

# name: (config function, seed, recipe, prompt tokens, decode steps, layers override)
CASES = {
    "c3": ("config_c3", 2, "Q4KM", 1024, 128, 0),
    "c2": ("config_c2", 1, "Q4K", 512, 128, 0),
}
N_TOP, N_RAND = 64, 1024


def fixture_path(name):
    return os.path.join(HERE, f"model_{name}.json")


def build(lrs, name, threads=0):
    fn, seed, recipe, n_prompt, n_decode, layers = CASES[name]
    cfg = getattr(lrs, fn)()
    if layers:
        cfg.num_hidden_layers = layers
    sm = lrs.SynthModel(cfg, seed, lrs.LoadQuantization[recipe], threads=threads)
    prompt = lrs.prompt_tokens(seed, n_prompt, cfg.vocab_size)
    return cfg, sm, prompt, n_decode


def model_digest(desc, cfg):
    """SHA-256 over every tensor and vector of a model description, in a fixed order."""
    import ctypes as C
    d = desc.contents
    h, kvw = cfg.hidden_size, cfg.num_key_value_heads * cfg.resolved_head_dim()
    sha = hashlib.sha256()

    def blob(ptr, n):
        if ptr:
            sha.update(bytes((C.c_uint8 * n).from_address(ptr)))
        else:
            sha.update(b"-")

    def tens(t):
        sha.update(f"{t.rows}x{t.cols}:{t.ggml_type}".encode())
        blob(t.data, t.nbytes)

    tens(d.embed_tokens)
    tens(d.lm_head)
    blob(d.final_norm, 4 * h)
    for i in range(cfg.num_hidden_layers):
        L = d.layers[i]
        for n in ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj"):
            tens(getattr(L, n))
        for n, ln in (("input_layernorm", h), ("post_attention_layernorm", h), ("q_bias", h),
                      ("k_bias", kvw), ("v_bias", kvw)):
            blob(getattr(L, n), 4 * ln)
    return sha.hexdigest()


def logit_indices(ref_logits, vocab, seed):
    top = np.argsort(ref_logits, kind="stable")[-N_TOP:]
    rnd = np.random.default_rng(seed).choice(vocab, N_RAND, replace=False)
    return np.unique(np.concatenate([top, rnd]))


def make(name):
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import conftest
    import oracle
    lrs = conftest.load_package()
    cfg, sm, prompt, n_decode = build(lrs, name)
    digest = model_digest(sm.desc(), cfg)
    t0 = time.time()
    om = oracle.OracleModel(sm.desc(), len(prompt) + n_decode + 1, oracle.SCALAR, 0)
    ref = om.benchmark_tokens(prompt, n_decode, keep_logits=True)
    took = time.time() - t0
    out = {"case": name, "config": CASES[name][0], "seed": CASES[name][1],
           "recipe": CASES[name][2], "prompt": len(prompt), "decode": n_decode,
           "layers": cfg.num_hidden_layers, "model_sha256": digest,
           "tokens": ref["tokens"].tolist(), "margins": ref["margins"].tolist(),
           "oracle": "oracle/ scalar path (dot_row_scalar, forward_impl), per token",
           "oracle_seconds": round(took, 1), "logits": {}}
    for step in (0, n_decode):
        lg = ref["logits"][step]
        idx = logit_indices(lg, cfg.vocab_size, 1000 + step)
        out["logits"][str(step)] = {"index": idx.tolist(),
                                    "value": [float(v) for v in lg[idx]],
                                    "argmax": int(oracle.argmax(lg))}
    with open(fixture_path(name), "w") as f:
        json.dump(out, f)
    print(f"{name}: {took:.0f} s, digest {digest[:16]}", flush=True)


if __name__ == "__main__":
    for n in sys.argv[1:] or ["c3", "c2"]:
        make(n)

"""Mixed-type GGUF files (Q4_K_M-style quantizations hold several block types
across tensors and layers; README.md:19-20 of the reference runs such files).

An F32 synthetic model is written as GGUF with a per-tensor, per-layer type
mix: q/k/v of up to three types in one layer, o in Q4_K / Q4_1 / Q5_1, gate
and up of different types on odd layers, down in Q6_K / Q5_K, a Q6_K
embedding and a Q8_0 head.  GgufLoader (src/loader.rs:233-398) takes every
tensor as stored.

* CPU: every tensor of the loaded description has the mixed type and the
  bytes of the reference encoder for that type.
* GPU: the model
  decodes like the oracle on the same description, batch 1 and batched.
"""
import os

import numpy as np

from conftest import assert_greedy
import pytest

LOGIT_TOL = 2e-2


def mix_type(lrs, layers):
    QT = lrs.QuantType

    def pick(name, rows, cols):
        if name == "token_embd.weight":
            return QT.Q6_K
        if name == "output.weight":
            return QT.Q8_0
        _, i, kind, _ = name.split(".")
        i = int(i)
        edge = i in (0, layers - 1)
        return {
            "attn_q": QT.Q4_K,
            "attn_k": QT.Q8_0 if i == 1 else QT.Q4_K,
            "attn_v": QT.Q6_K if edge else QT.Q5_0,
            "attn_output": {2: QT.Q4_1, 3: QT.Q5_1}.get(i, QT.Q4_K),
            "ffn_gate": QT.Q4_K,
            "ffn_up": QT.Q5_K if i % 2 else QT.Q4_K,
            "ffn_down": QT.Q6_K if i % 2 == 0 else QT.Q5_K,
        }[kind]
    return pick


def _cfg(lrs):
    return lrs.LlamaConfig(512, 1024, 4, 2, 4, 2000, 1e-6, 1e6, 32768, 128, False)


def _write_mixed(lrs, path, seed=21):
    cfg = _cfg(lrs)
    sm = lrs.SynthModel(cfg, seed, lrs.LoadQuantization.NONE)  # F32 source
    lrs.write_qwen2_gguf(path, sm.desc(), retype=mix_type(lrs, cfg.num_hidden_layers))
    return cfg, sm


NAMES = {"q_proj": "attn_q", "k_proj": "attn_k", "v_proj": "attn_v", "o_proj": "attn_output",
         "gate_proj": "ffn_gate", "up_proj": "ffn_up", "down_proj": "ffn_down"}


def test_mixed_gguf_types_and_bytes(lrs, tmp_path):
    path = str(tmp_path / "mixed.gguf")
    cfg, sm = _write_mixed(lrs, path)
    pick = mix_type(lrs, cfg.num_hidden_layers)
    g = lrs.GgufFile(path)
    d = g.qwen2_desc(lrs.LoadQuantization.NONE).contents
    src = sm.desc().contents

    def check(td, std, name):
        want = pick(name, td.rows, td.cols)
        assert lrs.QuantType(td.ggml_type) == want, name
        vals = np.ctypeslib.as_array((np.ctypeslib.ctypes.c_float * (std.rows * std.cols))
                                     .from_address(std.data))
        ref = lrs.QuantTensor.quantize(vals, std.rows, std.cols, want)
        got = np.ctypeslib.as_array((np.ctypeslib.ctypes.c_uint8 * td.nbytes).from_address(td.data))
        assert td.nbytes == ref.data.size and np.array_equal(got, ref.data), name

    check(d.embed_tokens, src.embed_tokens, "token_embd.weight")
    check(d.lm_head, src.lm_head, "output.weight")
    seen = set()
    for i in range(cfg.num_hidden_layers):
        for field, gname in NAMES.items():
            td = getattr(d.layers[i], field)
            check(td, getattr(src.layers[i], field), f"blk.{i}.{gname}.weight")
            seen.add(td.ggml_type)
    assert len(seen) >= 7  # Q4_K Q8_0 Q6_K Q5_0 Q4_1 Q5_1 Q5_K
    assert any(d.layers[i].gate_proj.ggml_type != d.layers[i].up_proj.ggml_type
               for i in range(cfg.num_hidden_layers))


def test_mixed_gguf_oracle_runs(lrs, orc, tmp_path):
    # the reference's scalar and AVX2 paths agree on the mixed file (the GPU test's oracle)
    path = str(tmp_path / "mixed.gguf")
    cfg, _ = _write_mixed(lrs, path)
    g = lrs.GgufFile(path)
    desc = g.qwen2_desc(lrs.LoadQuantization.NONE)
    prompt = lrs.prompt_tokens(21, 8, cfg.vocab_size)
    a = orc.OracleModel(desc, 64, orc.SCALAR, 0).benchmark_tokens(prompt, 4, keep_logits=True)
    b = orc.OracleModel(desc, 64, orc.AVX2, 0).benchmark_tokens(prompt, 4, keep_logits=True)
    assert np.abs(a["logits"][0] - b["logits"][0]).max() < 1e-3




@pytest.mark.gpu
def test_mixed_gguf_decodes_like_oracle(lrs, orc, backend, tmp_path):
    path = str(tmp_path / "mixed.gguf")
    cfg, _ = _write_mixed(lrs, path)
    g = lrs.GgufFile(path)
    desc = g.qwen2_desc(lrs.LoadQuantization.NONE)
    prompt = lrs.prompt_tokens(21, 40, cfg.vocab_size)
    ref = orc.OracleModel(desc, 256, orc.SCALAR, 0).benchmark_tokens(prompt, 24, keep_logits=True)
    model = lrs.CudaQwen2Model(backend, desc, max_seq_len=256)
    logits, first = model.prefill(prompt, 0)
    assert np.abs(logits - ref["logits"][0]).max() < LOGIT_TOL
    produced = model.decode_greedy([first], [len(prompt)], 24)[:, 0]
    assert_greedy(ref, np.concatenate([[first], produced[:-1]]))
    model.close()


@pytest.mark.gpu
def test_mixed_gguf_batched_sequences(lrs, orc, backend, tmp_path):
    path = str(tmp_path / "mixed.gguf")
    cfg, _ = _write_mixed(lrs, path)
    g = lrs.GgufFile(path)
    desc = g.qwen2_desc(lrs.LoadQuantization.NONE)
    B, n_dec = 6, 12
    m = lrs.CudaQwen2Model(backend, desc, max_seq_len=256, max_sequences=B)
    prompts = [lrs.prompt_tokens(500 + s, 16 + s, cfg.vocab_size) for s in range(B)]
    firsts = [m.prefill(p, 0, seq=s)[1] for s, p in enumerate(prompts)]
    produced = m.decode_greedy(firsts, [len(p) for p in prompts], n_dec, list(range(B)))
    fed = np.concatenate([np.array(firsts, np.uint32)[None, :], produced[:-1]], axis=0)
    for s in (0, B - 1):
        ref = orc.OracleModel(desc, 256).benchmark_tokens(prompts[s], n_dec)
        assert_greedy(ref, fed[:, s])
    m.close()

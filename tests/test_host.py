"""CPU tests of the host side: the C-ABI library, the load recipe and the
synthetic-model builder.  No compute call needs a GPU here."""
import ctypes
import os
import re

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared_symbols():
    names = set()
    for h in ("llamars.h", "llamars_synth.h", "llamars_gguf.h", "llamars_sample.h",
              "llamars_safetensors.h"):
        src = open(os.path.join(ROOT, "include", h)).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        names.update(re.findall(r"\b(lrs_[a-z0-9_]+)\s*\(", src))
    return names


def test_library_exports_every_declared_symbol(lrs):
    lib = lrs.library()
    declared = _declared_symbols()
    assert len(declared) >= 25
    for name in declared:
        assert hasattr(lib, name), name
    assert declared == set(lrs.EXPORTED_SYMBOLS)


def test_library_is_built_for_sm100a():
    so = os.path.join(ROOT, "llama.rs_b200", "libllamars.so")
    assert os.path.exists(so)
    # the fatbin section names its target architecture
    assert b"sm_100a" in open(so, "rb").read()


def test_backend_without_gpu_fails_loudly(lrs):
    try:
        import torch
        if torch.cuda.is_available():
            pytest.skip("a GPU is present")
    except ImportError:
        pass
    with pytest.raises(lrs.LrsError):
        lrs.CudaBackend(0)


def test_type_geometry_matches_reference(lrs):
    lib = lrs.library()
    # QuantType::block_size / type_size, src/quant.rs:46-67
    want = {0: (1, 4), 1: (1, 2), 30: (1, 2), 2: (32, 18), 3: (32, 20), 6: (32, 22),
            7: (32, 24), 8: (32, 34), 12: (256, 144), 13: (256, 176), 14: (256, 210)}
    for t, (bv, bb) in want.items():
        a, b = ctypes.c_uint32(), ctypes.c_uint32()
        assert lib.lrs_type_geometry(t, ctypes.byref(a), ctypes.byref(b)) == 0
        assert (a.value, b.value) == (bv, bb)
    assert lib.lrs_type_geometry(9, None, None) == 2  # Q8_1 is not supported


def test_quant_tensor_validation(lrs):
    with pytest.raises(lrs.LrsError):
        lrs.QuantTensor(np.zeros(10, np.uint8), (1, 32), lrs.QuantType.Q4_0)  # 18 bytes needed
    with pytest.raises(lrs.LrsError):
        lrs.QuantTensor(np.zeros(18, np.uint8), (1, 31), lrs.QuantType.Q4_0)
    with pytest.raises(lrs.LrsError):
        lrs.QuantType.from_ggml_type(9)


def test_recipe_types_match_survey_table(lrs):
    L, Q = lrs.LoadQuantization, lrs.QuantType
    rt = lrs.recipe_type
    # c0 (q4km, hidden 896): no Q4_K anywhere
    assert rt(L.Q4KM, "model.layers.0.self_attn.q_proj.weight", 896, 896) == Q.Q5_0
    assert rt(L.Q4KM, "model.layers.0.self_attn.v_proj.weight", 128, 896) == Q.Q8_0
    assert rt(L.Q4KM, "model.layers.0.mlp.down_proj.weight", 896, 4864) == Q.Q6_K
    assert rt(L.Q4KM, "model.layers.0.mlp.gate_proj.weight", 4864, 896) == Q.Q5_0
    assert rt(L.Q4KM, "model.embed_tokens.weight", 151936, 896) == Q.Q8_0
    # c3 (q4km, hidden 3584)
    assert rt(L.Q4KM, "model.layers.3.self_attn.k_proj.weight", 512, 3584) == Q.Q4_K
    assert rt(L.Q4KM, "model.layers.3.mlp.down_proj.weight", 3584, 18944) == Q.Q6_K
    assert rt(L.Q4KM, "lm_head.weight", 152064, 3584) == Q.Q8_0
    # c2 (q4k): all Q4_K
    assert rt(L.Q4K, "model.layers.0.mlp.down_proj.weight", 1536, 8960) == Q.Q4_K  # 35 * 256
    assert rt(L.Q4K, "model.layers.0.mlp.down_proj.weight", 896, 4864) == Q.Q4_K
    assert rt(L.Q4K, "model.layers.0.self_attn.o_proj.weight", 896, 896) == Q.Q5_0
    assert rt(L.Q4K, "model.layers.0.mlp.up_proj.weight", 8960, 1536) == Q.Q4_K
    assert rt(L.NONE, "lm_head.weight", 10, 32) == Q.F32


def test_synth_values_are_counter_based(lrs):
    a = lrs.synth_values(7, "model.layers.1.mlp.up_proj.weight", 1000)
    b = lrs.synth_values(7, "model.layers.1.mlp.up_proj.weight", 400, offset=600)
    assert np.array_equal(a[600:], b)
    c = lrs.synth_values(8, "model.layers.1.mlp.up_proj.weight", 1000)
    assert not np.array_equal(a, c)
    big = lrs.synth_values(1, "x", 200000)
    assert abs(big.mean()) < 3e-4 and abs(big.std() - 0.02) < 3e-4


def _tiny_config(lrs, tied=True):
    return lrs.LlamaConfig(hidden_size=256, intermediate_size=512, num_attention_heads=4,
                           num_key_value_heads=2, num_hidden_layers=2, vocab_size=1000,
                           rms_norm_eps=1e-6, rope_theta=1e6, max_position_embeddings=4096,
                           head_dim=64, tie_word_embeddings=tied)


def test_synth_model_is_deterministic_and_follows_recipe(lrs):
    cfg = _tiny_config(lrs)
    a = lrs.SynthModel(cfg, 0, lrs.LoadQuantization.Q4KM, threads=3)
    b = lrs.SynthModel(cfg, 0, lrs.LoadQuantization.Q4KM, threads=1)
    for name in ("q_proj", "v_proj", "down_proj", "gate_proj"):
        ta, tb = a.tensor(name, 1), b.tensor(name, 1)
        assert ta.quant_type == tb.quant_type
        assert np.array_equal(ta.data, tb.data)
    assert a.tensor("q_proj", 0).quant_type == lrs.QuantType.Q4_K
    assert a.tensor("v_proj", 0).quant_type == lrs.QuantType.Q8_0
    assert a.tensor("down_proj", 0).quant_type == lrs.QuantType.Q6_K
    d = a.desc().contents
    assert d.lm_head.data == d.embed_tokens.data  # tied head reuses the quantized embedding


def test_model_file_round_trip(lrs, tmp_path):
    """save_model_file / ModelFile reproduce the synthetic model byte for byte."""
    for tied in (True, False):
        cfg = lrs.LlamaConfig(256, 512, 4, 2, 2, 300, 1e-6, 1e6, 4096, 64, tied)
        sm = lrs.SynthModel(cfg, 7, lrs.LoadQuantization.Q4KM)
        path = str(tmp_path / f"m{int(tied)}.lrs")
        lrs.save_model_file(sm.desc(), path)
        mf = lrs.ModelFile(path)
        got = mf.config
        assert abs(got.rms_norm_eps - cfg.rms_norm_eps) < 1e-12
        got.rms_norm_eps = cfg.rms_norm_eps
        assert got == cfg
        for name in ("embed", "lm_head"):
            a = sm.tensor(name)
            d = mf.desc().contents
            td = d.embed_tokens if name == "embed" else d.lm_head
            b = np.ctypeslib.as_array((ctypes.c_uint8 * td.nbytes).from_address(td.data))
            assert td.ggml_type == int(a.quant_type) and np.array_equal(a.data, b)
        for i in range(cfg.num_hidden_layers):
            for n in ("q_proj", "v_proj", "down_proj"):
                a = sm.tensor(n, i)
                td = getattr(mf.desc().contents.layers[i], n)
                b = np.ctypeslib.as_array((ctypes.c_uint8 * td.nbytes).from_address(td.data))
                assert np.array_equal(a.data, b)
            for n, width in (("input_layernorm", 256), ("k_bias", 128)):
                pa = getattr(sm.desc().contents.layers[i], n)
                pb = getattr(mf.desc().contents.layers[i], n)
                assert np.array_equal(np.ctypeslib.as_array((ctypes.c_float * width).from_address(pa)),
                                      np.ctypeslib.as_array((ctypes.c_float * width).from_address(pb)))


def _c_param_counts():
    """name -> number of parameters of every lrs_* function in include/*.h."""
    counts = {}
    for h in ("llamars.h", "llamars_synth.h", "llamars_gguf.h", "llamars_sample.h",
              "llamars_safetensors.h"):
        src = open(os.path.join(ROOT, "include", h)).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        for name, params in re.findall(r"\b(lrs_[a-z0-9_]+)\s*\(([^;{]*?)\)\s*;", src, flags=re.S):
            p = params.strip()
            counts[name] = 0 if p in ("", "void") else p.count(",") + 1
    return counts


def test_integration_rust_bindings_match_the_headers():
    """The Rust `extern "C"` block a maintainer adds to the reference
     binds functions the headers declare, with the same
    number of parameters."""
    md = open(os.path.join(ROOT, "INTEGRATION.md")).read()
    decls = re.findall(r"pub fn (lrs_[a-z0-9_]+)\s*\(([^;]*?)\)\s*(?:->[^;]*)?;", md, flags=re.S)
    assert len(decls) >= 15
    c = _c_param_counts()
    for name, params in decls:
        params = re.sub(r"/\*.*?\*/", "", params, flags=re.S)
        n = 0 if not params.strip() else params.count(",") + 1
        assert name in c, f"{name} is bound in INTEGRATION.md but not declared"
        assert n == c[name], f"{name}: {n} parameters in INTEGRATION.md, {c[name]} in the header"

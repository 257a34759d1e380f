"""SafeTensors checkpoints and ModelLoader::load's format dispatch (host, no
GPU): SafetensorStore / SafetensorsLoader (src/loader.rs:80-230, 535-645) and
LlamaConfig::from_json (src/config.rs) restated in csrc/safetensors.cpp.

* an F32 checkpoint loaded with q4k / q4km holds the bytes of the synthetic
  model built with that recipe (maybe_quantize on the Hugging Face names);
* F16 / BF16 checkpoints: views without a recipe, the encoders with one;
* one file and index-sharded directories give the same description;
* tied heads, absent q/k/v biases, the reference's error messages;
* ModelLoader::load picks GGUF or SafeTensors as the reference does.
"""
import ctypes
import json
import os

import numpy as np

from conftest import assert_greedy
import pytest

MATS = ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj")


def _cfg(lrs, tied):
    return lrs.LlamaConfig(512, 1024, 4, 2, 2, 1000, 1e-6, 1e6, 32768, 128, tied)


def _bytes(td):
    return bytes((ctypes.c_uint8 * td.nbytes).from_address(td.data))


def _f32(ptr, n):
    return np.frombuffer((ctypes.c_float * n).from_address(ptr), dtype=np.float32).copy()


def _same_desc(a, b, kvw):
    a, b = a.contents, b.contents
    for f in ("hidden_size", "intermediate_size", "num_attention_heads", "num_key_value_heads",
              "num_hidden_layers", "vocab_size", "head_dim"):
        assert getattr(a.config, f) == getattr(b.config, f), f
    assert a.config.rms_norm_eps == b.config.rms_norm_eps
    assert a.config.rope_theta == b.config.rope_theta
    h = a.config.hidden_size
    for name in ("embed_tokens", "lm_head"):
        ta, tb = getattr(a, name), getattr(b, name)
        assert ta.ggml_type == tb.ggml_type and _bytes(ta) == _bytes(tb), name
    assert np.array_equal(_f32(a.final_norm, h), _f32(b.final_norm, h))
    for i in range(a.config.num_hidden_layers):
        La, Lb = a.layers[i], b.layers[i]
        for m in MATS:
            ta, tb = getattr(La, m), getattr(Lb, m)
            assert (ta.rows, ta.cols, ta.ggml_type) == (tb.rows, tb.cols, tb.ggml_type), (i, m)
            assert _bytes(ta) == _bytes(tb), (i, m)
        for v, n in (("input_layernorm", h), ("post_attention_layernorm", h), ("q_bias", h),
                     ("k_bias", kvw), ("v_bias", kvw)):
            pa, pb = getattr(La, v), getattr(Lb, v)
            if pa or pb:
                assert np.array_equal(_f32(pa, n), _f32(pb, n)), (i, v)


@pytest.mark.parametrize("tied", [False, True])
@pytest.mark.parametrize("recipe", ["NONE", "Q4K", "Q4KM"])
def test_f32_checkpoint_matches_synthetic_recipe(lrs, tmp_path, recipe, tied):
    cfg = _cfg(lrs, tied)
    src = lrs.SynthModel(cfg, 4, lrs.LoadQuantization.NONE)
    lrs.write_qwen2_safetensors(str(tmp_path), src.desc())
    st = lrs.SafetensorsFile(str(tmp_path))
    got = st.qwen2_desc(lrs.LoadQuantization[recipe])
    want = lrs.SynthModel(cfg, 4, lrs.LoadQuantization[recipe])
    _same_desc(got, want.desc(), 2 * 128)
    d = got.contents
    assert (d.lm_head.data == d.embed_tokens.data) == tied


def test_sharded_equals_single_file(lrs, tmp_path):
    cfg = _cfg(lrs, False)
    src = lrs.SynthModel(cfg, 5, lrs.LoadQuantization.NONE)
    one, three = tmp_path / "one", tmp_path / "three"
    lrs.write_qwen2_safetensors(str(one), src.desc())
    lrs.write_qwen2_safetensors(str(three), src.desc(), shards=3)
    assert os.path.exists(three / "model.safetensors.index.json")
    a = lrs.SafetensorsFile(str(one))
    b = lrs.SafetensorsFile(str(three))
    assert a.tensor_count == b.tensor_count
    _same_desc(a.qwen2_desc(lrs.LoadQuantization.Q4KM), b.qwen2_desc(lrs.LoadQuantization.Q4KM), 256)


@pytest.mark.parametrize("dtype", ["F16", "BF16"])
def test_half_checkpoints(lrs, tmp_path, dtype):
    cfg = _cfg(lrs, False)
    src = lrs.SynthModel(cfg, 6, lrs.LoadQuantization.NONE)
    lrs.write_qwen2_safetensors(str(tmp_path), src.desc(), dtype=dtype)
    st = lrs.SafetensorsFile(str(tmp_path))
    q = st.tensor("model.layers.1.self_attn.q_proj.weight")
    assert q.quant_type == lrs.QuantType[dtype] and q.shape == (512, 512)
    # no recipe: the half-precision view itself
    d0 = st.qwen2_desc(lrs.LoadQuantization.NONE).contents
    assert d0.layers[1].q_proj.ggml_type == int(lrs.QuantType[dtype])
    # q4km: the encoders on the widened values (QuantTensor::to_vec_f32)
    d1 = st.qwen2_desc(lrs.LoadQuantization.Q4KM).contents
    vals = st.tensor("model.layers.0.mlp.down_proj.weight")  # a view: st stays open
    f32 = _widen(vals, dtype)
    ref = lrs.QuantTensor.quantize(f32, 512, 1024, lrs.QuantType.Q6_K)
    td = d1.layers[0].down_proj
    assert td.ggml_type == int(lrs.QuantType.Q6_K) and _bytes(td) == ref.data.tobytes()
    # norms are widened to f32
    n = _f32(d1.final_norm, 512)
    assert np.array_equal(n, _widen(st.tensor("model.norm.weight"), dtype))


def _widen(t, dtype):
    raw = np.asarray(t.data)
    if dtype == "F16":
        return raw.view(np.float16).astype(np.float32)
    return (raw.view(np.uint16).astype(np.uint32) << 16).view(np.float32)


def test_missing_biases_are_zero(lrs, tmp_path):
    cfg = _cfg(lrs, False)
    src = lrs.SynthModel(cfg, 7, lrs.LoadQuantization.NONE)
    lrs.write_qwen2_safetensors(str(tmp_path), src.desc())
    _drop(lrs, tmp_path, {"model.layers.0.self_attn.k_proj.bias"})
    d = lrs.SafetensorsFile(str(tmp_path)).qwen2_desc().contents
    assert not d.layers[0].k_bias and d.layers[0].q_bias and d.layers[1].k_bias


def _drop(lrs, model_dir, names):
    """Rewrites model.safetensors without `names`."""
    st = lrs.SafetensorsFile(str(model_dir))
    path = os.path.join(str(model_dir), "model.safetensors")
    with open(path, "rb") as f:
        n = int.from_bytes(f.read(8), "little")
        header = json.loads(f.read(n))
        data = f.read()
    keep = [(k, v) for k, v in header.items() if k != "__metadata__" and k not in names]
    keep.sort(key=lambda kv: kv[1]["data_offsets"][0])
    tensors = [(k, v["dtype"], v["shape"], data[v["data_offsets"][0]:v["data_offsets"][1]])
               for k, v in keep]
    st.close()
    lrs.write_safetensors(path, tensors)


def _write_raw(path, header: dict, data: bytes, pad=True):
    h = json.dumps(header).encode()
    if pad:
        h += b" " * ((8 - len(h) % 8) % 8)
    with open(path, "wb") as f:
        f.write(len(h).to_bytes(8, "little") + h + data)


def test_errors_like_reference(lrs, tmp_path):
    cfg = _cfg(lrs, False)
    src = lrs.SynthModel(cfg, 8, lrs.LoadQuantization.NONE)
    d = tmp_path / "m"
    lrs.write_qwen2_safetensors(str(d), src.desc())
    cfg_path = d / "config.json"
    good = json.loads(cfg_path.read_text())

    def load():
        return lrs.SafetensorsFile(str(d)).qwen2_desc()

    def with_config(**change):
        c = dict(good)
        for k, v in change.items():
            if v is None:
                c.pop(k, None)
            else:
                c[k] = v
        cfg_path.write_text(json.dumps(c))

    with_config(model_type=None)
    with pytest.raises(lrs.LrsError, match="config.json is missing model_type"):
        load()
    with_config(model_type="llama")
    with pytest.raises(lrs.LrsError, match='unsupported Hugging Face model_type "llama"'):
        load()
    with_config(hidden_size=None)
    with pytest.raises(lrs.LrsError, match="missing field `hidden_size`"):
        load()
    with_config(num_key_value_heads=3)
    with pytest.raises(lrs.LrsError, match="num_attention_heads must be divisible by num_key_value_heads"):
        load()
    with_config(head_dim=64)
    with pytest.raises(lrs.LrsError, match="num_attention_heads \\* head_dim must equal hidden_size"):
        load()
    with_config(rms_norm_eps=-1.0)
    with pytest.raises(lrs.LrsError, match="rms_norm_eps must be finite and positive"):
        load()
    with_config(rope_theta=0.0)
    with pytest.raises(lrs.LrsError, match="rope_theta must be finite and positive"):
        load()
    with_config(vocab_size=999)
    with pytest.raises(lrs.LrsError, match=r"tensor model.embed_tokens.weight has shape \[1000, 512\], "
                                           r"expected \[999, 512\]"):
        load()
    with_config()
    load()  # back to a valid config
    _drop(lrs, d, {"model.norm.weight"})
    with pytest.raises(lrs.LrsError, match="missing safetensors tensor model.norm.weight"):
        load()
    os.remove(cfg_path)
    with pytest.raises(lrs.LrsError, match="failed to read .*config.json"):
        load()

    e = tmp_path / "empty"
    e.mkdir()
    with pytest.raises(lrs.LrsError, match="no .safetensors files in"):
        lrs.SafetensorsFile(str(e))

    bad = tmp_path / "bad"
    bad.mkdir()
    x = np.zeros(4, np.float32).tobytes()
    _write_raw(bad / "a.safetensors", {"x": {"dtype": "F32", "shape": [4], "data_offsets": [0, 16]}}, x)
    _write_raw(bad / "b.safetensors", {"x": {"dtype": "F32", "shape": [4], "data_offsets": [0, 16]}}, x)
    with pytest.raises(lrs.LrsError, match="duplicate safetensors tensor x"):
        lrs.SafetensorsFile(str(bad))
    os.remove(bad / "b.safetensors")
    _write_raw(bad / "a.safetensors", {"x": {"dtype": "F32", "shape": [4], "data_offsets": [0, 12]},
                                       "y": {"dtype": "F32", "shape": [1], "data_offsets": [12, 16]}}, x)
    with pytest.raises(lrs.LrsError, match="invalid safetensors file .*do not match its dtype and shape"):
        lrs.SafetensorsFile(str(bad))
    _write_raw(bad / "a.safetensors", {"x": {"dtype": "F32", "shape": [3], "data_offsets": [4, 16]}}, x)
    with pytest.raises(lrs.LrsError, match="invalid safetensors file .*gap or overlap"):
        lrs.SafetensorsFile(str(bad))
    _write_raw(bad / "a.safetensors", {"x": {"dtype": "I64", "shape": [2], "data_offsets": [0, 16]}}, x)
    st = lrs.SafetensorsFile(str(bad))
    with pytest.raises(lrs.LrsError, match="unsupported safetensors dtype I64; use F32/F16/BF16"):
        st.tensor("x")
    with open(bad / "a.safetensors", "wb") as f:
        f.write((10 ** 9).to_bytes(8, "little") + b"{}")
    with pytest.raises(lrs.LrsError, match="header too large"):
        lrs.SafetensorsFile(str(bad))


def test_model_loader_dispatch(lrs, tmp_path):
    cfg = _cfg(lrs, True)
    src = lrs.SynthModel(cfg, 9, lrs.LoadQuantization.NONE)
    st_dir = tmp_path / "hf"
    lrs.write_qwen2_safetensors(str(st_dir), src.desc())
    want = lrs.SynthModel(cfg, 9, lrs.LoadQuantization.Q4KM)
    # a directory with model.safetensors, and the .safetensors file itself
    for p in (st_dir, st_dir / "model.safetensors"):
        m = lrs.LoadedModel(str(p), lrs.LoadQuantization.Q4KM)
        _same_desc(m.desc(), want.desc(), 256)
    # a directory with a single GGUF file, and the file itself
    g_dir = tmp_path / "gg"
    g_dir.mkdir()
    lrs.write_qwen2_gguf(str(g_dir / "m.gguf"), want.desc())
    for p in (g_dir, g_dir / "m.gguf"):
        m = lrs.LoadedModel(str(p), lrs.LoadQuantization.NONE)
        _same_desc(m.desc(), want.desc(), 256)
    lrs.write_qwen2_gguf(str(g_dir / "n.gguf"), want.desc())
    with pytest.raises(lrs.LrsError, match="contains multiple GGUF files; pass the desired file explicitly"):
        lrs.LoadedModel(str(g_dir))
    with pytest.raises(lrs.LrsError, match="cannot detect model format at"):
        lrs.LoadedModel(str(tmp_path / "nothing-here"))


def test_oracle_decodes_the_loaded_model(lrs, orc, tmp_path):
    # the description from disk drives the reference loop like the in-memory one
    cfg = _cfg(lrs, False)
    src = lrs.SynthModel(cfg, 10, lrs.LoadQuantization.NONE)
    lrs.write_qwen2_safetensors(str(tmp_path), src.desc(), dtype="BF16")
    m = lrs.LoadedModel(str(tmp_path), lrs.LoadQuantization.Q4KM)
    prompt = lrs.prompt_tokens(10, 12, cfg.vocab_size)
    a = orc.OracleModel(m.desc(), 64).benchmark_tokens(prompt, 6)
    b = orc.OracleModel(m.desc(), 64).benchmark_tokens(prompt, 6)
    assert np.array_equal(a["tokens"], b["tokens"])


@pytest.mark.gpu
def test_safetensors_model_decodes_like_oracle(lrs, orc, backend, tmp_path):
    cfg = _cfg(lrs, False)
    src = lrs.SynthModel(cfg, 11, lrs.LoadQuantization.NONE)
    lrs.write_qwen2_safetensors(str(tmp_path), src.desc(), dtype="BF16")
    m = lrs.LoadedModel(str(tmp_path), lrs.LoadQuantization.Q4KM)
    prompt = lrs.prompt_tokens(11, 30, cfg.vocab_size)
    ref = orc.OracleModel(m.desc(), 256).benchmark_tokens(prompt, 16, keep_logits=True)
    model = lrs.CudaQwen2Model(backend, m.desc(), max_seq_len=256)
    logits, first = model.prefill(prompt, 0)
    assert np.abs(logits - ref["logits"][0]).max() < 2e-2
    produced = model.decode_greedy([first], [len(prompt)], 16)[:, 0]
    assert_greedy(ref, np.concatenate([[first], produced[:-1]]))


def test_config_json_forms(lrs, tmp_path):
    """config.json as Hugging Face writes it: unknown and nested fields are
    ignored (serde), numbers in any JSON form, escapes in strings."""
    cfg = _cfg(lrs, True)
    src = lrs.SynthModel(cfg, 12, lrs.LoadQuantization.NONE)
    lrs.write_qwen2_safetensors(str(tmp_path), src.desc())
    text = r"""{
      "architectures": ["Qwen2ForCausalLM"], "model_type": "qwen2",
      "name_or_path": "café 😀 \"quoted\" \\ \/",
      "rope_scaling": {"type": "yarn", "factor": 4.0, "nested": [1, [2, {"x": null}]]},
      "hidden_size": 512, "intermediate_size": 1024, "num_attention_heads": 4,
      "num_key_value_heads": 2, "num_hidden_layers": 2, "vocab_size": 1000,
      "rms_norm_eps": 1E-06, "rope_theta": 1.0e6, "max_position_embeddings": 32768,
      "head_dim": null, "tie_word_embeddings": true, "use_cache": false
    }"""
    (tmp_path / "config.json").write_text(text)
    d = lrs.SafetensorsFile(str(tmp_path)).qwen2_desc().contents
    assert d.config.head_dim == 128 and d.config.rms_norm_eps == np.float32(1e-6)
    assert d.config.rope_theta == np.float32(1e6) and d.config.max_position_embeddings == 32768
    for bad, msg in [('{"model_type": "qwen2", "hidden_size": 5.5}', "model_type|invalid type"),
                     ('{"model_type": "qwen2",}', "invalid config.json"),
                     ('{"model_type": "qwen2" "x": 1}', "invalid config.json"),
                     ('{"model_type": "\\ud800"}', "invalid config.json"),
                     ('[1, 2]', "missing model_type")]:
        (tmp_path / "config.json").write_text(bad)
        with pytest.raises(lrs.LrsError, match=msg):
            lrs.SafetensorsFile(str(tmp_path)).qwen2_desc()


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", ["F32", "BF16"])
def test_device_recipe_equals_host_recipe(lrs, backend, tmp_path, dtype):
    """maybe_quantize on the GPU (lrs_model_options.device_recipe): the float
    checkpoint encoded at model creation gives bit-identical logits to the
    host-encoded description."""
    cfg = _cfg(lrs, False)
    src = lrs.SynthModel(cfg, 13, lrs.LoadQuantization.NONE)
    lrs.write_qwen2_safetensors(str(tmp_path), src.desc(), dtype=dtype)
    raw = lrs.LoadedModel(str(tmp_path), lrs.LoadQuantization.NONE)
    host = lrs.LoadedModel(str(tmp_path), lrs.LoadQuantization.Q4KM)
    prompt = lrs.prompt_tokens(13, 24, cfg.vocab_size)
    a = lrs.CudaQwen2Model(backend, raw.desc(), max_seq_len=128,
                           device_recipe=lrs.LoadQuantization.Q4KM)
    b = lrs.CudaQwen2Model(backend, host.desc(), max_seq_len=128)
    la, fa = a.prefill(prompt, 0)
    lb, fb = b.prefill(prompt, 0)
    assert np.array_equal(la, lb) and fa == fb
    assert np.array_equal(a.decode_greedy([fa], [24], 12), b.decode_greedy([fb], [24], 12))

"""GGUF reader and Qwen2 loader (host, no GPU): src/gguf.rs and
src/loader.rs:231-398 restated in csrc/gguf.cpp.

* the reference's own test (gguf.rs `parses_a_minimal_v3_file`);
* a pre-quantized synthetic model written as GGUF and read back: every byte,
  type and config field identical, tied and untied heads;
* an F32 GGUF quantized at load time with the q4k / q4km recipes gives the
  same bytes as the synthetic model built with that recipe (maybe_quantize on
  GGUF names);
* malformed files fail with the reference's messages.
"""
import ctypes
import struct

import numpy as np
import pytest


def _put_string(out: bytearray, value: str):
    out += struct.pack("<Q", len(value)) + value.encode()


def _minimal_v3():
    # bytes of src/gguf.rs:382-401
    b = bytearray(b"GGUF")
    b += struct.pack("<I", 3)
    b += struct.pack("<Q", 1)  # tensors
    b += struct.pack("<Q", 1)  # metadata
    _put_string(b, "general.alignment")
    b += struct.pack("<I", 4)  # UINT32
    b += struct.pack("<I", 4)
    _put_string(b, "x")
    b += struct.pack("<I", 2)
    b += struct.pack("<Q", 2)  # columns
    b += struct.pack("<Q", 2)  # rows
    b += struct.pack("<I", 0)  # F32
    b += struct.pack("<Q", 0)
    while len(b) % 4:
        b.append(0)
    for v in (1.0, 2.0, 3.0, 4.0):
        b += struct.pack("<f", v)
    return bytes(b)


def test_parses_a_minimal_v3_file(lrs, tmp_path):
    path = tmp_path / "m.gguf"
    path.write_bytes(_minimal_v3())
    g = lrs.GgufFile(str(path))
    assert g.version == 3 and g.tensor_count == 1
    assert g.metadata_u64("general.alignment") == 4
    t = g.tensor("x")
    assert t.shape == (2, 2)
    assert t.data.view(np.float32).tolist() == [1.0, 2.0, 3.0, 4.0]


def _tensors(desc):
    d = desc.contents
    out = {"embed": d.embed_tokens, "lm_head": d.lm_head}
    for i in range(d.config.num_hidden_layers):
        for n in ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj"):
            out[f"{i}.{n}"] = getattr(d.layers[i], n)
    return out


def _bytes(td):
    return ctypes.string_at(td.data, td.nbytes)


def _vec(ptr, n):
    return None if not ptr else np.ctypeslib.as_array((ctypes.c_float * n).from_address(ptr)).copy()


def _same_model(a, b):
    da, db = a.contents, b.contents
    for k, _ in da.config._fields_:
        assert getattr(da.config, k) == getattr(db.config, k), k
    ta, tb = _tensors(a), _tensors(b)
    for k in ta:
        assert ta[k].ggml_type == tb[k].ggml_type, k
        assert (ta[k].rows, ta[k].cols) == (tb[k].rows, tb[k].cols), k
        assert _bytes(ta[k]) == _bytes(tb[k]), k
    assert (da.lm_head.data == da.embed_tokens.data) == (db.lm_head.data == db.embed_tokens.data)
    h, kvw = da.config.hidden_size, da.config.num_key_value_heads * da.config.head_dim
    assert np.array_equal(_vec(da.final_norm, h), _vec(db.final_norm, h))
    for i in range(da.config.num_hidden_layers):
        for n, w in (("input_layernorm", h), ("post_attention_layernorm", h), ("q_bias", h),
                     ("k_bias", kvw), ("v_bias", kvw)):
            va, vb = _vec(getattr(da.layers[i], n), w), _vec(getattr(db.layers[i], n), w)
            assert (va is None and vb is None) or np.array_equal(va, vb), (i, n)


def _cfg(lrs, tied):
    return lrs.LlamaConfig(512, 1024, 8, 2, 2, 1000, 1e-6, 1e6, 4096, 64, tied)


@pytest.mark.parametrize("tied", [True, False])
def test_prequantized_round_trip(lrs, tmp_path, tied):
    sm = lrs.SynthModel(_cfg(lrs, tied), 5, lrs.LoadQuantization.Q4KM)
    path = str(tmp_path / "q4km.gguf")
    lrs.write_qwen2_gguf(path, sm.desc())
    g = lrs.GgufFile(path)
    assert g.metadata_str("general.architecture") == "qwen2"
    # pre-quantized tensors are kept verbatim whatever the load recipe
    for recipe in (lrs.LoadQuantization.NONE, lrs.LoadQuantization.Q4K):
        _same_model(g.qwen2_desc(recipe), sm.desc())


@pytest.mark.parametrize("recipe", ["Q4K", "Q4KM"])
def test_f32_gguf_quantized_at_load(lrs, tmp_path, recipe):
    cfg = _cfg(lrs, False)
    f32 = lrs.SynthModel(cfg, 6, lrs.LoadQuantization.NONE)
    path = str(tmp_path / "f32.gguf")
    lrs.write_qwen2_gguf(path, f32.desc())
    g = lrs.GgufFile(path)
    assert g.tensor("blk.0.ffn_down.weight").quant_type == lrs.QuantType.F32
    want = lrs.SynthModel(cfg, 6, lrs.LoadQuantization[recipe])
    _same_model(g.qwen2_desc(lrs.LoadQuantization[recipe]), want.desc())


def test_missing_biases_load_as_zeros_and_head_ties(lrs, tmp_path):
    sm = lrs.SynthModel(_cfg(lrs, True), 7, lrs.LoadQuantization.Q4K)
    d = sm.desc().contents
    for i in range(d.config.num_hidden_layers):
        d.layers[i].q_bias = None
    path = str(tmp_path / "nobias.gguf")
    lrs.write_qwen2_gguf(path, sm.desc())
    out = lrs.GgufFile(path).qwen2_desc(lrs.LoadQuantization.NONE).contents
    assert not out.layers[0].q_bias and out.layers[0].k_bias
    assert out.lm_head.data == out.embed_tokens.data


def _expect(lrs, tmp_path, data, match):
    path = tmp_path / "bad.gguf"
    path.write_bytes(data)
    with pytest.raises(lrs.LrsError, match=match):
        g = lrs.GgufFile(str(path))
        g.qwen2_desc(lrs.LoadQuantization.NONE)


def test_malformed_files_fail_like_the_reference(lrs, tmp_path):
    good = _minimal_v3()
    _expect(lrs, tmp_path, b"GGUX" + good[4:], "is not a GGUF file")
    _expect(lrs, tmp_path, good[:4] + struct.pack("<I", 1) + good[8:], "unsupported GGUF version 1")
    _expect(lrs, tmp_path, good[:30], "truncated GGUF file")
    _expect(lrs, tmp_path, good[:-4], "is outside the GGUF file")
    # F32 tensor claimed as Q4_K: 4 elements are not a multiple of 256
    i = good.index(b"x") + 1 + 4 + 16
    bad = good[:i] + struct.pack("<I", 12) + good[i + 4:]
    _expect(lrs, tmp_path, bad, "tensor x element count is incompatible with Q4_K")
    bad = good[:i] + struct.pack("<I", 99) + good[i + 4:]
    _expect(lrs, tmp_path, bad, "unsupported GGML tensor type 99")
    # a valid file without the qwen2 metadata
    _expect(lrs, tmp_path, good, "missing or non-string GGUF metadata general.architecture")


def test_unsupported_architecture(lrs, tmp_path):
    path = str(tmp_path / "llama.gguf")
    lrs.write_gguf(path, [("general.architecture", lrs.GGUF_STR, "llama")], [])
    with pytest.raises(lrs.LrsError, match='unsupported GGUF architecture "llama"'):
        lrs.GgufFile(path).qwen2_desc(lrs.LoadQuantization.NONE)

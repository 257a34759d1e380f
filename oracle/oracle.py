"""TEST INFRASTRUCTURE ONLY -- ctypes binding of oracle/liboracle.so.

The oracle is a CPU restatement of llama.rs's scalar token loop (see
oracle.h for what it follows and how far its parity is pinned).  Only tests/,
__graft_entry__.smoke() and bench.py's CPU-baseline leg use it, as the checker
or the timed CPU baseline; the CUDA product never calls it.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "liboracle.so")

SCALAR = 0
AVX2 = 1


def build() -> str:
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB


def _load():
    if not os.path.exists(LIB):
        build()
    lib = C.CDLL(LIB)
    P, F, U32 = C.c_void_p, C.POINTER(C.c_float), C.POINTER(C.c_uint32)

    def sig(name, res, *args):
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = list(args)

    sig("orc_type_geometry", C.c_int, C.c_uint32, U32, U32)
    sig("orc_value_at", C.c_float, P, C.c_uint32, C.c_size_t)
    sig("orc_dequantize_row", None, P, C.c_uint32, C.c_size_t, F)
    sig("orc_dot_row", C.c_float, C.c_int, P, C.c_uint32, F, C.c_size_t)
    sig("orc_matvec", C.c_int, C.c_int, C.c_int, P, C.c_uint32, C.c_size_t, C.c_size_t, F, F)
    sig("orc_avx2_available", C.c_int)
    sig("orc_model_create", P, P, C.c_size_t, C.c_int, C.c_int)
    sig("orc_model_destroy", None, P)
    sig("orc_model_forward_token", C.c_int, P, C.c_uint32, C.c_size_t, C.c_int, F)
    sig("orc_model_prefill", C.c_int, P, U32, C.c_size_t, C.c_size_t, F)
    sig("orc_benchmark_tokens", C.c_int, P, U32, C.c_size_t, C.c_size_t, U32, F, F,
        C.POINTER(C.c_double), C.POINTER(C.c_double))
    sig("orc_argmax", C.c_uint32, F, C.c_size_t)
    sig("orc_sample", C.c_uint32, F, C.c_size_t, U32, C.c_size_t, C.c_float, C.c_float,
        C.c_size_t, C.c_float, C.c_float, F)
    sig("orc_last_error", C.c_char_p)
    return lib


_lib = _load()


def _f(a):
    return a.ctypes.data_as(C.POINTER(C.c_float))


def _u(a):
    return a.ctypes.data_as(C.POINTER(C.c_uint32))


def _bytes_ptr(data: np.ndarray):
    return data.ctypes.data_as(C.c_void_p)


def dequantize_row(row: np.ndarray, ggml_type: int, cols: int) -> np.ndarray:
    out = np.empty(cols, dtype=np.float32)
    _lib.orc_dequantize_row(_bytes_ptr(row), ggml_type, cols, _f(out))
    return out


def dequantize(data: np.ndarray, ggml_type: int, rows: int, cols: int, row0: int = 0,
               nrows: int | None = None) -> np.ndarray:
    nrows = rows - row0 if nrows is None else nrows
    bv, bb = geometry(ggml_type)
    rb = cols // bv * bb
    out = np.empty((nrows, cols), dtype=np.float32)
    for i in range(nrows):
        r = row0 + i
        out[i] = dequantize_row(data[r * rb:(r + 1) * rb], ggml_type, cols)
    return out


def geometry(ggml_type: int):
    a, b = C.c_uint32(), C.c_uint32()
    if _lib.orc_type_geometry(ggml_type, C.byref(a), C.byref(b)):
        raise ValueError(f"unsupported type {ggml_type}")
    return a.value, b.value


def dot_row(kind: int, row: np.ndarray, ggml_type: int, x: np.ndarray) -> float:
    x = np.ascontiguousarray(x, dtype=np.float32)
    return float(_lib.orc_dot_row(kind, _bytes_ptr(row), ggml_type, _f(x), x.size))


def matvec(kind: int, data: np.ndarray, ggml_type: int, rows: int, cols: int, x: np.ndarray,
           threads: int = 0) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty(rows, dtype=np.float32)
    rc = _lib.orc_matvec(kind, threads, _bytes_ptr(data), ggml_type, rows, cols, _f(x), _f(y))
    if rc:
        raise ValueError("orc_matvec failed")
    return y


def avx2_available() -> bool:
    return bool(_lib.orc_avx2_available())


def sample(logits: np.ndarray, recent, temperature: float, top_p: float, top_k: int,
           repetition_penalty: float, u: float):
    """sample_current_logits (src/engine.rs:253-325) with the draw u in [0, 1):
    (token, distance of its decisions from their boundaries)."""
    l = np.ascontiguousarray(logits, dtype=np.float32)
    r = np.ascontiguousarray(np.asarray(recent, dtype=np.uint32))
    m = np.zeros(1, np.float32)
    tok = _lib.orc_sample(_f(l), l.size, _u(r), r.size, temperature, top_p, top_k,
                          repetition_penalty, u, _f(m))
    return int(tok), float(m[0])


def argmax(logits: np.ndarray) -> int:
    l = np.ascontiguousarray(logits, dtype=np.float32)
    return int(_lib.orc_argmax(_f(l), l.size))


class OracleModel:
    """Qwen2Model on the CPU restatement; desc is a pointer to an lrs_model_desc."""

    def __init__(self, desc, max_seq_len: int, kind: int = SCALAR, threads: int = 0):
        addr = C.cast(desc, C.c_void_p).value
        self._h = _lib.orc_model_create(addr, max_seq_len, kind, threads)
        if not self._h:
            raise ValueError(_lib.orc_last_error().decode())
        self.vocab = C.cast(desc, C.POINTER(C.c_uint32))[5]  # lrs_config.vocab_size

    def close(self):
        if self._h:
            _lib.orc_model_destroy(self._h)
            self._h = None

    def __del__(self):
        self.close()

    def forward_token(self, token: int, pos: int, compute: bool = True):
        out = np.empty(self.vocab, dtype=np.float32) if compute else None
        rc = _lib.orc_model_forward_token(self._h, token, pos, 1 if compute else 0,
                                          _f(out) if compute else None)
        if rc:
            raise ValueError(_lib.orc_last_error().decode())
        return out

    def prefill(self, tokens, start_pos: int = 0):
        t = np.ascontiguousarray(tokens, dtype=np.uint32)
        out = np.empty(self.vocab, dtype=np.float32)
        rc = _lib.orc_model_prefill(self._h, _u(t), t.size, start_pos, _f(out))
        if rc:
            raise ValueError(_lib.orc_last_error().decode())
        return out

    def benchmark_tokens(self, prompt, decode: int, keep_logits: bool = False):
        """Returns dict(tokens, margins, logits (optional), prefill_s, decode_s)."""
        t = np.ascontiguousarray(prompt, dtype=np.uint32)
        toks = np.zeros(decode, dtype=np.uint32)
        margins = np.zeros(decode + 1, dtype=np.float32)
        logits = np.empty((decode + 1, self.vocab), dtype=np.float32) if keep_logits else None
        ps, ds = C.c_double(), C.c_double()
        rc = _lib.orc_benchmark_tokens(self._h, _u(t), t.size, decode, _u(toks),
                                       _f(logits) if keep_logits else None, _f(margins),
                                       C.byref(ps), C.byref(ds))
        if rc:
            raise ValueError(_lib.orc_last_error().decode())
        return dict(tokens=toks, margins=margins, logits=logits, prefill_s=ps.value,
                    decode_s=ds.value)


# ----------------------------------------------------------------------------
# Model files written by the package's save_model_file (bench.py's model
# cache), read without the CUDA library: the reference arm of bench.py maps
# the model with this and drives the oracle alone.  The structs mirror
# lrs_model_desc of include/llamars.h.
class _Config(C.Structure):
    _fields_ = [("hidden_size", C.c_uint32), ("intermediate_size", C.c_uint32),
                ("num_attention_heads", C.c_uint32), ("num_key_value_heads", C.c_uint32),
                ("num_hidden_layers", C.c_uint32), ("vocab_size", C.c_uint32),
                ("head_dim", C.c_uint32), ("max_position_embeddings", C.c_uint32),
                ("rms_norm_eps", C.c_float), ("rope_theta", C.c_float)]


class _TensorDesc(C.Structure):
    _fields_ = [("data", C.c_void_p), ("nbytes", C.c_uint64), ("rows", C.c_uint64),
                ("cols", C.c_uint64), ("ggml_type", C.c_uint32), ("reserved", C.c_uint32)]


class _LayerDesc(C.Structure):
    _fields_ = [("input_layernorm", C.c_void_p), ("post_attention_layernorm", C.c_void_p),
                ("q_proj", _TensorDesc), ("k_proj", _TensorDesc), ("v_proj", _TensorDesc),
                ("o_proj", _TensorDesc), ("gate_proj", _TensorDesc), ("up_proj", _TensorDesc),
                ("down_proj", _TensorDesc), ("q_bias", C.c_void_p), ("k_bias", C.c_void_p),
                ("v_bias", C.c_void_p)]


class _ModelDesc(C.Structure):
    _fields_ = [("config", _Config), ("embed_tokens", _TensorDesc), ("lm_head", _TensorDesc),
                ("final_norm", C.c_void_p), ("layers", C.POINTER(_LayerDesc))]


class MappedModel:
    """A model file (magic LRSMODL1, JSON index, 64-byte aligned blobs) mapped
    read-only; desc() points at an lrs_model_desc valid while this lives."""

    _LAYER_T = ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj")
    _LAYER_V = ("input_layernorm", "post_attention_layernorm", "q_bias", "k_bias", "v_bias")

    def __init__(self, path: str):
        import json
        with open(path, "rb") as f:
            head = f.read(16)
            if head[:8] != b"LRSMODL1":
                raise ValueError(f"{path}: not a model file")
            n = int.from_bytes(head[8:16], "little")
            meta = json.loads(f.read(n))
        self._map = np.memmap(path, dtype=np.uint8, mode="r")
        base = self._map.ctypes.data + (16 + n + 63) // 64 * 64
        blobs = meta["blobs"]

        def ptr(i):
            return None if i is None else base + blobs[i][0]

        def tens(t):
            return _TensorDesc(ptr(t["blob"]), blobs[t["blob"]][1], t["rows"], t["cols"], t["type"], 0)

        c = meta["config"]
        self._layers = (_LayerDesc * c["num_hidden_layers"])()
        for i, ent in enumerate(meta["layers"]):
            L = self._layers[i]
            for k in self._LAYER_T:
                setattr(L, k, tens(ent[k]))
            for k in self._LAYER_V:
                setattr(L, k, ptr(ent[k]))
        self._desc = _ModelDesc()
        self._desc.config = _Config(*[c[k] for k, _ in _Config._fields_])
        self._desc.embed_tokens = tens(meta["embed_tokens"])
        self._desc.lm_head = tens(meta["lm_head"])
        self._desc.final_norm = ptr(meta["final_norm"])
        self._desc.layers = C.cast(self._layers, C.POINTER(_LayerDesc))
        self.vocab_size = c["vocab_size"]

    def desc(self):
        return C.pointer(self._desc)

"""B200 (sm_100a) CUDA backend for llama.rs's Qwen2 token loop -- Python host module.

This module binds ``libllamars.so`` (the C ABI declared in ``include/llamars.h``
and ``include/llamars_synth.h``) with ctypes and mirrors the reference
engine's interfaces for the hot path:

* ``QuantType`` / ``QuantTensor``      -- src/quant.rs:10-324
* ``CudaBackend`` (``KernelBackend``)  -- src/backend.rs:67-73 (name, threads, matvec)
* ``CudaQwen2Model`` (``CausalModel``) -- src/architecture.rs:42-78 (forward_token, prefill)
  plus the greedy loop of ``InferenceEngine::benchmark_tokens`` (src/engine.rs:189-241)
* ``synth_model``                      -- the load path (src/loader.rs:83-227 + maybe_quantize
  :406-447) for seeded synthetic checkpoints.

Errors surface as ``LrsError`` carrying the library's message, the way the
reference surfaces ``anyhow`` errors.  There is no CPU fallback: if the CUDA
library is missing, importing this module raises.
"""
from __future__ import annotations

import ctypes as C
import enum
import os
import weakref
from dataclasses import dataclass, field
from typing import Optional, Sequence

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libllamars.so")

if not os.path.exists(LIB_PATH):
    raise ImportError(
        f"{LIB_PATH} is missing: build the CUDA backend first (make -C llama.rs_b200, "
        "or __graft_entry__.build())")
_lib = C.CDLL(LIB_PATH)


class LrsError(RuntimeError):
    """A failed call into the CUDA backend (the reference's anyhow::Error)."""

    def __init__(self, code: int, message: str):
        super().__init__(f"[{code}] {message}")
        self.code = code


# ------------------------------------------------------------------ types --
class QuantType(enum.IntEnum):
    """QuantType with its GGML ids (src/quant.rs:10-44)."""

    F32 = 0
    F16 = 1
    Q4_0 = 2
    Q4_1 = 3
    Q5_0 = 6
    Q5_1 = 7
    Q8_0 = 8
    Q4_K = 12
    Q5_K = 13
    Q6_K = 14
    BF16 = 30

    @classmethod
    def from_ggml_type(cls, value: int) -> "QuantType":
        try:
            return cls(value)
        except ValueError:
            raise LrsError(2, f"unsupported GGML tensor type {value}; supported: F32, F16, BF16, "
                              "Q4_0, Q4_1, Q5_0, Q5_1, Q8_0, Q4_K, Q5_K, Q6_K") from None

    def block_size(self) -> int:
        return _GEOM[self][0]

    def type_size(self) -> int:
        return _GEOM[self][1]

    def display_name(self) -> str:
        return "Q4_K" if self is QuantType.Q4_K else (
            "Q5_K" if self is QuantType.Q5_K else ("Q6_K" if self is QuantType.Q6_K else self.name))


_GEOM = {
    QuantType.F32: (1, 4), QuantType.F16: (1, 2), QuantType.BF16: (1, 2),
    QuantType.Q4_0: (32, 18), QuantType.Q4_1: (32, 20), QuantType.Q5_0: (32, 22),
    QuantType.Q5_1: (32, 24), QuantType.Q8_0: (32, 34), QuantType.Q4_K: (256, 144),
    QuantType.Q5_K: (256, 176), QuantType.Q6_K: (256, 210),
}


class LoadQuantization(enum.IntEnum):
    """LoadQuantization (src/loader.rs:16-25)."""

    NONE = 0
    Q4K = 1
    Q4KM = 2


class LogitsMode(enum.IntEnum):
    """LogitsMode (src/architecture.rs:34-38)."""

    SKIP = 0
    COMPUTE = 1


# ------------------------------------------------------------ C structs --
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


class _ModelOptions(C.Structure):
    _fields_ = [("max_seq_len", C.c_uint32), ("max_sequences", C.c_uint32),
                ("kv_dtype", C.c_uint32), ("use_graph", C.c_uint32),
                ("device_recipe", C.c_uint32), ("tp_allreduce", C.c_uint32),
                ("persistent_decode", C.c_uint32)]


class _SynthSpec(C.Structure):
    _fields_ = [("config", _Config), ("seed", C.c_uint64), ("recipe", C.c_uint32),
                ("tie_word_embeddings", C.c_uint32), ("init_std", C.c_float),
                ("threads", C.c_uint32)]


class Sampler(C.Structure):
    """EngineOptions' sampling fields (src/engine.rs:11-33), with the reference's
    defaults: temperature 0.7, top_p 0.9, top_k 40, repetition_penalty 1.1."""
    _fields_ = [("temperature", C.c_float), ("top_p", C.c_float), ("top_k", C.c_uint32),
                ("repetition_penalty", C.c_float)]

    def __init__(self, temperature: float = 0.7, top_p: float = 0.9, top_k: int = 40,
                 repetition_penalty: float = 1.1):
        super().__init__(temperature, top_p, top_k, repetition_penalty)


#: LRS_SAMPLE_MAX_TOP_K: the largest top_k the device sampler takes
SAMPLE_MAX_TOP_K = 4096

_P = C.c_void_p
_F = C.POINTER(C.c_float)
_U32 = C.POINTER(C.c_uint32)


def _sig(name, res, *args):
    fn = getattr(_lib, name)
    fn.restype = res
    fn.argtypes = list(args)
    return fn


_lib_last_error = _sig("lrs_last_error", C.c_char_p)
_sig("lrs_type_geometry", C.c_int32, C.c_uint32, _U32, _U32)
_sig("lrs_backend_create", C.c_int32, C.c_int, C.POINTER(_P))
_sig("lrs_backend_destroy", None, _P)
_sig("lrs_backend_name", C.c_char_p, _P)
_sig("lrs_backend_threads", C.c_size_t, _P)
_sig("lrs_backend_synchronize", C.c_int32, _P)
_sig("lrs_backend_stream", _P, _P)
_sig("lrs_tensor_upload", C.c_int32, _P, _P, C.c_size_t, C.c_size_t, C.c_size_t, C.c_uint32,
     C.POINTER(_P))
_sig("lrs_tensor_free", None, _P)
_sig("lrs_tensor_device_ptr", _P, _P)
_sig("lrs_dequantize_rows", C.c_int32, _P, _P, C.c_size_t, C.c_size_t, _F)
_sig("lrs_matvec", C.c_int32, _P, _P, _F, C.c_size_t, _F, C.c_size_t)
_sig("lrs_matvec_batched", C.c_int32, _P, _P, _F, C.c_size_t, C.c_size_t, _F, C.c_size_t)
_sig("lrs_matvec_noalloc", C.c_int32, _P, _P, _F, C.c_size_t, _F, C.c_size_t)
_sig("lrs_matvec_device", C.c_int32, _P, _P, C.c_void_p, C.c_size_t, C.c_void_p, C.c_void_p)
_sig("lrs_quantize_matrix_device", C.c_int32, _P, C.c_uint32, C.c_void_p, C.c_size_t, C.c_size_t,
     C.c_void_p, C.c_size_t, _U32, C.POINTER(C.c_size_t))
_sig("lrs_gguf_open", C.c_int32, C.c_char_p, C.POINTER(_P))
_sig("lrs_gguf_close", None, _P)
_sig("lrs_gguf_version", C.c_uint32, _P)
_sig("lrs_gguf_tensor_count", C.c_size_t, _P)
_sig("lrs_gguf_metadata_u64", C.c_int32, _P, C.c_char_p, C.POINTER(C.c_uint64))
_sig("lrs_gguf_metadata_f32", C.c_int32, _P, C.c_char_p, C.POINTER(C.c_float))
_sig("lrs_gguf_metadata_str", C.c_int32, _P, C.c_char_p, C.POINTER(C.c_char_p))
_sig("lrs_gguf_tensor", C.c_int32, _P, C.c_char_p, C.POINTER(_TensorDesc))
_sig("lrs_gguf_qwen2_desc", C.c_int32, _P, C.c_uint32, C.POINTER(C.POINTER(_ModelDesc)))
_sig("lrs_tp_unique_id", C.c_int32, C.c_char_p)
_sig("lrs_model_create_tp", C.c_int32, _P, C.POINTER(_ModelDesc), C.POINTER(_ModelOptions),
     C.c_uint32, C.c_uint32, C.c_char_p, C.POINTER(_P))
_sig("lrs_model_tp_world", C.c_uint32, _P)
_sig("lrs_model_create", C.c_int32, _P, C.POINTER(_ModelDesc), C.POINTER(_ModelOptions),
     C.POINTER(_P))
_sig("lrs_model_destroy", None, _P)
_sig("lrs_model_reset", C.c_int32, _P, C.c_uint32)
_sig("lrs_model_forward_token", C.c_int32, _P, C.c_uint32, C.c_uint32, C.c_uint32, C.c_int, _F,
     _U32)
_sig("lrs_model_prefill", C.c_int32, _P, C.c_uint32, _U32, C.c_size_t, C.c_uint32, _F, _U32)
_sig("lrs_model_decode_greedy", C.c_int32, _P, C.c_size_t, _U32, _U32, _U32, C.c_size_t, _U32)
_sig("lrs_model_decode_enqueue", C.c_int32, _P, C.c_size_t, _U32, _U32, _U32, C.c_size_t)
_sig("lrs_model_read_tokens", C.c_int32, _P, C.c_size_t, C.c_size_t, _U32)
_sig("lrs_model_weight_bytes", C.c_uint64, _P)
_sig("lrs_model_weights_digest", C.c_int32, _P, C.POINTER(C.c_uint64))
_sig("lrs_model_profile_step", C.c_int32, _P, C.c_size_t, _U32, _U32, _U32, _F, _U32, _F, _F)
_sig("lrs_model_step_kernels", C.c_uint32, _P)
_sig("lrs_recipe_type", C.c_uint32, C.c_uint32, C.c_char_p, C.c_size_t, C.c_size_t)
_sig("lrs_quantize_matrix", C.c_int32, C.c_uint32, _F, C.c_size_t, C.c_size_t, _P, C.c_size_t,
     _U32, C.POINTER(C.c_size_t))
_sig("lrs_quantized_size", C.c_size_t, C.c_uint32, C.c_size_t, C.c_size_t)
_sig("lrs_synth_fill", None, C.c_uint64, C.c_char_p, C.c_float, C.c_uint64, C.c_size_t, _F)
_sig("lrs_synth_model_create", C.c_int32, C.POINTER(_SynthSpec), C.POINTER(_P))
_sig("lrs_synth_model_desc", C.POINTER(_ModelDesc), _P)
_sig("lrs_synth_model_destroy", None, _P)
_sig("lrs_st_open", C.c_int32, C.c_char_p, C.POINTER(_P))
_sig("lrs_st_close", None, _P)
_sig("lrs_st_tensor_count", C.c_size_t, _P)
_sig("lrs_st_tensor", C.c_int32, _P, C.c_char_p, C.POINTER(_TensorDesc))
_sig("lrs_st_qwen2_desc", C.c_int32, _P, C.c_uint32, C.POINTER(C.POINTER(_ModelDesc)))
_sig("lrs_model_load", C.c_int32, C.c_char_p, C.c_uint32, C.POINTER(_P),
     C.POINTER(C.POINTER(_ModelDesc)))
_sig("lrs_loaded_close", None, _P)
_sig("lrs_sampler_check", C.c_int32, C.POINTER(Sampler), C.c_size_t)
_sig("lrs_sample_logits", C.c_int32, _P, C.c_void_p, C.c_size_t, C.POINTER(Sampler), _U32,
     C.c_size_t, C.c_float, _U32)
_sig("lrs_model_forward_sample", C.c_int32, _P, C.c_uint32, C.c_uint32, C.c_uint32,
     C.POINTER(Sampler), _U32, C.c_size_t, C.c_float, _U32)

#: every symbol include/*.h declares (checked by the CPU tests)
EXPORTED_SYMBOLS = (
    "lrs_last_error", "lrs_type_geometry", "lrs_backend_create", "lrs_backend_destroy",
    "lrs_backend_name", "lrs_backend_threads", "lrs_backend_synchronize", "lrs_backend_stream",
    "lrs_tensor_upload", "lrs_tensor_free", "lrs_tensor_device_ptr", "lrs_dequantize_rows",
    "lrs_matvec", "lrs_matvec_noalloc", "lrs_matvec_batched", "lrs_matvec_device",
    "lrs_model_create",
    "lrs_model_destroy", "lrs_model_reset", "lrs_model_forward_token", "lrs_model_prefill",
    "lrs_model_decode_greedy", "lrs_model_decode_enqueue", "lrs_model_read_tokens",
    "lrs_model_weight_bytes", "lrs_model_weights_digest", "lrs_model_profile_step", "lrs_model_step_kernels",
    "lrs_tp_unique_id", "lrs_model_create_tp", "lrs_model_tp_world",
    "lrs_quantize_matrix_device", "lrs_gguf_open", "lrs_gguf_close", "lrs_gguf_version", "lrs_gguf_tensor_count",
    "lrs_gguf_metadata_u64", "lrs_gguf_metadata_f32", "lrs_gguf_metadata_str", "lrs_gguf_tensor",
    "lrs_gguf_qwen2_desc", "lrs_recipe_type", "lrs_quantize_matrix", "lrs_quantized_size",
    "lrs_synth_fill", "lrs_synth_model_create", "lrs_synth_model_desc", "lrs_synth_model_destroy",
    "lrs_sampler_check", "lrs_sample_logits", "lrs_model_forward_sample",
    "lrs_st_open", "lrs_st_close", "lrs_st_tensor_count", "lrs_st_tensor", "lrs_st_qwen2_desc",
    "lrs_model_load", "lrs_loaded_close",
)


def _check(code: int) -> None:
    if code != 0:
        raise LrsError(code, (_lib.lrs_last_error() or b"").decode(errors="replace"))


def _fptr(a: np.ndarray):
    return a.ctypes.data_as(_F)


def _uptr(a: np.ndarray):
    return a.ctypes.data_as(_U32)


def library():
    """The loaded ctypes handle of libllamars.so."""
    return _lib


# ----------------------------------------------------------- QuantTensor --
class QuantTensor:
    """Row-major [rows, cols] GGML tensor (QuantTensor, src/quant.rs:105-324).

    ``data`` is a contiguous uint8 numpy array of exactly
    rows * cols / block_size * type_size bytes.
    """

    def __init__(self, data, shape: Sequence[int], quant_type: QuantType):
        quant_type = QuantType(quant_type)
        shape = tuple(int(s) for s in shape)
        if not (1 <= len(shape) <= 2):
            raise LrsError(1, "only 1D and 2D tensors are supported")
        cols = shape[-1]
        if cols % quant_type.block_size():
            raise LrsError(1, f"last dimension {cols} is not divisible by "
                              f"{quant_type.block_size()} for {quant_type.display_name()}")
        elems = int(np.prod(shape))
        expected = elems // quant_type.block_size() * quant_type.type_size()
        buf = np.ascontiguousarray(np.frombuffer(data, dtype=np.uint8) if isinstance(
            data, (bytes, bytearray, memoryview)) else data, dtype=np.uint8).reshape(-1)
        if buf.size != expected:
            raise LrsError(1, f"bad {quant_type.display_name()} tensor byte length: got "
                              f"{buf.size}, expected {expected}")
        self.data = buf
        self.shape = shape
        self.quant_type = quant_type

    def rows(self) -> int:
        return 1 if len(self.shape) == 1 else self.shape[0]

    def cols(self) -> int:
        return self.shape[-1]

    def row_bytes(self) -> int:
        return self.cols() // self.quant_type.block_size() * self.quant_type.type_size()

    def row_data(self, row: int) -> np.ndarray:
        rb = self.row_bytes()
        return self.data[row * rb:(row + 1) * rb]

    @classmethod
    def from_f32(cls, values: np.ndarray, shape: Sequence[int]) -> "QuantTensor":
        v = np.ascontiguousarray(values, dtype=np.float32).reshape(-1)
        return cls(v.view(np.uint8), shape, QuantType.F32)

    @classmethod
    def quantize(cls, values: np.ndarray, rows: int, cols: int, quant_type: QuantType) -> "QuantTensor":
        """Encodes F32 values as ``quant_type`` (QuantTensor::quantize_*, src/quant.rs:187-259,
        with the reference fallbacks; see lrs_quantize_matrix)."""
        v = np.ascontiguousarray(values, dtype=np.float32).reshape(-1)
        if v.size != rows * cols:
            raise LrsError(1, "quantization shape/data mismatch")
        size = _lib.lrs_quantized_size(int(quant_type), rows, cols)
        out = np.zeros(size, dtype=np.uint8)
        t = C.c_uint32()
        n = C.c_size_t()
        _check(_lib.lrs_quantize_matrix(int(quant_type), _fptr(v), rows, cols,
                                        out.ctypes.data_as(_P), size, C.byref(t), C.byref(n)))
        return cls(out, (rows, cols), QuantType(t.value))

    @classmethod
    def quantize_q4k(cls, values, rows, cols):
        return cls.quantize(values, rows, cols, QuantType.Q4_K)

    @classmethod
    def quantize_q5_0(cls, values, rows, cols):
        return cls.quantize(values, rows, cols, QuantType.Q5_0)

    @classmethod
    def quantize_q8_0(cls, values, rows, cols):
        return cls.quantize(values, rows, cols, QuantType.Q8_0)

    @classmethod
    def quantize_q6k(cls, values, rows, cols):
        return cls.quantize(values, rows, cols, QuantType.Q6_K)

    def desc(self) -> _TensorDesc:
        return _TensorDesc(self.data.ctypes.data, self.data.size, self.rows(), self.cols(),
                           int(self.quant_type), 0)


def recipe_type(recipe: LoadQuantization, name: str, rows: int, cols: int) -> QuantType:
    """Type maybe_quantize (src/loader.rs:406-447) assigns to an F32 tensor."""
    return QuantType(_lib.lrs_recipe_type(int(recipe), name.encode(), rows, cols))


def synth_values(seed: int, name: str, n: int, offset: int = 0, std: float = 0.02) -> np.ndarray:
    """The N(0, std) values of tensor ``name`` in the seeded synthetic models."""
    out = np.empty(n, dtype=np.float32)
    _lib.lrs_synth_fill(seed, name.encode(), std, offset, n, _fptr(out))
    return out


# ------------------------------------------------------------ backend ----
class CudaBackend:
    """KernelBackend over one CUDA device (src/backend.rs:67-73).

    Tensors are uploaded to HBM once, in their native block layout, and cached
    by the address of their host bytes -- the lookup a Rust ``CudaBackend``
    shim does for ``matvec(&QuantTensor, ..)``.
    """

    def __init__(self, device: int = 0):
        h = _P()
        _check(_lib.lrs_backend_create(device, C.byref(h)))
        self._h = h
        self.device = device
        self._cache = {}
        self._models = weakref.WeakSet()  # models on this backend: destroyed first

    def close(self):
        for m in list(self._models):
            m.close()
        for _, (t, _keep) in list(self._cache.items()):
            _lib.lrs_tensor_free(t)
        self._cache.clear()
        if self._h:
            _lib.lrs_backend_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def handle(self):
        return self._h

    def name(self) -> str:
        return _lib.lrs_backend_name(self._h).decode()

    def threads(self) -> int:
        return int(_lib.lrs_backend_threads(self._h))

    def stream(self) -> int:
        return _lib.lrs_backend_stream(self._h)

    def synchronize(self) -> None:
        _check(_lib.lrs_backend_synchronize(self._h))

    def upload(self, weight: QuantTensor):
        key = (weight.data.ctypes.data, weight.data.size, int(weight.quant_type))
        hit = self._cache.get(key)
        if hit is not None:
            return hit[0]
        t = _P()
        _check(_lib.lrs_tensor_upload(self._h, weight.data.ctypes.data_as(_P), weight.data.size,
                                      weight.rows(), weight.cols(), int(weight.quant_type),
                                      C.byref(t)))
        self._cache[key] = (t, weight.data)
        return t

    def release(self, weight: QuantTensor) -> None:
        key = (weight.data.ctypes.data, weight.data.size, int(weight.quant_type))
        hit = self._cache.pop(key, None)
        if hit is not None:
            _lib.lrs_tensor_free(hit[0])

    def matvec(self, weight: QuantTensor, input: np.ndarray, output: np.ndarray) -> None:
        """output[r] = dot(row r, input)  (KernelBackend::matvec)."""
        t = self.upload(weight)
        _check(_lib.lrs_matvec(self._h, t, _fptr(input), input.size, _fptr(output), output.size))

    def matvec_batched(self, weight: QuantTensor, inputs: np.ndarray) -> np.ndarray:
        """[B, cols] -> [B, rows]; equals B independent matvec calls."""
        x = np.ascontiguousarray(inputs, dtype=np.float32)
        b = x.shape[0]
        out = np.empty((b, weight.rows()), dtype=np.float32)
        t = self.upload(weight)
        _check(_lib.lrs_matvec_batched(self._h, t, _fptr(x), b, x.shape[1], _fptr(out),
                                       weight.rows()))
        return out

    def matvec_device(self, weight: QuantTensor, d_in: int, batch: int, d_out: int,
                      stream: Optional[int] = None) -> None:
        """Queues a batched matvec on device pointers (no synchronization)."""
        t = self.upload(weight)
        _check(_lib.lrs_matvec_device(self._h, t, d_in, batch, d_out, stream))

    def sample_logits(self, d_logits: int, vocab: int, params: Sampler, recent, u: float) -> int:
        """sample_current_logits (src/engine.rs:253-325) on device logits
        (lrs_sample_logits); u in [0, 1) is the reference's thread_rng draw."""
        r = np.ascontiguousarray(np.asarray(recent, dtype=np.uint32))
        out = np.zeros(1, dtype=np.uint32)
        _check(_lib.lrs_sample_logits(self._h, d_logits, vocab, C.byref(params), _uptr(r), r.size,
                                      u, _uptr(out)))
        return int(out[0])

    def quantize_device(self, d_values: int, rows: int, cols: int, quant_type: "QuantType",
                        d_out: int, out_cap: int):
        """The load-time encoders on the GPU (lrs_quantize_matrix_device): device
        pointers in and out; returns (type produced, bytes written)."""
        t = np.zeros(1, np.uint32)
        n = C.c_size_t()
        _check(_lib.lrs_quantize_matrix_device(self._h, int(quant_type), d_values, rows, cols, d_out,
                                               out_cap, _uptr(t), C.byref(n)))
        return QuantType(int(t[0])), n.value

    def dequantize_rows(self, weight: QuantTensor, row0: int, nrows: int) -> np.ndarray:
        """value_at for rows [row0, row0 + nrows) (QuantTensor::row_into)."""
        out = np.empty((nrows, weight.cols()), dtype=np.float32)
        t = self.upload(weight)
        _check(_lib.lrs_dequantize_rows(self._h, t, row0, nrows, _fptr(out)))
        return out


# --------------------------------------------------------------- model ---
@dataclass
class LlamaConfig:
    """LlamaConfig (src/config.rs:18-39) with head_dim resolved."""

    hidden_size: int
    intermediate_size: int
    num_attention_heads: int
    num_key_value_heads: int
    num_hidden_layers: int
    vocab_size: int
    rms_norm_eps: float = 1e-6
    rope_theta: float = 10000.0
    max_position_embeddings: int = 32768
    head_dim: Optional[int] = None
    tie_word_embeddings: bool = False

    def resolved_head_dim(self) -> int:
        return self.head_dim or self.hidden_size // self.num_attention_heads

    def kv_width(self) -> int:
        return self.num_key_value_heads * self.resolved_head_dim()

    def to_c(self) -> _Config:
        return _Config(self.hidden_size, self.intermediate_size, self.num_attention_heads,
                       self.num_key_value_heads, self.num_hidden_layers, self.vocab_size,
                       self.resolved_head_dim(), self.max_position_embeddings,
                       self.rms_norm_eps, self.rope_theta)


class SynthModel:
    """A seeded synthetic Qwen2 checkpoint, quantized at load time like the reference."""

    def __init__(self, config: LlamaConfig, seed: int, recipe: LoadQuantization,
                 init_std: float = 0.02, threads: int = 0):
        spec = _SynthSpec(config.to_c(), seed, int(recipe), 1 if config.tie_word_embeddings else 0,
                          init_std, threads)
        h = _P()
        _check(_lib.lrs_synth_model_create(C.byref(spec), C.byref(h)))
        self._h = h
        self.config = config
        self.seed = seed
        self.recipe = recipe

    def close(self):
        if self._h:
            _lib.lrs_synth_model_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def desc(self):
        """Pointer to the lrs_model_desc (host views stay valid while this object
        lives; the pointer keeps it alive)."""
        p = _lib.lrs_synth_model_desc(self._h)
        p._owner = self
        return p

    def tensor(self, which: str, layer: Optional[int] = None) -> QuantTensor:
        """A weight as a QuantTensor view: 'embed', 'lm_head' or a layer projection name."""
        d = self.desc().contents
        if layer is None:
            td = getattr(d, "embed_tokens" if which == "embed" else which)
        else:
            td = getattr(d.layers[layer], which)
        buf = (C.c_uint8 * td.nbytes).from_address(td.data)
        return QuantTensor(np.frombuffer(buf, dtype=np.uint8), (td.rows, td.cols),
                           QuantType(td.ggml_type))


_MF_MAGIC = b"LRSMODL1"
_MF_LAYER_TENSORS = ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj")
_MF_LAYER_VECS = ("input_layernorm", "post_attention_layernorm", "q_bias", "k_bias", "v_bias")


def save_model_file(desc, path: str) -> None:
    """Writes the host model behind an lrs_model_desc as one flat file: the
    pre-quantized tensors (GGML block bytes, as the load-time quantizers of
    src/loader.rs:406-447 left them), norms and biases, plus a JSON index.
    A tied head (same bytes as the embedding) is stored once.  The file is
    written under a temporary name and renamed, so readers never see a partial
    file."""
    import json
    d = desc.contents
    c = d.config
    h, kvw = c.hidden_size, c.num_key_value_heads * c.head_dim
    blobs, index = [], {}

    def add(ptr, nbytes):
        if not ptr:
            return None
        key = (int(ptr), int(nbytes))
        if key not in index:
            index[key] = len(blobs)
            blobs.append(key)
        return index[key]

    def tens(td):
        return {"blob": add(td.data, td.nbytes), "rows": int(td.rows), "cols": int(td.cols),
                "type": int(td.ggml_type)}

    cfg = {k: getattr(c, k) for k, _ in _Config._fields_}
    meta = {"config": cfg, "embed_tokens": tens(d.embed_tokens), "lm_head": tens(d.lm_head),
            "final_norm": add(d.final_norm, 4 * h), "layers": []}
    vec_len = {"input_layernorm": h, "post_attention_layernorm": h, "q_bias": h,
               "k_bias": kvw, "v_bias": kvw}
    for i in range(c.num_hidden_layers):
        L = d.layers[i]
        ent = {n: tens(getattr(L, n)) for n in _MF_LAYER_TENSORS}
        for n in _MF_LAYER_VECS:
            ent[n] = add(getattr(L, n), 4 * vec_len[n])
        meta["layers"].append(ent)
    off = 0
    table = []
    for ptr, nbytes in blobs:
        table.append([off, nbytes])
        off += (nbytes + 63) // 64 * 64
    meta["blobs"] = table
    hdr = json.dumps(meta).encode()
    data_start = (16 + len(hdr) + 63) // 64 * 64
    tmp = f"{path}.tmp{os.getpid()}"
    with open(tmp, "wb") as f:
        f.write(_MF_MAGIC + len(hdr).to_bytes(8, "little") + hdr)
        f.write(b"\0" * (data_start - 16 - len(hdr)))
        for (ptr, nbytes), (o, _) in zip(blobs, table):
            f.seek(data_start + o)
            f.write((C.c_uint8 * nbytes).from_address(ptr))
        f.truncate(data_start + off)
    os.replace(tmp, path)


class ModelFile:
    """A model written by save_model_file, memory-mapped; ``desc()`` has the
    same shape as SynthModel.desc() and stays valid while this object lives."""

    def __init__(self, path: str):
        import json
        with open(path, "rb") as f:
            head = f.read(16)
            if head[:8] != _MF_MAGIC:
                raise LrsError(1, f"{path}: not a model file")
            n = int.from_bytes(head[8:16], "little")
            meta = json.loads(f.read(n))
        data_start = (16 + n + 63) // 64 * 64
        self._map = np.memmap(path, dtype=np.uint8, mode="r")
        base = self._map.ctypes.data + data_start
        blobs = meta["blobs"]

        def ptr(i):
            return None if i is None else base + blobs[i][0]

        def tens(t):
            return _TensorDesc(ptr(t["blob"]), blobs[t["blob"]][1], t["rows"], t["cols"], t["type"], 0)

        cfgd = meta["config"]
        self.config = LlamaConfig(cfgd["hidden_size"], cfgd["intermediate_size"],
                                  cfgd["num_attention_heads"], cfgd["num_key_value_heads"],
                                  cfgd["num_hidden_layers"], cfgd["vocab_size"],
                                  cfgd["rms_norm_eps"], cfgd["rope_theta"],
                                  cfgd["max_position_embeddings"], cfgd["head_dim"],
                                  meta["embed_tokens"]["blob"] == meta["lm_head"]["blob"])
        nl = cfgd["num_hidden_layers"]
        self._layers = (_LayerDesc * nl)()
        for i, ent in enumerate(meta["layers"]):
            L = self._layers[i]
            for n in _MF_LAYER_TENSORS:
                setattr(L, n, tens(ent[n]))
            for n in _MF_LAYER_VECS:
                setattr(L, n, ptr(ent[n]))
        self._desc = _ModelDesc()
        self._desc.config = _Config(*[cfgd[k] for k, _ in _Config._fields_])
        self._desc.embed_tokens = tens(meta["embed_tokens"])
        self._desc.lm_head = tens(meta["lm_head"])
        self._desc.final_norm = ptr(meta["final_norm"])
        self._desc.layers = C.cast(self._layers, C.POINTER(_LayerDesc))

    def desc(self):
        p = C.pointer(self._desc)
        p._owner = self  # the views stay valid while the pointer lives
        return p


class CudaQwen2Model:
    """CausalModel on the CUDA backend (src/architecture.rs:42-78).

    Owns the device weights, a paged KV cache with ``max_sequences`` slots and
    the activation buffers.  ``forward_token`` / ``prefill`` follow the trait;
    ``decode_greedy`` is the decode half of benchmark_tokens with the argmax on
    the device and each step replayed as one CUDA graph.
    """

    def __init__(self, backend: CudaBackend, desc, max_seq_len: int = 4096,
                 max_sequences: int = 1, kv_bf16: bool = False, use_graph: bool = True,
                 keepalive=None, tp_rank: int = 0, tp_world: int = 1, tp_id: bytes = b"",
                 device_recipe: LoadQuantization = LoadQuantization.NONE,
                 tp_p2p: bool = False, persistent_decode: bool = False):
        """tp_world > 1 makes this process shard tp_rank of a tensor-parallel
        model (every rank passes the full desc and the same tp_id, made once by
        tp_unique_id() and shared out of band).  device_recipe encodes the
        desc's F32/F16/BF16 matrices on the GPU (the load-time recipe)."""
        opts = _ModelOptions(max_seq_len, max_sequences, 1 if kv_bf16 else 0,
                             1 if use_graph else 0, int(device_recipe), 1 if tp_p2p else 0,
                             1 if persistent_decode else 0)
        h = _P()
        if tp_world > 1:
            if len(tp_id) != 128:
                raise LrsError(1, "tp_id must be the 128 bytes of tp_unique_id()")
            _check(_lib.lrs_model_create_tp(backend.handle, desc, C.byref(opts), tp_rank,
                                            tp_world, tp_id, C.byref(h)))
        else:
            _check(_lib.lrs_model_create(backend.handle, desc, C.byref(opts), C.byref(h)))
        self._h = h
        self.backend = backend
        backend._models.add(self)
        self.keepalive = keepalive
        cfg = desc.contents.config
        self.vocab_size = cfg.vocab_size
        self.max_seq_len = max_seq_len
        self.max_sequences = max_sequences

    def close(self):
        # a model must go before its backend; the backend's close() closes it first
        if self._h and self.backend._h:
            _lib.lrs_model_destroy(self._h)
        self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def weight_bytes(self) -> int:
        return int(_lib.lrs_model_weight_bytes(self._h))

    def weights_digest(self) -> int:
        """FNV-1a digest of the weight bytes on the device (lrs_model_weights_digest)."""
        d = C.c_uint64()
        _check(_lib.lrs_model_weights_digest(self._h, C.byref(d)))
        return int(d.value)

    def reset(self, seq: int = 0) -> None:
        _check(_lib.lrs_model_reset(self._h, seq))

    def forward_token(self, token_id: int, pos: int, logits: LogitsMode = LogitsMode.COMPUTE,
                      seq: int = 0):
        """Returns (logits, argmax) for LogitsMode.COMPUTE, else None."""
        if logits == LogitsMode.COMPUTE:
            out = np.empty(self.vocab_size, dtype=np.float32)
            am = np.zeros(1, dtype=np.uint32)
            _check(_lib.lrs_model_forward_token(self._h, seq, token_id, pos, 1, _fptr(out),
                                                _uptr(am)))
            return out, int(am[0])
        _check(_lib.lrs_model_forward_token(self._h, seq, token_id, pos, 0, None, None))
        return None

    def forward_sample(self, token_id: int, pos: int, params: Sampler, recent, u: float,
                       seq: int = 0) -> int:
        """InferenceEngine::forward_step (src/engine.rs:96-106) with the sampler on
        the device: the next token for draw u in [0, 1)."""
        r = np.ascontiguousarray(np.asarray(recent, dtype=np.uint32))
        out = np.zeros(1, dtype=np.uint32)
        _check(_lib.lrs_model_forward_sample(self._h, seq, token_id, pos, C.byref(params),
                                             _uptr(r), r.size, u, _uptr(out)))
        return int(out[0])

    def prefill(self, tokens: Sequence[int], start_pos: int = 0, seq: int = 0,
                want_logits: bool = True):
        """Prompt pass; returns (last logits, argmax) like the reference's prefill."""
        t = np.ascontiguousarray(tokens, dtype=np.uint32)
        out = np.empty(self.vocab_size, dtype=np.float32) if want_logits else None
        am = np.zeros(1, dtype=np.uint32)
        _check(_lib.lrs_model_prefill(self._h, seq, _uptr(t), t.size, start_pos,
                                      _fptr(out) if out is not None else None, _uptr(am)))
        return out, int(am[0])

    def decode_greedy(self, first_tokens: Sequence[int], start_pos: Sequence[int], n_steps: int,
                      seqs: Optional[Sequence[int]] = None) -> np.ndarray:
        """[n_steps, n_seqs]: row s = token produced by greedy step s (fed to step s + 1)."""
        ft = np.ascontiguousarray(first_tokens, dtype=np.uint32)
        n = ft.size
        sp = np.ascontiguousarray(start_pos, dtype=np.uint32)
        sq = np.ascontiguousarray(seqs if seqs is not None else range(n), dtype=np.uint32)
        out = np.zeros((n_steps, n), dtype=np.uint32)
        _check(_lib.lrs_model_decode_greedy(self._h, n, _uptr(sq), _uptr(ft), _uptr(sp), n_steps,
                                            _uptr(out)))
        return out

    def decode_enqueue(self, first_tokens, start_pos, n_steps: int, seqs=None) -> None:
        ft = np.ascontiguousarray(first_tokens, dtype=np.uint32)
        sp = np.ascontiguousarray(start_pos, dtype=np.uint32)
        sq = np.ascontiguousarray(seqs if seqs is not None else range(ft.size), dtype=np.uint32)
        self._enq_keep = (ft, sp, sq)
        _check(_lib.lrs_model_decode_enqueue(self._h, ft.size, _uptr(sq), _uptr(ft), _uptr(sp),
                                             n_steps))

    def read_tokens(self, n_seqs: int, n_steps: int) -> np.ndarray:
        out = np.zeros((n_steps, n_seqs), dtype=np.uint32)
        _check(_lib.lrs_model_read_tokens(self._h, n_seqs, n_steps, _uptr(out)))
        return out

    def step_kernels(self) -> int:
        """Kernel launches per decode step of the last decode_enqueue (graph nodes)."""
        return int(_lib.lrs_model_step_kernels(self._h))

    def profile_step(self, tokens, pos, seqs=None):
        """One greedy step outside the graph with per-GEMV and per-layer
        attention CUDA events: returns (gemv_ms, gemv_launches, step_ms, attn_ms)."""
        t = np.ascontiguousarray(tokens, dtype=np.uint32)
        p = np.ascontiguousarray(pos, dtype=np.uint32)
        sq = np.ascontiguousarray(seqs if seqs is not None else range(t.size), dtype=np.uint32)
        g = np.zeros(1, np.float32)
        n = np.zeros(1, np.uint32)
        s = np.zeros(1, np.float32)
        a = np.zeros(1, np.float32)
        _check(_lib.lrs_model_profile_step(self._h, t.size, _uptr(sq), _uptr(t), _uptr(p),
                                           _fptr(g), _uptr(n), _fptr(s), _fptr(a)))
        return float(g[0]), int(n[0]), float(s[0]), float(a[0])

    def benchmark_tokens(self, prompt: Sequence[int], decode_tokens: int, seq: int = 0):
        """InferenceEngine::benchmark_tokens (src/engine.rs:189-223) on the device:
        returns the decode_tokens tokens fed to the decode steps."""
        _, first = self.prefill(prompt, 0, seq, want_logits=False)
        if decode_tokens == 0:
            return np.zeros(0, dtype=np.uint32)
        produced = self.decode_greedy([first], [len(prompt)], decode_tokens, [seq])[:, 0]
        return np.concatenate([[first], produced[:-1]]).astype(np.uint32)


# ------------------------------------------------------ benchmark configs --
class GgufFile:
    """GgufFile (src/gguf.rs:72-230) over the C reader: metadata, QuantTensor
    views into the mapped file, and the Qwen2 model description of
    GgufLoader::load (src/loader.rs:233-398) for lrs_model_create."""

    def __init__(self, path: str):
        h = _P()
        _check(_lib.lrs_gguf_open(os.fsencode(path), C.byref(h)))
        self._h = h

    def close(self):
        if self._h:
            _lib.lrs_gguf_close(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def version(self) -> int:
        return int(_lib.lrs_gguf_version(self._h))

    @property
    def tensor_count(self) -> int:
        return int(_lib.lrs_gguf_tensor_count(self._h))

    def metadata_u64(self, key: str) -> int:
        v = C.c_uint64()
        _check(_lib.lrs_gguf_metadata_u64(self._h, key.encode(), C.byref(v)))
        return v.value

    def metadata_f32(self, key: str) -> float:
        v = C.c_float()
        _check(_lib.lrs_gguf_metadata_f32(self._h, key.encode(), C.byref(v)))
        return v.value

    def metadata_str(self, key: str) -> str:
        v = C.c_char_p()
        _check(_lib.lrs_gguf_metadata_str(self._h, key.encode(), C.byref(v)))
        return v.value.decode()

    def tensor(self, name: str) -> QuantTensor:
        td = _TensorDesc()
        _check(_lib.lrs_gguf_tensor(self._h, name.encode(), C.byref(td)))
        buf = (C.c_uint8 * td.nbytes).from_address(td.data) if td.nbytes else b""
        return QuantTensor(np.frombuffer(buf, dtype=np.uint8), (td.rows, td.cols),
                           QuantType(td.ggml_type))

    def qwen2_desc(self, recipe: LoadQuantization = LoadQuantization.NONE):
        """The model description (valid while this object lives)."""
        out = C.POINTER(_ModelDesc)()
        _check(_lib.lrs_gguf_qwen2_desc(self._h, int(recipe), C.byref(out)))
        out._owner = self
        return out


# GGUF metadata value types (the format's numbering, src/gguf.rs:313-343)
GGUF_U32, GGUF_I32, GGUF_F32, GGUF_STR, GGUF_U64 = 4, 5, 6, 8, 10


def write_gguf(path: str, metadata, tensors, alignment: int = 32, version: int = 3) -> None:
    """Writes a GGUF file.  metadata: [(key, gguf_type, value)] with the scalar
    types above; tensors: [(name, ggml_type, dims in GGML order (row width
    first), bytes)].  Tensor data is aligned to `alignment`."""
    import struct

    def gstr(v: str) -> bytes:
        b = v.encode()
        return struct.pack("<Q", len(b)) + b

    fmt = {4: "<I", 5: "<i", 6: "<f", 10: "<Q"}
    head = bytearray(b"GGUF" + struct.pack("<IQQ", version, len(tensors), len(metadata)))
    for key, ty, val in metadata:
        head += gstr(key) + struct.pack("<I", ty)
        head += gstr(val) if ty == GGUF_STR else struct.pack(fmt[ty], val)
    off = 0
    offsets = []
    for name, ty, dims, data in tensors:
        head += gstr(name) + struct.pack("<I", len(dims))
        head += b"".join(struct.pack("<Q", d) for d in dims)
        head += struct.pack("<IQ", ty, off)
        offsets.append(off)
        off += (len(data) + alignment - 1) // alignment * alignment
    data_start = (len(head) + alignment - 1) // alignment * alignment
    with open(path, "wb") as f:
        f.write(head)
        f.write(b"\0" * (data_start - len(head)))
        for (name, ty, dims, data), o in zip(tensors, offsets):
            f.seek(data_start + o)
            f.write(data)
        f.truncate(data_start + off)


def write_qwen2_gguf(path: str, desc, alignment: int = 32, retype=None) -> None:
    """Writes the model behind an lrs_model_desc as a Qwen2 GGUF file with the
    names GgufLoader expects (src/loader.rs:244-398); a tied head (the
    embedding's bytes) is written without output.weight.

    retype(name, rows, cols) -> QuantType or None re-encodes F32 matrices per
    tensor, as a quantizing tool writes mixed files (Q4_K_M-style files hold
    several block types across tensors and layers)."""
    d = desc.contents
    c = d.config
    h, kvw = c.hidden_size, c.num_key_value_heads * c.head_dim
    meta = [("general.architecture", GGUF_STR, "qwen2"),
            ("general.alignment", GGUF_U32, alignment),
            ("qwen2.embedding_length", GGUF_U64, c.hidden_size),
            ("qwen2.feed_forward_length", GGUF_U64, c.intermediate_size),
            ("qwen2.attention.head_count", GGUF_U32, c.num_attention_heads),
            ("qwen2.attention.head_count_kv", GGUF_U32, c.num_key_value_heads),
            ("qwen2.block_count", GGUF_U32, c.num_hidden_layers),
            ("qwen2.attention.layer_norm_rms_epsilon", GGUF_F32, c.rms_norm_eps),
            ("qwen2.rope.freq_base", GGUF_F32, c.rope_theta),
            ("qwen2.context_length", GGUF_U64, c.max_position_embeddings)]
    tensors = []

    def mat(name, td):
        data = bytes((C.c_uint8 * td.nbytes).from_address(td.data))
        ty = td.ggml_type
        want = retype(name, td.rows, td.cols) if retype else None
        if want is not None and int(want) != ty:
            if ty != int(QuantType.F32):
                raise LrsError(1, f"{name}: only F32 tensors can be re-encoded")
            q = QuantTensor.quantize(np.frombuffer(data, dtype=np.float32), td.rows, td.cols, want)
            data, ty = q.data.tobytes(), int(q.quant_type)
        tensors.append((name, ty, [td.cols, td.rows], data))

    def vec(name, ptr, n):
        if ptr:
            tensors.append((name, int(QuantType.F32), [n],
                            bytes((C.c_uint8 * (4 * n)).from_address(ptr))))

    mat("token_embd.weight", d.embed_tokens)
    vec("output_norm.weight", d.final_norm, h)
    for i in range(c.num_hidden_layers):
        L, p = d.layers[i], f"blk.{i}"
        vec(f"{p}.attn_norm.weight", L.input_layernorm, h)
        mat(f"{p}.attn_q.weight", L.q_proj)
        vec(f"{p}.attn_q.bias", L.q_bias, h)
        mat(f"{p}.attn_k.weight", L.k_proj)
        vec(f"{p}.attn_k.bias", L.k_bias, kvw)
        mat(f"{p}.attn_v.weight", L.v_proj)
        vec(f"{p}.attn_v.bias", L.v_bias, kvw)
        mat(f"{p}.attn_output.weight", L.o_proj)
        vec(f"{p}.ffn_norm.weight", L.post_attention_layernorm, h)
        mat(f"{p}.ffn_gate.weight", L.gate_proj)
        mat(f"{p}.ffn_up.weight", L.up_proj)
        mat(f"{p}.ffn_down.weight", L.down_proj)
    if d.lm_head.data != d.embed_tokens.data:
        mat("output.weight", d.lm_head)
    write_gguf(path, meta, tensors, alignment)


class SafetensorsFile:
    """SafetensorStore (src/loader.rs:535-645) over the C reader: a model
    directory's shards, tensor views, and the description of
    SafetensorsLoader::load (src/loader.rs:83-230) for lrs_model_create."""

    def __init__(self, model_dir: str):
        h = _P()
        _check(_lib.lrs_st_open(os.fsencode(model_dir), C.byref(h)))
        self._h = h

    def close(self):
        if self._h:
            _lib.lrs_st_close(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def tensor_count(self) -> int:
        return int(_lib.lrs_st_tensor_count(self._h))

    def tensor(self, name: str) -> QuantTensor:
        td = _TensorDesc()
        _check(_lib.lrs_st_tensor(self._h, name.encode(), C.byref(td)))
        buf = (C.c_uint8 * td.nbytes).from_address(td.data) if td.nbytes else b""
        return QuantTensor(np.frombuffer(buf, dtype=np.uint8), (td.rows, td.cols),
                           QuantType(td.ggml_type))

    def qwen2_desc(self, recipe: LoadQuantization = LoadQuantization.NONE):
        """The model description (valid while this object lives)."""
        out = C.POINTER(_ModelDesc)()
        _check(_lib.lrs_st_qwen2_desc(self._h, int(recipe), C.byref(out)))
        out._owner = self
        return out


class LoadedModel:
    """ModelLoader::load (src/loader.rs:46-79): a .gguf file, a .safetensors
    file or a model directory, by the reference's format detection."""

    def __init__(self, path: str, recipe: LoadQuantization = LoadQuantization.NONE):
        h = _P()
        d = C.POINTER(_ModelDesc)()
        _check(_lib.lrs_model_load(os.fsencode(path), int(recipe), C.byref(h), C.byref(d)))
        self._h = h
        self._desc = d

    def desc(self):
        p = C.pointer(self._desc.contents)
        p._owner = self  # the description stays valid while the pointer lives
        return p

    def close(self):
        if self._h:
            _lib.lrs_loaded_close(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


_ST_DTYPES = {"F32": (np.float32, 4), "F16": (np.float16, 2), "BF16": (None, 2)}


def write_safetensors(path: str, tensors, metadata=None) -> None:
    """Writes a .safetensors file: tensors = [(name, dtype, shape, bytes)],
    data in the listed order; metadata: optional {str: str}."""
    import json
    import struct
    header = {}
    off = 0
    for name, dtype, shape, data in tensors:
        header[name] = {"dtype": dtype, "shape": list(shape), "data_offsets": [off, off + len(data)]}
        off += len(data)
    if metadata:
        header["__metadata__"] = dict(metadata)
    h = json.dumps(header, separators=(",", ":")).encode()
    h += b" " * ((8 - len(h) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for _, _, _, data in tensors:
            f.write(data)


def _f32_to(values: np.ndarray, dtype: str) -> bytes:
    v = np.ascontiguousarray(values, dtype=np.float32)
    if dtype == "F32":
        return v.tobytes()
    if dtype == "F16":
        return v.astype(np.float16).tobytes()
    b = v.view(np.uint32)  # BF16, round to nearest even
    r = ((b + 0x7FFF + ((b >> 16) & 1)) >> 16).astype(np.uint16)
    r = np.where(np.isnan(v), (b >> 16).astype(np.uint16) | 0x40, r)
    return r.tobytes()


def write_qwen2_safetensors(model_dir: str, desc, dtype: str = "F32", shards: int = 1,
                            config_extra=None) -> None:
    """Writes the F32 model behind an lrs_model_desc as a Hugging Face Qwen2
    directory (config.json, model.safetensors or `shards` files with
    model.safetensors.index.json), tensors in `dtype` (F32, F16 or BF16); a
    tied head is written without lm_head.weight."""
    import json
    d = desc.contents
    c = d.config
    h, kvw = c.hidden_size, c.num_key_value_heads * c.head_dim
    os.makedirs(model_dir, exist_ok=True)
    tensors = []

    def f32(ptr, n):
        return np.frombuffer((C.c_float * n).from_address(ptr), dtype=np.float32)

    def mat(name, td):
        if td.ggml_type != int(QuantType.F32):
            raise LrsError(1, f"{name}: write_qwen2_safetensors takes an F32 model")
        tensors.append((name, dtype, [td.rows, td.cols], _f32_to(f32(td.data, td.rows * td.cols), dtype)))

    def vec(name, ptr, n):
        if ptr:
            tensors.append((name, dtype, [n], _f32_to(f32(ptr, n), dtype)))

    mat("model.embed_tokens.weight", d.embed_tokens)
    vec("model.norm.weight", d.final_norm, h)
    for i in range(c.num_hidden_layers):
        L, p = d.layers[i], f"model.layers.{i}"
        vec(f"{p}.input_layernorm.weight", L.input_layernorm, h)
        vec(f"{p}.post_attention_layernorm.weight", L.post_attention_layernorm, h)
        mat(f"{p}.self_attn.q_proj.weight", L.q_proj)
        vec(f"{p}.self_attn.q_proj.bias", L.q_bias, h)
        mat(f"{p}.self_attn.k_proj.weight", L.k_proj)
        vec(f"{p}.self_attn.k_proj.bias", L.k_bias, kvw)
        mat(f"{p}.self_attn.v_proj.weight", L.v_proj)
        vec(f"{p}.self_attn.v_proj.bias", L.v_bias, kvw)
        mat(f"{p}.self_attn.o_proj.weight", L.o_proj)
        mat(f"{p}.mlp.gate_proj.weight", L.gate_proj)
        mat(f"{p}.mlp.up_proj.weight", L.up_proj)
        mat(f"{p}.mlp.down_proj.weight", L.down_proj)
    tied = d.lm_head.data == d.embed_tokens.data
    if not tied:
        mat("lm_head.weight", d.lm_head)
    cfg = {"model_type": "qwen2", "architectures": ["Qwen2ForCausalLM"],
           "hidden_size": c.hidden_size, "intermediate_size": c.intermediate_size,
           "num_attention_heads": c.num_attention_heads,
           "num_key_value_heads": c.num_key_value_heads,
           "num_hidden_layers": c.num_hidden_layers, "vocab_size": c.vocab_size,
           "rms_norm_eps": float(np.float32(c.rms_norm_eps)),
           "rope_theta": float(np.float32(c.rope_theta)),
           "max_position_embeddings": c.max_position_embeddings,
           "tie_word_embeddings": bool(tied), "torch_dtype": "float32"}
    if config_extra:
        cfg.update(config_extra)
    with open(os.path.join(model_dir, "config.json"), "w") as f:
        json.dump(cfg, f, indent=2)
    if shards <= 1:
        write_safetensors(os.path.join(model_dir, "model.safetensors"), tensors)
        return
    per = (len(tensors) + shards - 1) // shards
    weight_map = {}
    for k in range(shards):
        fname = f"model-{k + 1:05d}-of-{shards:05d}.safetensors"
        part = tensors[k * per:(k + 1) * per]
        write_safetensors(os.path.join(model_dir, fname), part)
        weight_map.update({t[0]: fname for t in part})
    with open(os.path.join(model_dir, "model.safetensors.index.json"), "w") as f:
        json.dump({"metadata": {"total_size": sum(len(t[3]) for t in tensors)},
                   "weight_map": weight_map}, f)


def sampler_check(params: Sampler, vocab: int) -> None:
    """validate_sampling (src/engine.rs:327-339) plus the device top_k limit."""
    _check(_lib.lrs_sampler_check(C.byref(params), vocab))


def tp_unique_id() -> bytes:
    """The 128-byte NCCL id for lrs_model_create_tp (rank 0 makes it)."""
    buf = C.create_string_buffer(128)
    _check(_lib.lrs_tp_unique_id(buf))
    return buf.raw


def config_c0() -> LlamaConfig:
    """Qwen2.5-0.5B shape (benchmark config 0)."""
    return LlamaConfig(896, 4864, 14, 2, 24, 151936, 1e-6, 1e6, 32768, 64, True)


def config_c2() -> LlamaConfig:
    """Qwen2.5-1.5B shape (benchmark config 2)."""
    return LlamaConfig(1536, 8960, 12, 2, 28, 151936, 1e-6, 1e6, 32768, 128, True)


def config_c3() -> LlamaConfig:
    """Qwen2.5-7B shape (benchmark config 3)."""
    return LlamaConfig(3584, 18944, 28, 4, 28, 152064, 1e-6, 1e6, 32768, 128, False)


def config_c4() -> LlamaConfig:
    """Qwen2.5-32B shape (benchmark config 4)."""
    return LlamaConfig(5120, 27648, 40, 8, 64, 152064, 1e-6, 1e6, 32768, 128, False)


def prompt_tokens(seed: int, n: int, vocab: int, sequence: int = 0) -> np.ndarray:
    """Uniform prompt token ids of the benchmark workloads (numpy PCG64).

    Sequence 0 uses seed + 1000; sequence g > 0 of a multi-sequence workload
    uses the seed sequence [seed, g]."""
    rng = np.random.default_rng(seed + 1000 if sequence == 0 else [seed, sequence])
    return rng.integers(0, vocab, n, dtype=np.int64).astype(np.uint32)

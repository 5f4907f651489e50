"""ctypes binding of the engine API in ``include/opc_engine.h`` (the ``bf_engine_*`` calls of the
reference's C runtime, runtime/include/opacc1ty.h:69-212, implemented in
``csrc/opc_engine.cu`` inside ``libopc_b200.so``).

    from opac1ty_b200.engine import Engine
    with Engine("model.bf2") as eng:
        logits = eng.forward([1, 2, 3])          # np.float32 [vocab]
        ids = eng.generate_tokens([1, 2, 3], 16, temperature=0)
"""

from __future__ import annotations

import ctypes
from typing import Optional, Sequence

import numpy as np

from . import _lib


class ModelConfig(ctypes.Structure):
    _fields_ = [
        ("architecture", ctypes.c_char * 64),
        ("vocab_size", ctypes.c_uint32),
        ("hidden_size", ctypes.c_uint32),
        ("intermediate_size", ctypes.c_uint32),
        ("num_hidden_layers", ctypes.c_uint32),
        ("num_attention_heads", ctypes.c_uint32),
        ("num_kv_heads", ctypes.c_uint32),
        ("max_position_embeddings", ctypes.c_uint32),
        ("rope_theta", ctypes.c_float),
        ("head_dim", ctypes.c_uint32),
    ]


class SamplingParams(ctypes.Structure):
    _fields_ = [
        ("temperature", ctypes.c_float),
        ("top_p", ctypes.c_float),
        ("top_k", ctypes.c_int32),
        ("repetition_penalty", ctypes.c_float),
        ("seed", ctypes.c_uint32),
    ]


class Stats(ctypes.Structure):
    _fields_ = [
        ("total_tokens_generated", ctypes.c_uint64),
        ("total_time_seconds", ctypes.c_double),
        ("tokens_per_second", ctypes.c_double),
        ("peak_memory_bytes", ctypes.c_size_t),
        ("n_kernel_dispatches", ctypes.c_uint32),
    ]


_P = ctypes.c_void_p
_I32P = ctypes.POINTER(ctypes.c_int32)
_F32P = ctypes.POINTER(ctypes.c_float)

# name -> (restype, argtypes); every function include/opc_engine.h declares
PROTOTYPES = {
    "bf_engine_create": (_P, [ctypes.c_char_p]),
    "bf_engine_create_ex": (_P, [ctypes.c_char_p, ctypes.c_int32, ctypes.c_uint32]),
    "bf_engine_destroy": (None, [_P]),
    "bf_engine_get_config": (ctypes.POINTER(ModelConfig), [_P]),
    "bf_engine_get_error": (ctypes.c_char_p, [_P]),
    "bf_engine_vocab_size": (ctypes.c_uint32, [_P]),
    "bf_engine_generate": (ctypes.c_int32, [_P, ctypes.c_char_p, ctypes.c_uint32, ctypes.POINTER(SamplingParams), _P]),
    "bf_engine_generate_tokens": (ctypes.c_int32, [_P, _I32P, ctypes.c_uint32, ctypes.c_uint32,
                                                   ctypes.POINTER(SamplingParams), _I32P]),
    "bf_engine_forward": (ctypes.c_int, [_P, _I32P, ctypes.c_uint32, _F32P, ctypes.c_uint32]),
    "bf_engine_prefill": (ctypes.c_int, [_P, _I32P, ctypes.c_uint32]),
    "bf_engine_forward_step": (ctypes.c_int, [_P, ctypes.c_int32, _F32P, ctypes.c_uint32]),
    "bf_engine_reset_kv_cache": (None, [_P]),
    "bf_engine_kv_cache_size": (ctypes.c_size_t, [_P]),
    "bf_engine_position": (ctypes.c_uint32, [_P]),
    "bf_engine_get_stats": (None, [_P, ctypes.POINTER(Stats)]),
    "bf_engine_reset_stats": (None, [_P]),
    "bf_version": (ctypes.c_char_p, []),
    "bf_has_metal_gpu": (ctypes.c_int, []),
    "bf_has_cuda_gpu": (ctypes.c_int, []),
}

_bound = None


def lib():
    """The shared library with the engine prototypes applied."""
    global _bound
    if _bound is None:
        L = _lib.load()
        for name, (res, args) in PROTOTYPES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _bound = L
    return _bound


def default_sampling() -> SamplingParams:
    """BF_DEFAULT_SAMPLING as exported by the library."""
    return SamplingParams.in_dll(lib(), "BF_DEFAULT_SAMPLING")


class EngineError(RuntimeError):
    pass


def _i32(tokens: Sequence[int]) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(tokens, dtype=np.int32).reshape(-1))


class Engine:
    """One loaded .bf2 model on one GPU (``bf_engine_create_ex``)."""

    def __init__(self, path: str, device: int = 0, max_context: int = 0):
        self._L = lib()
        self._h = self._L.bf_engine_create_ex(str(path).encode(), int(device), int(max_context))
        if not self._h:
            raise EngineError("bf_engine_create returned NULL")
        err = self._L.bf_engine_get_error(self._h)
        if err:
            msg = err.decode(errors="replace")
            self.close()
            raise EngineError(msg)
        c = self._L.bf_engine_get_config(self._h).contents
        self.config = {name: (getattr(c, name).decode() if name == "architecture" else getattr(c, name))
                       for name, _ in ModelConfig._fields_}
        self.vocab_size = int(c.vocab_size)

    def _check(self, rc: int, what: str):
        if rc != 0:
            err = self._L.bf_engine_get_error(self._h)
            raise EngineError(f"{what}: {err.decode(errors='replace') if err else 'failed'}")

    def forward(self, tokens: Sequence[int]) -> np.ndarray:
        t = _i32(tokens)
        out = np.empty(self.vocab_size, dtype=np.float32)
        self._check(self._L.bf_engine_forward(self._h, t.ctypes.data_as(_I32P), t.size, out.ctypes.data_as(_F32P),
                                              self.vocab_size), "bf_engine_forward")
        return out

    def prefill(self, tokens: Sequence[int]):
        t = _i32(tokens)
        self._check(self._L.bf_engine_prefill(self._h, t.ctypes.data_as(_I32P), t.size), "bf_engine_prefill")

    def forward_step(self, token: int) -> np.ndarray:
        out = np.empty(self.vocab_size, dtype=np.float32)
        self._check(self._L.bf_engine_forward_step(self._h, int(token), out.ctypes.data_as(_F32P), self.vocab_size),
                    "bf_engine_forward_step")
        return out

    def generate_tokens(self, prompt: Sequence[int], max_new_tokens: int, temperature: float = 0.0,
                        top_p: float = 0.0, top_k: int = 0, repetition_penalty: float = 1.0, seed: int = 0) -> list:
        t = _i32(prompt)
        out = np.zeros(max(int(max_new_tokens), 1), dtype=np.int32)
        p = SamplingParams(temperature, top_p, top_k, repetition_penalty, seed)
        n = self._L.bf_engine_generate_tokens(self._h, t.ctypes.data_as(_I32P) if t.size else None, t.size,
                                              int(max_new_tokens), ctypes.byref(p), out.ctypes.data_as(_I32P))
        if n < 0:
            self._check(n, "bf_engine_generate_tokens")
        return out[:n].tolist()

    def generate(self, prompt: str, max_new_tokens: int, params: Optional[SamplingParams] = None) -> int:
        """The text API: byte-level prompt, nothing printed; returns the tokens generated."""
        n = self._L.bf_engine_generate(self._h, prompt.encode(), int(max_new_tokens),
                                       ctypes.byref(params) if params is not None else None, None)
        if n < 0:
            self._check(n, "bf_engine_generate")
        return int(n)

    def reset(self):
        self._L.bf_engine_reset_kv_cache(self._h)

    @property
    def position(self) -> int:
        return int(self._L.bf_engine_position(self._h))

    @property
    def kv_cache_size(self) -> int:
        return int(self._L.bf_engine_kv_cache_size(self._h))

    def stats(self) -> dict:
        s = Stats()
        self._L.bf_engine_get_stats(self._h, ctypes.byref(s))
        return {name: getattr(s, name) for name, _ in Stats._fields_}

    def reset_stats(self):
        self._L.bf_engine_reset_stats(self._h)

    def close(self):
        if getattr(self, "_h", None):
            self._L.bf_engine_destroy(self._h)
            self._h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

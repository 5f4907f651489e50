"""CPU oracle for the fused 2-bit codebook dequant-matmul path.

TEST INFRASTRUCTURE ONLY: imported by tests/, by ``__graft_entry__.smoke()`` and by the
CPU-baseline legs of ``bench.py`` as the checker / timed CPU baseline.  The product package
(``opac1ty_b200``) never imports it.

Two restatements of opacc1ty's ``dequantize_layer`` (opacc1ty/export/converter.py:26-67):
``dequantize_np`` (vectorised numpy: gather + trim + ordered row replacement) and the plain-C
``oracle_dequant`` in opc_oracle.c.  Both are pinned bit-for-bit to fixtures produced by the
reference itself (tests/golden/make_golden.py).  ``gemv_f64`` recomputes y = x . W^T in double.
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path
from typing import Optional

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "libopc_oracle.so"

_lib: Optional[ctypes.CDLL] = None


def build() -> Path:
    """Compile opc_oracle.c with the Makefile beside it (gcc)."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB_PATH


def load() -> ctypes.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists() or LIB_PATH.stat().st_mtime < (HERE / "opc_oracle.c").stat().st_mtime:
        build()
    lib = ctypes.CDLL(str(LIB_PATH))
    P = ctypes.c_void_p
    lib.oracle_dequant.restype = ctypes.c_int
    lib.oracle_dequant.argtypes = [ctypes.c_int32] * 4 + [P, P, ctypes.c_int32, P, P, P]
    lib.oracle_gemv_f64.restype = None
    lib.oracle_gemv_f64.argtypes = [ctypes.c_int32, ctypes.c_int32, P, ctypes.c_int64, ctypes.c_int32, P,
                                    ctypes.c_int64, P, ctypes.c_int64]
    lib.oracle_gemv_cpu.restype = ctypes.c_int
    lib.oracle_gemv_cpu.argtypes = [ctypes.c_int32, ctypes.c_int32, P, P, P, P, ctypes.c_int32, P, P, ctypes.c_int32]
    lib.oracle_half_to_float.restype = ctypes.c_float
    lib.oracle_half_to_float.argtypes = [ctypes.c_uint16]
    lib.oracle_float_to_half.restype = ctypes.c_uint16
    lib.oracle_float_to_half.argtypes = [ctypes.c_float]
    _lib = lib
    return lib


def _np(t, dtype=None) -> np.ndarray:
    if hasattr(t, "detach"):  # torch tensor
        t = t.detach().cpu().numpy()
    a = np.asarray(t)
    if dtype is not None:
        a = a.astype(dtype, copy=False)
    return np.ascontiguousarray(a)


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


def layer_arrays(layer: dict):
    """(cb fp16 [M][4][svs], idx uint8 [M][G], ov fp16 [n][K] or None, oi int64 [n] or None, M, K)."""
    out_f, in_f = (int(v) for v in layer["shape"])
    cb = _np(layer["codebooks"], np.float16)
    if cb.ndim == 2:
        cb = cb[:, :, None]
    idx = _np(layer["indices"], np.uint8)
    ov, oi = layer.get("outlier_values"), layer.get("outlier_indices")
    if ov is None or oi is None or len(oi) == 0:
        ov, oi = None, None
    else:
        ov = _np(ov, np.float16)
        oi = _np(oi, np.int64)
    return cb, idx, ov, oi, out_f, in_f


def dequantize_np(layer: dict) -> np.ndarray:
    """Vectorised restatement of dequantize_layer for "quantized" layers (fp16 [M][Kc]).
    "sparse_outlier" layers (element-wise outliers, the layer type format/header.py:57-60
    reserves): the codebook lookup, then W[r][c] = v per entry in order (the last entry of a
    repeated position wins)."""
    if layer.get("type") == "sparse_outlier":
        base = dict(layer, type="quantized", outlier_values=None, outlier_indices=None)
        w = dequantize_np(base)
        ov, oi = layer.get("outlier_values"), layer.get("outlier_indices")
        if ov is not None and oi is not None:
            vals = _np(ov, np.float16).reshape(-1)
            pos = _np(oi, np.int64).reshape(-1, 2)
            M, K = w.shape
            if len(pos) and (pos.min() < 0 or (pos[:, 0] >= M).any() or (pos[:, 1] >= K).any()):
                raise IndexError("element outlier position out of range")
            for (r, c), v in zip(pos, vals):
                w[r, c] = v
        return w
    cb, idx, ov, oi, M, K = layer_arrays(layer)
    svs = cb.shape[2]
    if idx.size and int(idx.max()) > 3:
        raise IndexError("codebook index out of range")
    rows = np.arange(M)[:, None]
    w = cb[rows, idx.astype(np.int64)]          # [M][G][svs]  (converter.py:48-53)
    w = w.reshape(M, -1)[:, :K]                 # trim (converter.py:56)
    w = np.ascontiguousarray(w)
    if ov is not None:
        for i, r in enumerate(oi):               # ordered replacement (converter.py:59-63)
            w[int(r)] = ov[i]
    return w


def dequantize_c(layer: dict) -> np.ndarray:
    """The plain-C restatement (opc_oracle.c: oracle_dequant)."""
    lib = load()
    cb, idx, ov, oi, M, K = layer_arrays(layer)
    svs, G = cb.shape[2], idx.shape[1]
    Kc = min(G * svs, K)
    w = np.empty((M, Kc), dtype=np.float16)
    n = 0 if ov is None else len(oi)
    rc = lib.oracle_dequant(M, K, svs, G, _ptr(cb), _ptr(idx), n, _ptr(ov) if n else None,
                            _ptr(oi) if n else None, _ptr(w))
    if rc == -1:
        raise IndexError("codebook index out of range")
    if rc == -2:
        raise IndexError("outlier row id out of range")
    if rc == -3:
        raise ValueError("outlier rows do not match the trimmed width")
    return w


def gemv_f64(w: np.ndarray, x: np.ndarray) -> np.ndarray:
    """y64 [batch][M] = x . W^T in double (x fp16 [batch][K] or [K], W fp16 [M][K])."""
    lib = load()
    w = _np(w, np.float16)
    x = _np(x, np.float16)
    squeeze = x.ndim == 1
    if squeeze:
        x = x[None, :]
    M, K = w.shape
    B = x.shape[0]
    y = np.empty((B, M), dtype=np.float64)
    lib.oracle_gemv_f64(M, K, _ptr(w), w.strides[0] // 2, B, _ptr(x), x.strides[0] // 2, _ptr(y), M)
    return y[0] if squeeze else y


def outlier_slots(M: int, oi: Optional[np.ndarray]) -> Optional[np.ndarray]:
    """slot[r] = index of row r's outlier values (last occurrence wins) or -1."""
    if oi is None:
        return None
    slot = np.full(M, -1, dtype=np.int32)
    for i, r in enumerate(oi):
        slot[int(r)] = i
    return slot


def gemv_cpu(layer_or_arrays, x: np.ndarray, threads: int = 0) -> np.ndarray:
    """The reference CPU path (dequantize + fp32 dot, svs == 1) on ``threads`` host threads."""
    lib = load()
    if isinstance(layer_or_arrays, dict):
        cb, idx, ov, oi, M, K = layer_arrays(layer_or_arrays)
        slot = outlier_slots(M, oi)
        arrays = (cb, idx, ov, slot, M, K)
    else:
        arrays = layer_or_arrays
    cb, idx, ov, slot, M, K = arrays
    if cb.shape[-1] != 1 if cb.ndim == 3 else False:
        raise ValueError("gemv_cpu: sub_vector_size must be 1")
    x = _np(x, np.float16)
    squeeze = x.ndim == 1
    if squeeze:
        x = x[None, :]
    B = x.shape[0]
    y = np.empty((B, M), dtype=np.float16)
    threads = threads or os.cpu_count() or 1
    rc = lib.oracle_gemv_cpu(M, K, _ptr(np.ascontiguousarray(cb)), _ptr(idx), _ptr(ov) if ov is not None else None,
                             _ptr(slot) if slot is not None else None, B, _ptr(x), _ptr(y), threads)
    if rc != 0:
        raise MemoryError("oracle_gemv_cpu failed")
    return y[0] if squeeze else y


def rel_err(y: np.ndarray, y64: np.ndarray) -> float:
    """Norm-wise relative error max|y - y64| / max|y64| (the parity metric of the GEMV)."""
    y = np.asarray(y, dtype=np.float64)
    denom = float(np.max(np.abs(y64))) or 1.0
    return float(np.max(np.abs(y - y64))) / denom

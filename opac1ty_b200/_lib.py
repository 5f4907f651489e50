"""ctypes binding of the C ABI in ``include/opc_b200.h`` (``libopc_b200.so``).

The shared library is built in-tree by ``opac1ty_b200.build.build_library`` (called by
``__graft_entry__.build()``).  Nothing here falls back to a CPU or PyTorch implementation: if
the library is missing or cannot be loaded, every compute entry point raises.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path
from typing import Optional

LIB_NAME = "libopc_b200.so"
LIB_PATH = Path(__file__).resolve().parent / LIB_NAME

OPC_OK = 0
OPC_ERR_INVALID = -1
OPC_ERR_UNSUPPORTED = -2
OPC_ERR_CUDA = -3
OPC_ERR_WORKSPACE = -4
OPC_ERR_DEVICE = -5
OPC_CHAIN_L2_PREFETCH = 1
OPC_CHAIN_FORM_AUTO = 0
OPC_CHAIN_FORM_BARRIER = 1
OPC_CHAIN_FORM_DATAFLOW = 2
OPC_PEER_HANDLE_BYTES = 64
OPC_MAX_RANKS = 8

_ERR_NAMES = {
    OPC_ERR_INVALID: "OPC_ERR_INVALID",
    OPC_ERR_UNSUPPORTED: "OPC_ERR_UNSUPPORTED",
    OPC_ERR_CUDA: "OPC_ERR_CUDA",
    OPC_ERR_WORKSPACE: "OPC_ERR_WORKSPACE",
    OPC_ERR_DEVICE: "OPC_ERR_DEVICE",
}


class OpcError(RuntimeError):
    """A C-ABI call returned a negative status; ``code`` is the OPC_ERR_* value."""

    def __init__(self, code: int, message: str):
        super().__init__(f"{_ERR_NAMES.get(code, code)}: {message}")
        self.code = code


class LayerPlan(ctypes.Structure):
    _fields_ = [
        ("M", ctypes.c_int32),
        ("K", ctypes.c_int32),
        ("n_outliers", ctypes.c_int32),
        ("sub_vector_size", ctypes.c_int32),
        ("M_pad", ctypes.c_int32),
        ("K_pad", ctypes.c_int32),
        ("row_tiles", ctypes.c_int32),
        ("k_units", ctypes.c_int32),
        ("outlier_tiles", ctypes.c_int32),
        ("outlier_k_units", ctypes.c_int32),
        ("packed_units", ctypes.c_int64),
        ("total_units", ctypes.c_int64),
        ("units_bytes", ctypes.c_int64),
        ("codebook_bytes", ctypes.c_int64),
        ("tile_mask_bytes", ctypes.c_int64),
        ("outlier_rows_bytes", ctypes.c_int64),
    ]


class Layer(ctypes.Structure):
    _fields_ = [
        ("plan", LayerPlan),
        ("units", ctypes.c_void_p),
        ("codebooks", ctypes.c_void_p),
        ("tile_mask", ctypes.c_void_p),
        ("outlier_rows", ctypes.c_void_p),
    ]


class ChainStep(ctypes.Structure):
    _fields_ = [
        ("layer", ctypes.POINTER(Layer)),
        ("x", ctypes.c_void_p),
        ("ldx", ctypes.c_int64),
        ("y", ctypes.c_void_p),
        ("ldy", ctypes.c_int64),
    ]


class DeviceProps(ctypes.Structure):
    _fields_ = [
        ("name", ctypes.c_char * 256),
        ("device", ctypes.c_int32),
        ("sm_count", ctypes.c_int32),
        ("cc_major", ctypes.c_int32),
        ("cc_minor", ctypes.c_int32),
        ("total_mem_bytes", ctypes.c_int64),
        ("max_smem_per_block_optin", ctypes.c_int32),
        ("max_threads_per_block", ctypes.c_int32),
        ("l2_bytes", ctypes.c_int32),
        ("warp_size", ctypes.c_int32),
    ]


# Exported symbols and their prototypes: (restype, argtypes).  Kept in the order of the header.
_c = ctypes
PROTOTYPES = {
    "opc_version": (_c.c_char_p, []),
    "opc_last_error": (_c.c_char_p, []),
    "opc_device_info": (_c.c_int, [_c.c_int32, _c.POINTER(DeviceProps)]),
    "opc_plan_layer": (_c.c_int, [_c.c_int32, _c.c_int32, _c.c_int32, _c.c_int32, _c.POINTER(LayerPlan)]),
    "opc_repack_layer": (
        _c.c_int,
        [_c.POINTER(Layer), _c.c_void_p, _c.c_void_p, _c.c_void_p, _c.POINTER(_c.c_int64), _c.c_int32, _c.c_void_p],
    ),
    "opc_count_distinct_ids": (_c.c_int32, [_c.POINTER(_c.c_int64), _c.c_int32]),
    "opc_gemv_workspace_bytes": (_c.c_size_t, [_c.POINTER(LayerPlan), _c.c_int32, _c.c_int32]),
    "opc_workspace_init": (_c.c_int, [_c.c_void_p, _c.c_size_t, _c.c_void_p]),
    "opc_gemv": (
        _c.c_int,
        [_c.POINTER(Layer), _c.c_void_p, _c.c_int64, _c.c_void_p, _c.c_int64, _c.c_int32, _c.c_void_p, _c.c_size_t,
         _c.c_void_p],
    ),
    "opc_gemv_noalloc": (
        _c.c_int, [_c.POINTER(Layer), _c.c_void_p, _c.c_int64, _c.c_void_p, _c.c_int64, _c.c_int32, _c.c_void_p],
    ),
    "opc_gemm": (
        _c.c_int, [_c.POINTER(Layer), _c.c_void_p, _c.c_int64, _c.c_void_p, _c.c_int64, _c.c_int32, _c.c_void_p],
    ),
    "opc_chain_create": (_c.c_int, [_c.POINTER(ChainStep), _c.c_int32, _c.c_int32, _c.POINTER(_c.c_void_p)]),
    "opc_chain_create_ex": (
        _c.c_int, [_c.POINTER(ChainStep), _c.c_int32, _c.c_int32, _c.c_int32, _c.POINTER(_c.c_void_p)],
    ),
    "opc_chain_form": (_c.c_int32, [_c.c_void_p]),
    "opc_chain_launch": (_c.c_int, [_c.c_void_p, _c.c_void_p]),
    "opc_chain_destroy": (_c.c_int, [_c.c_void_p]),
    "opc_chain_trace_bytes": (_c.c_size_t, [_c.c_void_p]),
    "opc_chain_set_option": (_c.c_int, [_c.c_void_p, _c.c_int32, _c.c_int32]),
    "opc_chain_grid": (_c.c_int32, [_c.c_void_p]),
    "opc_chain_set_trace": (_c.c_int, [_c.c_void_p, _c.c_void_p]),
    "opc_peer_alloc": (_c.c_int, [_c.c_size_t, _c.POINTER(_c.c_void_p), _c.c_void_p]),
    "opc_peer_open": (_c.c_int, [_c.c_void_p, _c.POINTER(_c.c_void_p)]),
    "opc_peer_close": (_c.c_int, [_c.c_void_p]),
    "opc_peer_free": (_c.c_int, [_c.c_void_p]),
    "opc_chain_tp_scratch_bytes": (
        _c.c_int, [_c.POINTER(ChainStep), _c.c_int32, _c.c_int32, _c.c_int32, _c.POINTER(_c.c_size_t)],
    ),
    "opc_chain_tp_info": (
        _c.c_int,
        [_c.POINTER(ChainStep), _c.c_int32, _c.c_int32, _c.c_int32, _c.c_void_p, _c.c_size_t, _c.c_size_t,
         _c.c_void_p, _c.POINTER(_c.c_size_t)],
    ),
    "opc_chain_create_tp": (
        _c.c_int,
        [_c.POINTER(ChainStep), _c.c_int32, _c.c_int32, _c.c_int32, _c.c_int32, _c.POINTER(_c.c_void_p),
         _c.POINTER(_c.c_void_p), _c.POINTER(_c.c_void_p)],
    ),
    "opc_dequant": (_c.c_int, [_c.POINTER(Layer), _c.c_void_p, _c.c_int64, _c.c_void_p]),
    "opc_set_gemm_crossover": (_c.c_int, [_c.c_int32]),
    "opc_gemm_crossover": (_c.c_int32, []),
    "opc_xxh64": (_c.c_uint64, [_c.c_void_p, _c.c_size_t, _c.c_uint64]),
    "opc_coo_build": (_c.c_int, [_c.c_int32, _c.c_int32, _c.c_int32, _c.c_void_p, _c.c_void_p, _c.c_void_p,
                                _c.c_void_p, _c.c_int64, _c.c_void_p, _c.c_void_p, _c.c_void_p, _c.c_void_p,
                                _c.POINTER(_c.c_int64)]),
    "opc_coo_gemv": (_c.c_int, [_c.c_int32, _c.c_void_p, _c.c_void_p, _c.c_void_p, _c.c_void_p, _c.c_int64,
                               _c.c_void_p, _c.c_int64, _c.c_int32, _c.c_void_p]),
    "opc_coo_scatter": (_c.c_int, [_c.c_int32, _c.c_void_p, _c.c_void_p, _c.c_void_p, _c.c_void_p, _c.c_int64,
                                  _c.c_void_p]),
    "opc_take_device_error": (_c.c_int, [_c.c_int32, _c.POINTER(_c.c_int32)]),
}

_lib: Optional[ctypes.CDLL] = None


def library_path() -> Path:
    return Path(os.environ.get("OPC_B200_LIB", str(LIB_PATH)))


def load() -> ctypes.CDLL:
    """Load ``libopc_b200.so`` (idempotent).  Raises if it is missing: there is no fallback."""
    global _lib
    if _lib is not None:
        return _lib
    path = library_path()
    if not path.exists():
        raise RuntimeError(
            f"{path} not found: build it with `python -c 'import __graft_entry__ as g; g.build()'` "
            "(the CUDA library is required; there is no CPU fallback)"
        )
    lib = ctypes.CDLL(str(path))
    for name, (restype, argtypes) in PROTOTYPES.items():
        fn = getattr(lib, name)
        fn.restype = restype
        fn.argtypes = argtypes
    _lib = lib
    return lib


def last_error() -> str:
    return load().opc_last_error().decode("utf-8", "replace")


def check(rc: int) -> int:
    """Raise OpcError for a negative status, return it otherwise."""
    if rc < 0:
        raise OpcError(rc, last_error())
    return rc


def version() -> str:
    return load().opc_version().decode()

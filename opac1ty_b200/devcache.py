"""Device-format cache of repacked layers, keyed by the .bf2 file's content.

Putting a .bf2 model on the GPU repacks every layer (``opc_repack_layer``: index units, integer
and fp16 codebooks, tile masks, outlier rows; for element-wise outliers also the row-compressed
entries).  This module saves those device buffers, with each layer's plan, in one ``.npz`` file
and copies them back to the GPU on a later load instead of repacking.  The file name holds the
key: the XXH64 of the whole .bf2 file (the reference's header promises such a checksum,
opacc1ty/format/header.py:26), its size, the library version and the plan structure's size, so a
cache written for another file or by another build of the library is never read.  The buffers
are not interpreted on the host: they go back to the device as they were read from it, after a
check that every size matches the plan the current library computes for the layer's shape.
"""

from __future__ import annotations

import ctypes
import json
import mmap
import os
import zipfile
from pathlib import Path
from typing import Dict, Optional

import numpy as np
import torch

from . import _lib
from . import layer as L
from .format import BF2Reader
from .format.bf2 import xxh64

CACHE_VERSION = 1
_BUFFERS = ("units", "codebooks", "tile_mask", "outlier_rows")
_COO = ("row_ptr", "cols", "values", "delta")


class CacheMismatch(ValueError):
    """The cache file was written for another library build or does not match its plans."""


def _build_tag() -> str:
    return f"v{CACHE_VERSION}-p{ctypes.sizeof(_lib.LayerPlan)}-{_lib.version()}"


def bf2_key(path) -> str:
    """Cache key of a .bf2 file: XXH64 of its bytes, its size and the library build."""
    p = Path(path)
    size = p.stat().st_size
    with open(p, "rb") as f, mmap.mmap(f.fileno(), 0, access=mmap.ACCESS_READ) as mm:
        h = xxh64(memoryview(mm))
    tag = "".join(c if c.isalnum() or c in "-." else "_" for c in _build_tag())
    return f"{h:016x}-{size:x}-{tag}"


def save_layers(layers: Dict[str, L.DeviceLayer], path) -> None:
    """Write the layers' plans and device buffers to ``path`` (atomically: a temporary file
    renamed into place)."""
    arrays = {"build": np.array(_build_tag()), "names": np.array(json.dumps(list(layers)))}
    for i, dl in enumerate(layers.values()):
        p = f"l{i}_"
        arrays[p + "plan"] = np.frombuffer(bytes(dl.plan), dtype=np.uint8).copy()
        for k in _BUFFERS:
            arrays[p + k] = getattr(dl, k).cpu().numpy()
        if dl.coo is not None:
            for k in _COO:
                arrays[p + "coo_" + k] = getattr(dl.coo, k).cpu().numpy()
    path = Path(path)
    tmp = path.with_name(path.name + f".tmp{os.getpid()}")
    with open(tmp, "wb") as f:
        np.savez(f, **arrays)
    os.replace(tmp, path)


def _check_sizes(name: str, plan: _lib.LayerPlan, bufs: Dict[str, np.ndarray]) -> None:
    fresh = L.plan_layer(plan.M, plan.K, plan.n_outliers, plan.sub_vector_size)
    if bytes(fresh) != bytes(plan):
        raise CacheMismatch(f"{name}: cached plan differs from the library's plan for its shape")
    want = {"units": plan.units_bytes, "codebooks": plan.codebook_bytes, "tile_mask": plan.tile_mask_bytes,
            "outlier_rows": plan.outlier_rows_bytes}
    for k, nbytes in want.items():
        if bufs[k].nbytes != nbytes:
            raise CacheMismatch(f"{name}: cached {k} holds {bufs[k].nbytes} bytes, the plan {nbytes}")


def load_layers(path, device) -> Dict[str, L.DeviceLayer]:
    """The layers saved by ``save_layers``, copied to ``device``."""
    device = torch.device(device)
    out: Dict[str, L.DeviceLayer] = {}
    with np.load(path, allow_pickle=False) as z:
        if str(z["build"]) != _build_tag():
            raise CacheMismatch(f"cache written by build {str(z['build'])!r}, this is {_build_tag()!r}")
        names = json.loads(str(z["names"]))
        for i, name in enumerate(names):
            p = f"l{i}_"
            plan = _lib.LayerPlan.from_buffer_copy(z[p + "plan"].tobytes())
            bufs = {k: z[p + k] for k in _BUFFERS}
            _check_sizes(name, plan, bufs)
            t = {k: torch.from_numpy(np.ascontiguousarray(v)).to(device) for k, v in bufs.items()}
            coo = None
            if p + "coo_row_ptr" in z.files:
                c = {k: torch.from_numpy(np.ascontiguousarray(z[p + "coo_" + k])).to(device) for k in _COO}
                if c["row_ptr"].numel() != plan.M + 1:
                    raise CacheMismatch(f"{name}: cached row_ptr does not have M + 1 entries")
                coo = L.CooPart(c["row_ptr"], c["cols"], c["values"], c["delta"])
            out[name] = L.DeviceLayer(plan, t["units"], t["codebooks"], t["tile_mask"], t["outlier_rows"], device,
                                      name, coo)
    return out


def load_bf2_layers(path, device=None, cache_dir: Optional[str] = None) -> Dict[str, L.DeviceLayer]:
    """Every layer of a .bf2 file that runs on the GPU path ("quantized" and "sparse_outlier"),
    repacked onto ``device``.  With ``cache_dir``, a cache file for this exact file and library
    build is used when present (and written when not); a cache that fails its checks is ignored
    and rewritten."""
    device = L._as_cuda_device(device)
    cache = Path(cache_dir) / f"{bf2_key(path)}.npz" if cache_dir else None
    if cache is not None and cache.exists():
        try:
            return load_layers(cache, device)
        except (CacheMismatch, KeyError, ValueError, OSError, EOFError, zipfile.BadZipFile):
            pass  # unreadable or foreign: repack and rewrite it
    layers: Dict[str, L.DeviceLayer] = {}
    with BF2Reader(str(path)) as r:
        for name in r.layer_names():
            ly = r.load_layer(name)
            if ly["type"] in ("quantized", "sparse_outlier"):
                layers[name] = L.prepare_layer(ly, device, name)
    if cache is not None:
        cache.parent.mkdir(parents=True, exist_ok=True)
        save_layers(layers, cache)
    return layers

"""Device-resident repacked layers and the calls that run on them.

A ``DeviceLayer`` is one quantized layer from the reference's layer dictionaries
(``VectorQuantizer.quantize_layer``, opacc1ty/quantize/vq.py:191-200, or
``BF2Reader.load_layer``, opacc1ty/format/bf2.py:266-285) repacked once into the streamed
device layout of ``include/opc_b200.h``.  PyTorch only supplies device memory and the current
stream; every computation is a call into ``libopc_b200.so``.
"""

from __future__ import annotations

import ctypes
import threading
from dataclasses import dataclass
from typing import Dict, Optional, Tuple

import numpy as np
import torch

from . import _lib


def _stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _as_cuda_device(device) -> torch.device:
    if device is None:
        if not torch.cuda.is_available():
            raise RuntimeError("opac1ty_b200 needs a CUDA device (no CPU fallback)")
        return torch.device("cuda", torch.cuda.current_device())
    device = torch.device(device)
    if device.type != "cuda":
        raise RuntimeError(f"opac1ty_b200 runs on CUDA devices only, got {device}")
    if device.index is None:
        device = torch.device("cuda", torch.cuda.current_device())
    return device


def plan_layer(M: int, K: int, n_outliers: int, sub_vector_size: int = 1) -> _lib.LayerPlan:
    """Device geometry of an M x K layer (``opc_plan_layer``)."""
    lib = _lib.load()
    plan = _lib.LayerPlan()
    _lib.check(lib.opc_plan_layer(int(M), int(K), int(n_outliers), int(sub_vector_size), ctypes.byref(plan)))
    return plan


def algorithmic_bytes(M: int, K: int, n_outliers: int, batch: int = 1, sub_vector_size: int = 1) -> int:
    """Bytes a fused GEMV must move at least: 2-bit indices (one per sub-vector), fp16 codebooks
    (4 vectors of sub_vector_size per row), fp16 outlier rows with int32 ids, x in and y out (fp16)."""
    svs = int(sub_vector_size)
    return (M * (K // svs) // 4 + 8 * svs * M + n_outliers * (2 * K + 4) + 2 * K * batch + 2 * M * batch)


@dataclass
class CooPart:
    """Element-wise outliers of a "sparse_outlier" layer in row-compressed form (``opc_coo_build``):
    row_ptr [M+1] int32, then per unique position in (row, col) order cols int32, values fp16 and
    delta fp32 (value minus the codebook value there), all on the layer's device."""

    row_ptr: torch.Tensor
    cols: torch.Tensor
    values: torch.Tensor
    delta: torch.Tensor

    @property
    def nnz(self) -> int:
        return int(self.cols.numel())

    def apply_gemv(self, M: int, x2: torch.Tensor, y2: torch.Tensor, batch: int, stream: int):
        """y += delta . x per row (``opc_coo_gemv``), after the codebook part."""
        if self.nnz == 0:
            return
        _lib.check(_lib.load().opc_coo_gemv(int(M), self.row_ptr.data_ptr(), self.cols.data_ptr(), self.delta.data_ptr(),
                                            x2.data_ptr(), x2.stride(0), y2.data_ptr(), y2.stride(0), int(batch), stream))

    def apply_dequant(self, M: int, w: torch.Tensor, stream: int):
        if self.nnz == 0:
            return
        _lib.check(_lib.load().opc_coo_scatter(int(M), self.row_ptr.data_ptr(), self.cols.data_ptr(),
                                               self.values.data_ptr(), w.data_ptr(), w.stride(0), stream))


@dataclass
class DeviceLayer:
    """A quantized layer repacked for the sm_100a kernels, resident on ``device``."""

    plan: _lib.LayerPlan
    units: torch.Tensor
    codebooks: torch.Tensor
    tile_mask: torch.Tensor
    outlier_rows: torch.Tensor
    device: torch.device
    name: Optional[str] = None
    coo: Optional[CooPart] = None   # element-wise outliers ("sparse_outlier" layers)

    def __post_init__(self):
        self.c_layer = _lib.Layer(
            plan=self.plan,
            units=self.units.data_ptr(),
            codebooks=self.codebooks.data_ptr(),
            tile_mask=self.tile_mask.data_ptr(),
            outlier_rows=self.outlier_rows.data_ptr(),
        )

    @property
    def M(self) -> int:
        return self.plan.M

    @property
    def K(self) -> int:
        return self.plan.K

    @property
    def shape(self) -> Tuple[int, int]:
        return (self.plan.M, self.plan.K)

    @property
    def n_outliers(self) -> int:
        return self.plan.n_outliers

    @property
    def sub_vector_size(self) -> int:
        return self.plan.sub_vector_size

    def algorithmic_bytes(self, batch: int = 1) -> int:
        b = algorithmic_bytes(self.M, self.K, self.n_outliers, batch, self.plan.sub_vector_size)
        if self.coo is not None:  # CSR entries (col + delta) and the epilogue's pass over y
            b += 8 * self.coo.nnz + 4 * (self.M + 1) + 4 * self.M * batch
        return b

    def device_bytes(self) -> int:
        ts = [self.units, self.codebooks, self.tile_mask, self.outlier_rows]
        if self.coo is not None:
            ts += [self.coo.row_ptr, self.coo.cols, self.coo.values, self.coo.delta]
        return sum(t.numel() * t.element_size() for t in ts)


def _to_device_contig(t, dtype, device) -> torch.Tensor:
    if isinstance(t, np.ndarray):
        t = torch.from_numpy(np.ascontiguousarray(t))
    return t.to(device=device, dtype=dtype).contiguous()


def prepare_layer(layer: dict, device=None, name: Optional[str] = None) -> DeviceLayer:
    """Repack a reference layer dict (type "quantized") onto ``device``.

    Accepted keys follow ``VectorQuantizer.quantize_layer`` (opacc1ty/quantize/vq.py:191-200):
    ``shape`` (out_features, in_features), ``codebooks`` [M][4][svs] fp16, ``indices``
    [M][K/svs] uint8, optional ``outlier_values`` [n][K] fp16 and ``outlier_indices`` [n]
    (int32 or int64).
    """
    if layer.get("type") == "sparse_outlier":
        return _prepare_sparse(layer, device, name)
    if layer.get("type") != "quantized":
        raise ValueError(f"prepare_layer: only quantized layers run on the GPU path, got {layer.get('type')!r}")
    device = _as_cuda_device(device)
    out_f, in_f = (int(v) for v in layer["shape"])
    cb = layer["codebooks"]
    idx = layer["indices"]
    svs = int(cb.shape[2]) if cb.dim() == 3 else 1
    if svs not in (1, 8):
        raise _lib.OpcError(_lib.OPC_ERR_UNSUPPORTED, f"sub_vector_size={svs}: 1 and 8 are implemented on the GPU path")
    if svs == 8 and in_f % 8:
        raise _lib.OpcError(_lib.OPC_ERR_UNSUPPORTED, f"in_features={in_f} is not a multiple of sub_vector_size 8")
    if tuple(cb.shape[:2]) != (out_f, 4):
        raise ValueError(f"codebooks shape {tuple(cb.shape)} does not match ({out_f}, 4, {svs})")
    if tuple(idx.shape) != (out_f, in_f // svs):
        raise ValueError(f"indices shape {tuple(idx.shape)} does not match ({out_f}, {in_f // svs})")
    ov = layer.get("outlier_values")
    oi = layer.get("outlier_indices")
    if ov is None or oi is None or len(oi) == 0:
        ov, oi = None, None
        ids = np.zeros(0, dtype=np.int64)
    else:
        ids = np.ascontiguousarray(np.asarray(oi.cpu() if isinstance(oi, torch.Tensor) else oi, dtype=np.int64))
        if tuple(ov.shape) != (len(ids), in_f):
            raise ValueError(f"outlier_values shape {tuple(ov.shape)} does not match ({len(ids)}, {in_f})")

    lib = _lib.load()
    ids_ptr = ids.ctypes.data_as(ctypes.POINTER(ctypes.c_int64))
    n_distinct = int(lib.opc_count_distinct_ids(ids_ptr, len(ids)))
    plan = plan_layer(out_f, in_f, n_distinct, svs)
    with torch.cuda.device(device):
        units = torch.empty(plan.units_bytes, dtype=torch.uint8, device=device)
        codebooks = torch.empty(plan.codebook_bytes, dtype=torch.uint8, device=device)
        tile_mask = torch.empty(plan.tile_mask_bytes // 2, dtype=torch.int16, device=device)
        outlier_rows = torch.empty(plan.outlier_rows_bytes // 4, dtype=torch.int32, device=device)
        dl = DeviceLayer(plan, units, codebooks, tile_mask, outlier_rows, device, name)
        cb_d = _to_device_contig(cb, torch.float16, device)
        idx_d = _to_device_contig(idx, torch.uint8, device)
        ov_d = _to_device_contig(ov, torch.float16, device) if ov is not None else None
        _lib.check(
            lib.opc_repack_layer(
                ctypes.byref(dl.c_layer),
                cb_d.data_ptr(),
                idx_d.data_ptr(),
                ov_d.data_ptr() if ov_d is not None else None,
                ids_ptr if len(ids) else None,
                len(ids),
                _stream_ptr(device),
            )
        )
    return dl


def _prepare_sparse(layer: dict, device, name: Optional[str]) -> DeviceLayer:
    """A "sparse_outlier" layer: the codebook part repacked without outlier rows, the entries
    ("outlier_values" [nnz] fp16 at "outlier_indices" [nnz][2] (row, col)) row-compressed."""
    out_f, in_f = (int(v) for v in layer["shape"])
    base = {"type": "quantized", "shape": (out_f, in_f), "codebooks": layer["codebooks"], "indices": layer["indices"]}
    dl = prepare_layer(base, device, name)
    cb = np.ascontiguousarray(np.asarray(_cpu(layer["codebooks"]), dtype=np.float16))
    idx = np.ascontiguousarray(np.asarray(_cpu(layer["indices"]), dtype=np.uint8))
    ov, oi = layer.get("outlier_values"), layer.get("outlier_indices")
    coo = np.zeros((0, 2), dtype=np.int64) if oi is None else np.ascontiguousarray(
        np.asarray(_cpu(oi), dtype=np.int64).reshape(-1, 2))
    vals = np.zeros(0, dtype=np.float16) if ov is None else np.ascontiguousarray(
        np.asarray(_cpu(ov), dtype=np.float16).reshape(-1))
    if len(vals) != len(coo):
        raise ValueError(f"sparse_outlier: {len(vals)} values for {len(coo)} positions")
    svs = int(cb.shape[2]) if cb.ndim == 3 else 1
    lib = _lib.load()
    M = out_f
    row_ptr = np.zeros(M + 1, dtype=np.int32)
    n = len(coo)
    cols = np.zeros(max(n, 1), dtype=np.int32)
    vout = np.zeros(max(n, 1), dtype=np.float16)
    delta = np.zeros(max(n, 1), dtype=np.float32)
    nnz = ctypes.c_int64(0)
    p = lambda a: a.ctypes.data_as(ctypes.c_void_p)
    _lib.check(lib.opc_coo_build(M, in_f, svs, p(cb), p(idx), p(coo) if n else None, p(vals) if n else None, n,
                                 p(row_ptr), p(cols), p(vout), p(delta), ctypes.byref(nnz)))
    k = int(nnz.value)
    dev = dl.device
    dl.coo = CooPart(torch.from_numpy(row_ptr).to(dev), torch.from_numpy(cols[:k].copy()).to(dev),
                     torch.from_numpy(vout[:k].copy()).to(dev), torch.from_numpy(delta[:k].copy()).to(dev))
    return dl


def _cpu(t):
    return t.detach().cpu().numpy() if isinstance(t, torch.Tensor) else t


def dequantize(dl: DeviceLayer, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """W_hat [M][K] fp16 on the layer's device (``opc_dequant``), into ``out`` if given."""
    lib = _lib.load()
    with torch.cuda.device(dl.device):
        w = torch.empty(dl.M, dl.K, dtype=torch.float16, device=dl.device) if out is None else out
        if tuple(w.shape) != (dl.M, dl.K) or w.dtype != torch.float16 or w.stride(1) != 1:
            raise ValueError(f"dequantize: out must be float16 [{dl.M}, {dl.K}] with unit stride")
        _lib.check(lib.opc_dequant(ctypes.byref(dl.c_layer), w.data_ptr(), w.stride(0), _stream_ptr(dl.device)))
        if dl.coo is not None:
            dl.coo.apply_dequant(dl.M, w, _stream_ptr(dl.device))
    return w


class Workspace:
    """Zero-initialised GEMV workspace for one (device, stream).  opc_gemv leaves it zeroed, so
    it is cleared only when it grows."""

    def __init__(self, device: torch.device):
        self.device = device
        self.buf: Optional[torch.Tensor] = None

    def get(self, nbytes: int) -> torch.Tensor:
        if self.buf is None or self.buf.numel() < nbytes:
            size = max(nbytes, 1 << 20)
            self.buf = torch.zeros(size, dtype=torch.uint8, device=self.device)
        return self.buf


_ws_lock = threading.Lock()
_workspaces: Dict[Tuple[int, int], Workspace] = {}


def workspace_for(device: torch.device, stream: int) -> Workspace:
    key = (device.index, stream)
    with _ws_lock:
        ws = _workspaces.get(key)
        if ws is None:
            ws = _workspaces[key] = Workspace(device)
        return ws


def workspace_bytes(dl: DeviceLayer, batch: int) -> int:
    lib = _lib.load()
    return int(lib.opc_gemv_workspace_bytes(ctypes.byref(dl.plan), int(batch), dl.device.index))


def gemv(dl: DeviceLayer, x: torch.Tensor, out: Optional[torch.Tensor] = None,
         workspace: Optional[torch.Tensor] = None) -> torch.Tensor:
    """y = x @ W_hat^T for x of shape [K] or [B, K] (fp16, CUDA, unit stride along K)."""
    squeeze = x.dim() == 1
    x2 = x.unsqueeze(0) if squeeze else x
    if x2.dim() != 2 or x2.shape[1] != dl.K:
        raise ValueError(f"gemv: x shape {tuple(x.shape)} incompatible with K={dl.K}")
    if x2.dtype != torch.float16 or x2.device != dl.device:
        raise ValueError(f"gemv: x must be float16 on {dl.device}, got {x2.dtype} on {x2.device}")
    if x2.stride(1) != 1:
        x2 = x2.contiguous()
    batch = x2.shape[0]
    if out is None:
        out = torch.empty(batch, dl.M, dtype=torch.float16, device=dl.device)
    y2 = out.unsqueeze(0) if out.dim() == 1 else out
    if tuple(y2.shape) != (batch, dl.M) or y2.stride(1) != 1 or y2.dtype != torch.float16:
        raise ValueError(f"gemv: out must be float16 [{batch}, {dl.M}] with unit stride")
    lib = _lib.load()
    stream = _stream_ptr(dl.device)
    need = workspace_bytes(dl, batch)
    if workspace is None:
        workspace = workspace_for(dl.device, stream).get(need)
    _lib.check(
        lib.opc_gemv(ctypes.byref(dl.c_layer), x2.data_ptr(), x2.stride(0), y2.data_ptr(), y2.stride(0), batch,
                     workspace.data_ptr(), workspace.numel() * workspace.element_size(), stream)
    )
    if dl.coo is not None:
        dl.coo.apply_gemv(dl.M, x2, y2, batch, stream)
    return out.squeeze(0) if squeeze and out.dim() == 2 else out


def gemv_noalloc(dl: DeviceLayer, x: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """y = x @ W_hat^T through ``opc_gemv_noalloc``: no workspace, the library's built-in scratch
    (batch <= 8).  For callers that must not allocate device memory; ``out`` should then be
    passed in.  Calls that may overlap on the GPU share the scratch and must be serialised."""
    squeeze = x.dim() == 1
    x2 = x.unsqueeze(0) if squeeze else x
    if x2.dim() != 2 or x2.shape[1] != dl.K or x2.dtype != torch.float16 or x2.stride(1) != 1:
        raise ValueError(f"gemv_noalloc: x must be float16 [B, {dl.K}] with unit stride")
    if out is None:
        out = torch.empty(x2.shape[0], dl.M, dtype=torch.float16, device=dl.device)
    y2 = out.unsqueeze(0) if out.dim() == 1 else out
    _lib.check(_lib.load().opc_gemv_noalloc(ctypes.byref(dl.c_layer), x2.data_ptr(), x2.stride(0), y2.data_ptr(),
                                            y2.stride(0), x2.shape[0], _stream_ptr(dl.device)))
    if dl.coo is not None:
        dl.coo.apply_gemv(dl.M, x2, y2, x2.shape[0], _stream_ptr(dl.device))
    return out

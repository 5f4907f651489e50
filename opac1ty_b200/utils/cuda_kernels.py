"""CUDA kernel manager: the drop-in for opacc1ty's MetalKernelManager.

Same surface as opacc1ty/utils/metal_utils.py:79-310 -- ``compile_kernels()``,
``load_library()``, ``dequant_gemv(codebooks_buf, indices_buf, input_buf, output_buf, M, K,
outlier_vals_buf=None, outlier_idx_buf=None, n_outliers=0)`` -- with CUDA tensors as the
"buffers".  Differences, each deliberate:

  * ``compile_kernels`` builds ``libopc_b200.so`` for sm_100a with nvcc (in-tree) instead of
    xcrun metal/metallib; ``load_library`` loads it (idempotent).
  * The raw .bf2 arrays are repacked once into the streamed device layout; ``dequant_gemv``
    caches the repacked layer per set of input buffers, so repeated calls on the same weights
    only launch the GEMV.  ``prepare_layer`` exposes the repacked layer directly.
  * ``dequant_gemv`` blocks until the result is ready, like the reference's
    ``waitUntilCompleted`` (metal_utils.py:288), unless ``blocking=False``; the stream-ordered
    call is ``opac1ty_b200.gemv``.
  * ``dequant_gemm`` exists (the reference loads the GEMM pipeline but never dispatches it,
    metal_utils.py:188-196).
Errors raise ``OpcError`` (a RuntimeError) carrying the C library's message.
"""

from __future__ import annotations

import ctypes
import weakref
from dataclasses import dataclass
from pathlib import Path
from typing import Optional

import torch

from .. import _lib
from .. import layer as L


@dataclass
class GPUInfo:
    """Device capabilities; the reference's GPUInfo fields (metal_utils.py:24-36) filled with
    their CUDA equivalents, plus CUDA-specific fields."""

    name: str
    max_threads_per_threadgroup: int
    max_total_threads_per_threadgroup: int
    threadgroup_memory_size: int
    max_buffer_size: int
    supports_family_apple8: bool
    supports_family_apple7: bool
    supports_family_apple6: bool
    unified_memory_gb: float
    gpu_cores: int
    sm_count: int = 0
    compute_capability: tuple = (0, 0)
    l2_bytes: int = 0


def get_cuda_device_info(device: int = 0) -> Optional[GPUInfo]:
    """Capabilities of CUDA device ``device``, or None when no CUDA device is present."""
    if not torch.cuda.is_available():
        return None
    lib = _lib.load()
    p = _lib.DeviceProps()
    if lib.opc_device_info(int(device), ctypes.byref(p)) != _lib.OPC_OK:
        return None
    return GPUInfo(
        name=p.name.decode(), max_threads_per_threadgroup=p.max_threads_per_block,
        max_total_threads_per_threadgroup=p.max_threads_per_block, threadgroup_memory_size=p.max_smem_per_block_optin,
        max_buffer_size=p.total_mem_bytes, supports_family_apple8=False, supports_family_apple7=False,
        supports_family_apple6=False, unified_memory_gb=p.total_mem_bytes / 1e9, gpu_cores=p.sm_count,
        sm_count=p.sm_count, compute_capability=(p.cc_major, p.cc_minor), l2_bytes=p.l2_bytes)


def get_metal_device_info() -> None:
    """Metal is not available on this platform (kept so reference imports resolve)."""
    return None


def _key(t) -> tuple:
    if t is None:
        return (None,)
    if isinstance(t, torch.Tensor):
        return (t.data_ptr(), tuple(t.shape), t.dtype, t.device, t._version)
    return (id(t),)


class CudaKernelManager:
    """Loads libopc_b200.so and dispatches the fused dequant kernels on CUDA tensors."""

    def __init__(self, device=None):
        self.library_path: Optional[Path] = None
        self.device = L._as_cuda_device(device) if device is not None or torch.cuda.is_available() else None
        self._lib = None
        self._cache: "dict[tuple, L.DeviceLayer]" = {}

    def compile_kernels(self) -> Path:
        """Build libopc_b200.so for sm_100a (no-op when up to date); returns its path."""
        from ..build import build_library

        self.library_path = build_library()
        return self.library_path

    def load_library(self):
        """Load the CUDA library (after compile_kernels; builds it if missing)."""
        if not _lib.library_path().exists():
            self.compile_kernels()
        self._lib = _lib.load()
        self.library_path = _lib.library_path()
        return self._lib

    def _ensure(self):
        if self._lib is None:
            self.load_library()
        if self.device is None:
            self.device = L._as_cuda_device(None)

    def prepare_layer(self, layer: dict, name: Optional[str] = None) -> L.DeviceLayer:
        """Repack a reference layer dict for the GPU (one-time cost per layer)."""
        self._ensure()
        return L.prepare_layer(layer, self.device, name)

    def _layer_from_buffers(self, codebooks_buf, indices_buf, M, K, outlier_vals_buf, outlier_idx_buf,
                            n_outliers) -> L.DeviceLayer:
        key = (_key(codebooks_buf), _key(indices_buf), _key(outlier_vals_buf), _key(outlier_idx_buf), int(M),
               int(K), int(n_outliers))
        dl = self._cache.get(key)
        if dl is None:
            cb = torch.as_tensor(codebooks_buf)
            svs = int(cb.numel() // (int(M) * 4)) if cb.dim() != 3 else int(cb.shape[2])
            cb = cb.reshape(int(M), 4, svs)
            idx = torch.as_tensor(indices_buf).reshape(int(M), int(K) // svs)
            layer = {"type": "quantized", "shape": (int(M), int(K)), "codebooks": cb, "indices": idx}
            if outlier_vals_buf is not None and outlier_idx_buf is not None and n_outliers > 0:
                layer["outlier_values"] = torch.as_tensor(outlier_vals_buf).reshape(-1, int(K))[: int(n_outliers)]
                layer["outlier_indices"] = torch.as_tensor(outlier_idx_buf).reshape(-1)[: int(n_outliers)]
            dl = L.prepare_layer(layer, self.device)
            if len(self._cache) > 64:
                self._cache.clear()
            self._cache[key] = dl
        return dl

    def dequant_gemv(self, codebooks_buf, indices_buf, input_buf, output_buf, M: int, K: int,
                     outlier_vals_buf=None, outlier_idx_buf=None, n_outliers: int = 0, blocking: bool = True):
        """output = W_hat . input for the layer described by the buffers (or a DeviceLayer passed
        as ``codebooks_buf``).  input_buf: fp16 [K] or [B, K]; output_buf: fp16 [M] or [B, M]."""
        self._ensure()
        if isinstance(codebooks_buf, L.DeviceLayer):
            dl = codebooks_buf
            if (dl.M, dl.K) != (int(M), int(K)):
                raise ValueError(f"dequant_gemv: layer is {dl.shape}, called with M={M}, K={K}")
        else:
            dl = self._layer_from_buffers(codebooks_buf, indices_buf, M, K, outlier_vals_buf, outlier_idx_buf,
                                          n_outliers)
        L.gemv(dl, input_buf, out=output_buf)
        if blocking:
            torch.cuda.current_stream(dl.device).synchronize()
        return output_buf

    def dequant_gemm(self, layer, x: torch.Tensor, out: Optional[torch.Tensor] = None,
                     blocking: bool = True) -> torch.Tensor:
        """Prefill: out [N, M] = x [N, K] . W_hat^T for a DeviceLayer or layer dict."""
        self._ensure()
        dl = layer if isinstance(layer, L.DeviceLayer) else self.prepare_layer(layer)
        from .. import gemm

        y = gemm.gemm(dl, x, out=out)
        if blocking:
            torch.cuda.current_stream(dl.device).synchronize()
        return y

    def dequantize(self, layer) -> torch.Tensor:
        """W_hat [M][K] fp16 on the device (bit-exact dequantize_layer)."""
        self._ensure()
        dl = layer if isinstance(layer, L.DeviceLayer) else self.prepare_layer(layer)
        return L.dequantize(dl)


class MetalKernelManager:
    """The reference's Metal manager has no backend on this platform; constructing it raises.
    Use CudaKernelManager (same methods)."""

    def __init__(self, device=None):
        raise RuntimeError("Metal is unavailable on this platform (no Apple GPU); use CudaKernelManager")

"""Prefill GEMM: y [N, M] = x [N, K] . W_hat^T on the tcgen05 tensor cores (``opc_gemm``).

Replaces the reference's ``dequant_gemm_2bit`` pipeline (kernels/dequant_gemm.metal:34-149).
The CUDA library reads x with TMA, which needs rows 16-byte aligned with a stride that is a
multiple of 8 elements; other layouts are copied once into such a buffer.  Every computation is
a call into ``libopc_b200.so``.
"""

from __future__ import annotations

import ctypes
from typing import Optional

import torch

from . import _lib
from . import layer as L


def flops(dl: L.DeviceLayer, n_tok: int) -> int:
    """Dense-equivalent flops of one GEMM (2 * tokens * M * K)."""
    return 2 * n_tok * dl.M * dl.K


def gemm(dl: L.DeviceLayer, x: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """y = x @ W_hat^T for x [N, K] fp16 on the layer's device."""
    if x.dim() != 2 or x.shape[1] != dl.K:
        raise ValueError(f"gemm: x shape {tuple(x.shape)} incompatible with K={dl.K}")
    if x.dtype != torch.float16 or x.device != dl.device:
        raise ValueError(f"gemm: x must be float16 on {dl.device}, got {x.dtype} on {x.device}")
    n = x.shape[0]
    if x.stride(1) != 1 or x.stride(0) % 8 != 0 or x.data_ptr() % 16 != 0:
        ld = -(-dl.K // 8) * 8
        xp = torch.zeros(n, ld, dtype=torch.float16, device=dl.device)
        xp[:, : dl.K] = x
        x = xp
    if out is None:
        out = torch.empty(n, dl.M, dtype=torch.float16, device=dl.device)
    if tuple(out.shape) != (n, dl.M) or out.stride(1) != 1 or out.dtype != torch.float16:
        raise ValueError(f"gemm: out must be float16 [{n}, {dl.M}] with unit stride")
    lib = _lib.load()
    stream = torch.cuda.current_stream(dl.device).cuda_stream
    _lib.check(lib.opc_gemm(ctypes.byref(dl.c_layer), x.data_ptr(), x.stride(0), out.data_ptr(), out.stride(0), n,
                            stream))
    if dl.coo is not None:  # element-wise outliers: the CSR epilogue (opc_coo_gemv)
        dl.coo.apply_gemv(dl.M, x, out, n, stream)
    return out

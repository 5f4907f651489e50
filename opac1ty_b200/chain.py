"""Decode chain on one persistent kernel (``opc_chain_*``).

A chain is a fixed list of dependent GEMV steps (layer, x, y) whose step j >= 1 reads a prefix of
step j-1's output.  ``opc_chain_launch`` runs all of them in one cooperative kernel: a producer
warp per SM streams the weights of every step without waiting for activations, and each step's
outputs are published as tagged 32-bit words that the next step's readers poll (no grid barrier
between steps).  Results equal per-step ``opac1ty_b200.gemv`` calls bit for bit (batch 1..2).
At batch 1 the dataflow form exchanges fixed-point digits per 128-column block instead (no
barrier or per-CTA conversion between steps; see ``Chain``).
"""

from __future__ import annotations

import ctypes
from typing import List, Sequence, Tuple

import torch

from . import _lib
from . import layer as L


# stamps per step and CTA in a trace buffer: 8 phase stamps, then one per consumer warp
TRACE_SLOTS = 24
FORMS = {"auto": _lib.OPC_CHAIN_FORM_AUTO, "barrier": _lib.OPC_CHAIN_FORM_BARRIER,
         "dataflow": _lib.OPC_CHAIN_FORM_DATAFLOW}


class Chain:
    """Steps: (DeviceLayer, x tensor [B, >=K] fp16, y tensor [B, >=M] fp16), rows unit-stride.

    ``form``: "barrier" (each step's x staged from fp16 with its exponent from max|x|; results
    equal per-step ``gemv`` calls bit for bit; batch 1..2), "dataflow" (batch 1: steps exchange
    fixed-point digits at a scale fixed in advance from a norm bound, with no barrier between
    steps; results within the GEMV tolerance) or "auto" (the barrier form, measured faster)."""

    def __init__(self, steps: Sequence[Tuple[L.DeviceLayer, torch.Tensor, torch.Tensor]], form: str = "auto"):
        if form not in FORMS:
            raise ValueError(f"Chain: form must be one of {sorted(FORMS)}, got {form!r}")
        if not steps:
            raise ValueError("Chain: no steps")
        self.device = steps[0][0].device
        batch = steps[0][1].shape[0]
        arr = (_lib.ChainStep * len(steps))()
        self._keep: List[object] = []
        for i, (dl, x, y) in enumerate(steps):
            if x.dtype != torch.float16 or y.dtype != torch.float16 or x.stride(-1) != 1 or y.stride(-1) != 1:
                raise ValueError(f"Chain: step {i}: x/y must be fp16 with unit stride")
            if x.shape[0] != batch or y.shape[0] != batch:
                raise ValueError(f"Chain: step {i}: batch mismatch")
            if dl.coo is not None:
                raise _lib.OpcError(_lib.OPC_ERR_UNSUPPORTED, f"Chain: step {i}: element-wise outliers run on "
                                    "gemv + the CSR epilogue, not in the chain kernel")
            arr[i].layer = ctypes.pointer(dl.c_layer)
            arr[i].x = x.data_ptr()
            arr[i].ldx = x.stride(0) if x.dim() == 2 else dl.K
            arr[i].y = y.data_ptr()
            arr[i].ldy = y.stride(0) if y.dim() == 2 else dl.M
            self._keep += [dl, x, y]
        self.batch = batch
        self.n_steps = len(steps)
        handle = ctypes.c_void_p()
        lib = _lib.load()
        with torch.cuda.device(self.device):
            _lib.check(lib.opc_chain_create_ex(arr, len(steps), batch, FORMS[form], ctypes.byref(handle)))
        self._handle = handle
        self._steps = arr
        self.form = "dataflow" if lib.opc_chain_form(handle) == _lib.OPC_CHAIN_FORM_DATAFLOW else "barrier"

    def launch(self):
        lib = _lib.load()
        stream = torch.cuda.current_stream(self.device).cuda_stream
        _lib.check(lib.opc_chain_launch(self._handle, stream))

    def enable_trace(self) -> torch.Tensor:
        """Record per-step, per-CTA phase stamps on every launch; returns the [steps, grid, 24]
        int64 buffer (ns of %globaltimer, see opc_chain_set_trace in include/opc_b200.h)."""
        lib = _lib.load()
        n = int(lib.opc_chain_trace_bytes(self._handle)) // 8
        grid = int(lib.opc_chain_grid(self._handle))
        self._trace = torch.zeros(self.n_steps, grid, TRACE_SLOTS, dtype=torch.int64, device=self.device)
        assert self._trace.numel() == n
        _lib.check(lib.opc_chain_set_trace(self._handle, self._trace.data_ptr()))
        return self._trace

    def disable_trace(self):
        _lib.check(_lib.load().opc_chain_set_trace(self._handle, None))
        self._trace = None

    def set_l2_prefetch(self, on: bool):
        _lib.check(_lib.load().opc_chain_set_option(self._handle, _lib.OPC_CHAIN_L2_PREFETCH, int(bool(on))))

    def close(self):
        if getattr(self, "_handle", None) and self._handle.value:
            with torch.cuda.device(self.device):
                _lib.load().opc_chain_destroy(self._handle)
            self._handle = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

"""The allocation-free GEMV entry point (opc_gemv_noalloc), called through the C ABI.

It serves callers that cannot allocate device memory (plugin hosts that pass only preallocated
input/output buffers, serving processes whose device memory is owned by their own pool): the
GEMV's scratch comes from a fixed array inside the library instead of a workspace.  Its output
must match the workspace entry point (opc_gemv) within the GEMV tolerance, on two calls in a row
(the second call sees the scratch the first one left behind).  This file is collected last so a
run that stops at the first failure has already run every other test.
"""

import ctypes

import numpy as np
import pytest
import torch

from oracle import oracle
from opac1ty_b200 import _lib, layer as L, synthetic

pytestmark = pytest.mark.gpu

REL_TOL = 2e-3  # the GEMV tolerance used by every GPU parity test


def _call_noalloc(dl, x, y):
    lib = _lib.load()
    return lib.opc_gemv_noalloc(ctypes.byref(dl.c_layer), x.data_ptr(), x.stride(0), y.data_ptr(), y.stride(0),
                                x.shape[0], torch.cuda.current_stream(dl.device).cuda_stream)


@pytest.mark.parametrize("M,K,n_out,batch", [(1000, 2048, 9, 4), (14336, 4096, 143, 1)])
def test_noalloc_matches_workspace_gemv_twice(cuda_device, M, K, n_out, batch):
    layer = synthetic.random_layer(M, K, n_out, seed=M + K)
    dl = L.prepare_layer(layer, cuda_device)
    x = torch.from_numpy(synthetic.activations(batch, K, seed=batch)).to(cuda_device)
    y_ws = L.gemv(dl, x).cpu().numpy()  # existing entry point, caller workspace
    y64 = oracle.gemv_f64(oracle.dequantize_np(layer), x.cpu().numpy())
    for _ in range(2):
        y = torch.full((batch, M), float("nan"), dtype=torch.float16, device=cuda_device)
        _lib.check(_call_noalloc(dl, x, y))
        got = y.cpu().numpy()
        assert np.all(np.isfinite(got))
        assert oracle.rel_err(got, y_ws.astype(np.float64)) <= REL_TOL
        assert oracle.rel_err(got, y64) <= REL_TOL


@pytest.mark.parametrize("batch", [3, 8])
def test_noalloc_equals_workspace_gemv_bit_for_bit_at_batch_3_to_8(cuda_device, batch):
    # At batch 3..8 both entry points run the same fp16 GEMV kernel with a fixed summation order,
    # so the only difference is where the scratch lives: the results must be identical.
    M, K = 3000, 1536
    layer = synthetic.random_layer(M, K, 30, seed=batch, shuffle_ids=True)
    dl = L.prepare_layer(layer, cuda_device)
    x = torch.from_numpy(synthetic.activations(batch, K, seed=10 + batch)).to(cuda_device)
    y_ws = L.gemv(dl, x)
    for _ in range(2):
        y = torch.full((batch, M), float("nan"), dtype=torch.float16, device=cuda_device)
        _lib.check(_call_noalloc(dl, x, y))
        torch.cuda.synchronize()
        assert torch.equal(y, y_ws)


@pytest.mark.parametrize("batch", [1, 5])
def test_noalloc_svs8_layer_against_the_oracle(cuda_device, batch):
    # sub_vector_size 8 (the reference quantizer's default) needs no scratch; the entry point
    # must still run it and agree with the workspace call and with the fp64 oracle.
    M, K = 1000, 2048
    layer = synthetic.random_layer_vq8(M, K, 10, seed=77)
    dl = L.prepare_layer(layer, cuda_device)
    x = torch.from_numpy(synthetic.activations(batch, K, seed=3)).to(cuda_device)
    y64 = oracle.gemv_f64(oracle.dequantize_np(layer), x.cpu().numpy())
    y_ws = L.gemv(dl, x)
    for _ in range(2):
        y = torch.full((batch, M), float("nan"), dtype=torch.float16, device=cuda_device)
        _lib.check(_call_noalloc(dl, x, y))
        torch.cuda.synchronize()
        assert torch.equal(y, y_ws)
        assert oracle.rel_err(y.cpu().numpy(), y64) <= REL_TOL


def test_noalloc_rejects_requests_beyond_its_limits(cuda_device):
    layer = synthetic.random_layer(64, 128, 0, seed=1)
    dl = L.prepare_layer(layer, cuda_device)
    x = torch.zeros(9, 128, dtype=torch.float16, device=cuda_device)
    y = torch.zeros(9, 64, dtype=torch.float16, device=cuda_device)
    rc = _call_noalloc(dl, x, y)
    assert rc == _lib.OPC_ERR_INVALID and "batch 9" in _lib.last_error()
    # A plan larger than the static scratch is refused before anything is launched.
    big = _lib.Layer(plan=L.plan_layer(300000, 128, 0), units=dl.c_layer.units, codebooks=dl.c_layer.codebooks,
                     tile_mask=dl.c_layer.tile_mask, outlier_rows=dl.c_layer.outlier_rows)
    rc = _lib.load().opc_gemv_noalloc(ctypes.byref(big), x.data_ptr(), 128, y.data_ptr(), 300000, 1,
                                      torch.cuda.current_stream(cuda_device).cuda_stream)
    assert rc == _lib.OPC_ERR_INVALID and "static scratch limit" in _lib.last_error()

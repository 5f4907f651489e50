"""GPU parity of the fused dequant kernels against the CPU oracle, through the C ABI.

Bar (the path's stated tolerances):
  * dequantized weights: bit-exact against the oracle's dequantize_layer restatement;
  * GEMV / small-batch GEMM outputs: max |y - y64| / max |y64| <= 2e-3 against an fp64
    recompute of x . W_hat^T (REL_TOL below).
"""

import numpy as np
import pytest
import torch

from oracle import oracle
from opac1ty_b200 import _lib, layer as L, synthetic

pytestmark = pytest.mark.gpu

REL_TOL = 2e-3


def _dequant_check(layer, dev):
    dl = L.prepare_layer(layer, dev)
    w_gpu = L.dequantize(dl).cpu().numpy()
    w_ref = oracle.dequantize_np(layer)
    assert w_gpu.shape == w_ref.shape
    assert np.array_equal(w_gpu.view(np.uint16), w_ref.view(np.uint16)), "dequantized weights differ"
    return dl, w_ref


SHAPES = [
    # (M, K, n_outliers)
    (16, 128, 0),
    (48, 200, 3),      # K not a multiple of 16/128, M a multiple of 16
    (17, 37, 2),       # ragged M and K (K not a multiple of 4 or 8)
    (1, 1, 0),         # smallest layer
    (130, 1000, 17),   # more than one outlier tile
    (1024, 4096, 10),  # k/v projection shape, 1 % outliers
    (4096, 4096, 40),  # q/o projection shape, 1 % outliers
]


@pytest.mark.parametrize("M,K,n_out", SHAPES)
def test_dequant_bit_exact(cuda_device, M, K, n_out):
    layer = synthetic.random_layer(M, K, n_out, seed=M * 7919 + K)
    _dequant_check(layer, cuda_device)


def test_dequant_duplicate_ids_last_wins(cuda_device):
    layer = synthetic.random_layer(64, 256, 4, seed=5)
    ids = layer["outlier_indices"].clone()
    ids[2] = ids[0]  # repeated id: the later row must win (converter.py:59-63 replaces in order)
    layer["outlier_indices"] = ids
    _dequant_check(layer, cuda_device)


def test_dequant_unsorted_int32_ids_last_row(cuda_device):
    layer = synthetic.random_layer(96, 384, 5, seed=11, id_dtype=torch.int32, shuffle_ids=True)
    ids = layer["outlier_indices"].clone()
    ids[1] = 95  # outlier at the last row
    layer["outlier_indices"] = ids
    _dequant_check(layer, cuda_device)


@pytest.mark.parametrize("M,K,n_out", SHAPES)
@pytest.mark.parametrize("batch", [1, 3, 8])
def test_gemv_matches_fp64(cuda_device, M, K, n_out, batch):
    layer = synthetic.random_layer(M, K, n_out, seed=M * 31 + K + batch)
    dl, w_ref = _dequant_check(layer, cuda_device)
    x = synthetic.activations(batch, K, seed=1000 + batch)
    y64 = oracle.gemv_f64(w_ref, x)
    y = L.gemv(dl, torch.from_numpy(x).to(cuda_device)).cpu().numpy()
    assert y.shape == (batch, M)
    err = oracle.rel_err(y, y64)
    assert err <= REL_TOL, f"rel err {err:.3e}"


@pytest.mark.parametrize("batch", [9, 16, 17, 33, 64])
def test_gemv_larger_batches(cuda_device, batch):
    M, K, n_out = 320, 1536, 4
    layer = synthetic.random_layer(M, K, n_out, seed=batch)
    dl, w_ref = _dequant_check(layer, cuda_device)
    x = synthetic.activations(batch, K, seed=2000 + batch)
    y64 = oracle.gemv_f64(w_ref, x)
    y = L.gemv(dl, torch.from_numpy(x).to(cuda_device)).cpu().numpy()
    assert oracle.rel_err(y, y64) <= REL_TOL


def test_gemv_large_k_global_x(cuda_device):
    """batch x K too large for the shared-memory copy of x: exercises global B loads."""
    M, K, batch = 256, 14336, 8
    layer = synthetic.random_layer(M, K, 2, seed=3)
    dl, w_ref = _dequant_check(layer, cuda_device)
    x = synthetic.activations(batch, K, seed=3)
    y64 = oracle.gemv_f64(w_ref, x)
    y = L.gemv(dl, torch.from_numpy(x).to(cuda_device)).cpu().numpy()
    assert oracle.rel_err(y, y64) <= REL_TOL


def test_gemv_strided_io_and_determinism(cuda_device):
    M, K, batch = 1000, 2048, 4
    layer = synthetic.random_layer(M, K, 9, seed=77)
    dl, w_ref = _dequant_check(layer, cuda_device)
    xbig = torch.zeros(batch, K + 24, dtype=torch.float16, device=cuda_device)
    x = synthetic.activations(batch, K, seed=77)
    xbig[:, :K] = torch.from_numpy(x).to(cuda_device)
    ybig = torch.full((batch, M + 8), 7.0, dtype=torch.float16, device=cuda_device)
    L.gemv(dl, xbig[:, :K], out=ybig[:, :M])
    y1 = ybig.clone()
    for _ in range(3):
        L.gemv(dl, xbig[:, :K], out=ybig[:, :M])
    assert torch.equal(y1, ybig), "repeated calls must be bit-identical (fixed summation order)"
    assert torch.all(ybig[:, M:] == 7.0), "wrote outside the output rows"
    y64 = oracle.gemv_f64(w_ref, x)
    assert oracle.rel_err(ybig[:, :M].cpu().numpy(), y64) <= REL_TOL


def test_gemv_many_layers_shared_workspace(cuda_device):
    """Chained calls of different shapes on one stream share one workspace (self-resetting)."""
    shapes = [(4096, 4096, 40), (1024, 4096, 10), (14336, 4096, 143), (4096, 14336, 40)]
    layers = [synthetic.random_layer(M, K, n, seed=i) for i, (M, K, n) in enumerate(shapes)]
    dls = [L.prepare_layer(l, cuda_device) for l in layers]
    xs = [synthetic.activations(1, K, seed=100 + i) for i, (_, K, _) in enumerate(shapes)]
    outs = []
    for rep in range(2):
        outs.append([L.gemv(dl, torch.from_numpy(x).to(cuda_device)).cpu().numpy() for dl, x in zip(dls, xs)])
    for i, layer in enumerate(layers):
        assert np.array_equal(outs[0][i], outs[1][i])
        y64 = oracle.gemv_f64(oracle.dequantize_np(layer), xs[i])
        assert oracle.rel_err(outs[0][i], y64) <= REL_TOL


def test_invalid_index_rejected(cuda_device):
    layer = synthetic.random_layer(32, 64, 0, seed=1)
    idx = layer["indices"].clone()
    idx[3, 5] = 4
    layer["indices"] = idx
    with pytest.raises(_lib.OpcError) as ei:
        L.prepare_layer(layer, cuda_device)
    assert ei.value.code == _lib.OPC_ERR_INVALID


def test_out_of_range_outlier_id_rejected(cuda_device):
    layer = synthetic.random_layer(32, 64, 2, seed=1)
    layer["outlier_indices"] = torch.tensor([1, 32], dtype=torch.int64)
    with pytest.raises(_lib.OpcError):
        L.prepare_layer(layer, cuda_device)


def test_device_error_word_clear(cuda_device):
    import ctypes

    code = ctypes.c_int32(-1)
    _lib.check(_lib.load().opc_take_device_error(0, ctypes.byref(code)))
    assert code.value == 0


def test_shared_workspace_mixed_batches(cuda_device):
    """One workspace across batch sizes and shapes (counters must stay at a fixed offset)."""
    layers = [synthetic.random_layer(256, 14336, 2, seed=3), synthetic.random_layer(320, 1536, 4, seed=4)]
    dls = [L.prepare_layer(l, cuda_device) for l in layers]
    ws = torch.zeros(max(L.workspace_bytes(dl, 64) for dl in dls), dtype=torch.uint8, device=cuda_device)
    for batch in [64, 1, 33, 8, 16, 2, 64, 1]:
        for ly, dl in zip(layers, dls):
            x = synthetic.activations(batch, dl.K, seed=batch)
            y = L.gemv(dl, torch.from_numpy(x).to(cuda_device), workspace=ws).cpu().numpy()
            err = oracle.rel_err(y, oracle.gemv_f64(oracle.dequantize_np(ly), x))
            assert err <= REL_TOL, f"batch {batch} shape {dl.shape}: rel err {err:.3e}"

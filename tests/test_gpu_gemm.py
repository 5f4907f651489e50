"""Prefill GEMM (tcgen05) parity through the C ABI: y = x . W_hat^T against the oracle's fp64
recompute on the dequantized weights.  Tolerance: norm-wise max relative error 2e-3."""

import numpy as np
import pytest
import torch

from oracle import oracle
from opac1ty_b200 import gemm as G
from opac1ty_b200 import layer as L
from opac1ty_b200 import synthetic

REL_TOL = 2e-3


def _run(cuda_device, M, K, n_out, n_tok, seed=0, **kw):
    ly = synthetic.random_layer(M, K, n_out, seed=seed, **kw)
    dl = L.prepare_layer(ly, cuda_device)
    x = synthetic.activations(n_tok, K, seed=seed + 1)
    y = G.gemm(dl, torch.from_numpy(x).to(cuda_device))
    torch.cuda.synchronize()
    y64 = oracle.gemv_f64(oracle.dequantize_np(ly), x)
    return y.cpu().numpy(), y64, dl


@pytest.mark.gpu
@pytest.mark.parametrize("M,K,n_out,n_tok", [
    (128, 128, 0, 1),
    (256, 512, 3, 64),
    (300, 520, 5, 300),       # ragged M, K, tokens
    (1024, 1024, 10, 512),
    (4096, 4096, 40, 512),
    (640, 14336, 7, 257),     # long K (down projection), one partial token tile
])
def test_gemm_matches_fp64(cuda_device, M, K, n_out, n_tok):
    y, y64, _ = _run(cuda_device, M, K, n_out, n_tok)
    assert y.shape == (n_tok, M)
    assert np.all(np.isfinite(y))
    assert oracle.rel_err(y, y64) <= REL_TOL


@pytest.mark.gpu
def test_gemm_unaligned_k_and_duplicate_ids(cuda_device):
    M, K, n_tok = 200, 37, 33
    ly = synthetic.random_layer(M, K, 4, seed=3, shuffle_ids=True)
    ly["outlier_indices"] = torch.cat([ly["outlier_indices"], ly["outlier_indices"][:1], torch.tensor([M - 1])])
    ly["outlier_values"] = torch.cat([ly["outlier_values"], ly["outlier_values"][:1] * 3, ly["outlier_values"][1:2]])
    dl = L.prepare_layer(ly, cuda_device)
    x = synthetic.activations(n_tok, K, seed=9)
    y = G.gemm(dl, torch.from_numpy(x).to(cuda_device)).cpu().numpy()
    y64 = oracle.gemv_f64(oracle.dequantize_np(ly), x)
    assert oracle.rel_err(y, y64) <= REL_TOL


@pytest.mark.gpu
def test_gemm_matches_gemv_and_is_deterministic(cuda_device):
    M, K, n_tok = 512, 2048, 40
    ly = synthetic.random_layer(M, K, 6, seed=4)
    dl = L.prepare_layer(ly, cuda_device)
    x = torch.from_numpy(synthetic.activations(n_tok, K, seed=5)).to(cuda_device)
    y1 = G.gemm(dl, x)
    y2 = G.gemm(dl, x)
    yv = L.gemv(dl, x)
    torch.cuda.synchronize()
    assert torch.equal(y1, y2)
    y64 = oracle.gemv_f64(oracle.dequantize_np(ly), x.cpu().numpy())
    assert oracle.rel_err(y1.cpu().numpy(), y64) <= REL_TOL
    assert oracle.rel_err(yv.cpu().numpy(), y64) <= REL_TOL


@pytest.mark.gpu
def test_gemm_reports_no_device_error(cuda_device):
    from opac1ty_b200 import _lib
    import ctypes

    _run(cuda_device, 256, 256, 2, 100)
    code = ctypes.c_int32(-1)
    _lib.check(_lib.load().opc_take_device_error(0, ctypes.byref(code)))
    assert code.value == 0


@pytest.mark.gpu
@pytest.mark.parametrize("n_tok", [1, 16, 17, 32, 40, 64, 100, 128, 200, 256])
def test_gemm_every_token_tile_size(cuda_device, n_tok):
    # The host picks the token tile (16..256 columns of tensor memory) from the token count: every
    # tile size must give the same result as the fp64 recompute.
    y, y64, _ = _run(cuda_device, 1024, 1024, 9, n_tok, seed=n_tok)
    assert y.shape == (n_tok, 1024)
    assert oracle.rel_err(y, y64) <= REL_TOL


@pytest.mark.gpu
def test_gemm_persistent_ctas_cycle_both_accumulators(cuda_device):
    # More tiles than SMs: every CTA walks several tiles, alternating its two tensor-memory
    # accumulators (the epilogue of one tile overlaps the MMAs of the next).  Reference: fp64
    # matmul on the GPU of the oracle's (bit-exact) dequantized weights.
    M, K, n_out, n_tok = 8192, 1024, 50, 1024
    ly = synthetic.random_layer(M, K, n_out, seed=11)
    dl = L.prepare_layer(ly, cuda_device)
    x = torch.from_numpy(synthetic.activations(n_tok, K, seed=12)).to(cuda_device)
    y = G.gemm(dl, x)
    w = torch.from_numpy(oracle.dequantize_np(ly)).to(cuda_device).double()
    y64 = (x.double() @ w.T).cpu().numpy()
    torch.cuda.synchronize()
    assert oracle.rel_err(y.cpu().numpy(), y64) <= REL_TOL
    assert torch.equal(y, G.gemm(dl, x))  # deterministic


@pytest.mark.gpu
@pytest.mark.parametrize("M,K,n_out,batch", [(1024, 4096, 10, 32), (300, 14336, 3, 20), (4096, 4096, 40, 64)])
def test_gemv_route_to_gemm_with_k_split(cuda_device, M, K, n_out, batch):
    # Batches above the crossover run the GEMM; with few row tiles it splits K into items whose
    # fp32 partials the last arrival adds in slice order (deterministic).
    ly = synthetic.random_layer(M, K, n_out, seed=M ^ K)
    dl = L.prepare_layer(ly, cuda_device)
    x = torch.from_numpy(synthetic.activations(batch, K, seed=batch)).to(cuda_device)
    y1 = L.gemv(dl, x)
    y2 = L.gemv(dl, x)
    y64 = oracle.gemv_f64(oracle.dequantize_np(ly), x.cpu().numpy())
    torch.cuda.synchronize()
    assert torch.equal(y1, y2)
    assert oracle.rel_err(y1.cpu().numpy(), y64) <= REL_TOL
    assert oracle.rel_err(G.gemm(dl, x).cpu().numpy(), y64) <= REL_TOL  # the unsplit GEMM agrees too


@pytest.mark.gpu
def test_gemm_crossover_at_batch_8_uses_the_split_workspace(cuda_device):
    from opac1ty_b200 import measure

    M, K, batch = 2048, 8192, 12
    ly = synthetic.random_layer(M, K, 20, seed=5)
    dl = L.prepare_layer(ly, cuda_device)
    x = torch.from_numpy(synthetic.activations(batch, K, seed=6)).to(cuda_device)
    y64 = oracle.gemv_f64(oracle.dequantize_np(ly), x.cpu().numpy())
    with measure.gemm_crossover(8):
        ws = torch.zeros(L.workspace_bytes(dl, batch), dtype=torch.uint8, device=cuda_device)
        y = L.gemv(dl, x, workspace=ws)
        y_again = L.gemv(dl, x, workspace=ws)  # counters were left at zero by the first call
    torch.cuda.synchronize()
    assert torch.equal(y, y_again)
    assert oracle.rel_err(y.cpu().numpy(), y64) <= REL_TOL

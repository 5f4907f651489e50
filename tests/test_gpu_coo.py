"""Element-wise (COO) outliers on the GPU: the dequant is bit-exact against the oracle, and the
GEMV (integer, fp16 and GEMM routes), the prefill GEMM and the engine agree with the fp64
recompute within 2e-3 norm-wise (the CSR epilogue adds one fp16 rounding, <= 2^-11 of |y|)."""

import numpy as np
import pytest
import torch

from oracle import oracle
from opac1ty_b200 import gemm as G
from opac1ty_b200 import layer as L
from opac1ty_b200 import synthetic
from opac1ty_b200.quantize import QuantizeConfig, VectorQuantizer

pytestmark = pytest.mark.gpu
TOL = 2e-3


@pytest.mark.parametrize("svs,M,K,frac,dup", [(1, 256, 1024, 0.01, 0), (1, 100, 640, 0.05, 17), (8, 192, 512, 0.02, 9),
                                              (1, 64, 256, 0.0, 0)])
def test_sparse_dequant_is_bit_exact(cuda_device, svs, M, K, frac, dup):
    sp = synthetic.random_layer_sparse(M, K, frac, seed=M + K, svs=svs, duplicates=dup)
    dl = L.prepare_layer(sp, cuda_device)
    assert dl.coo is not None
    W = L.dequantize(dl).cpu().numpy()
    assert np.array_equal(W.view(np.uint16), oracle.dequantize_np(sp).view(np.uint16))


@pytest.mark.parametrize("svs", [1, 8])
@pytest.mark.parametrize("batch", [1, 2, 5, 16, 64])
def test_sparse_gemv_matches_fp64(cuda_device, svs, batch):
    M, K = 384, 1536
    sp = synthetic.random_layer_sparse(M, K, 0.01, seed=11 + batch, svs=svs, duplicates=4)
    dl = L.prepare_layer(sp, cuda_device)
    x = torch.from_numpy(synthetic.activations(batch, K, seed=batch)).to(cuda_device)
    y = L.gemv(dl, x).cpu().numpy()
    y64 = oracle.gemv_f64(oracle.dequantize_np(sp), x.cpu().numpy())
    assert oracle.rel_err(y, y64) < TOL


def test_sparse_gemv_noalloc_and_gemm(cuda_device):
    M, K = 512, 2048
    sp = synthetic.random_layer_sparse(M, K, 0.01, seed=21)
    dl = L.prepare_layer(sp, cuda_device)
    W = oracle.dequantize_np(sp)
    x = torch.from_numpy(synthetic.activations(4, K, seed=3)).to(cuda_device)
    assert oracle.rel_err(L.gemv_noalloc(dl, x).cpu().numpy(), oracle.gemv_f64(W, x.cpu().numpy())) < TOL
    xt = torch.from_numpy(synthetic.activations(100, K, seed=4)).to(cuda_device)
    assert oracle.rel_err(G.gemm(dl, xt).cpu().numpy(), oracle.gemv_f64(W, xt.cpu().numpy())) < TOL


def test_quantized_element_mode_layer_end_to_end(cuda_device):
    w = torch.from_numpy(synthetic.student_t_weights(256, 512, seed=31)).float()
    r = VectorQuantizer(QuantizeConfig(sub_vector_size=1, outlier_fraction=0.01, outlier_mode="element",
                                       codebook_iters=10)).quantize_layer(w)
    dl = L.prepare_layer(r, cuda_device)
    W = oracle.dequantize_np(r)
    assert np.array_equal(L.dequantize(dl).cpu().numpy().view(np.uint16), W.view(np.uint16))
    x = torch.from_numpy(synthetic.activations(1, 512, seed=5)).to(cuda_device)
    assert oracle.rel_err(L.gemv(dl, x).cpu().numpy(), oracle.gemv_f64(W, x.cpu().numpy())) < TOL


def test_engine_runs_element_outlier_layers(tmp_path, cuda_device):
    from engine_model import build, forward64, rel_err
    from opac1ty_b200.engine import Engine

    p = tmp_path / "sparse.bf2"
    m = build(p, seed=9, element=True)
    toks = np.random.default_rng(2).integers(1, m["vocab"], size=12).tolist()
    ref = forward64(m, toks)
    with Engine(p) as eng:
        assert rel_err(eng.forward(toks), ref[-1]) < 2e-2

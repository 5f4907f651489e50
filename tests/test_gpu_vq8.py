"""sub_vector_size 8 (true vector quantization) on the GPU through the C ABI: dequantized weights
bit-exact against the reference's own dequantize_layer (golden fixture) and the oracle; GEMV
against the fp64 recompute (norm-wise relative error <= 2e-3) for batches 1..16, ragged shapes,
outliers; the tcgen05 prefill GEMM against the same recompute; the decode chain (svs = 1 only)
rejects svs = 8 layers."""

from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import oracle
from opac1ty_b200 import _lib
from opac1ty_b200 import chain as C
from opac1ty_b200 import gemm as Gm
from opac1ty_b200 import layer as L
from opac1ty_b200 import synthetic

REL_TOL = 2e-3
GOLDEN = Path(__file__).resolve().parent / "golden"


def _golden(name):
    z = np.load(GOLDEN / f"{name}.npz")
    layer = {"type": "quantized", "shape": tuple(int(v) for v in z["shape"]), "codebooks": torch.from_numpy(z["codebooks"]),
             "indices": torch.from_numpy(z["indices"]),
             "outlier_values": torch.from_numpy(z["outlier_values"]) if "outlier_values" in z else None,
             "outlier_indices": torch.from_numpy(z["outlier_indices"]) if "outlier_indices" in z else None}
    return layer, z


@pytest.mark.gpu
def test_vq8_dequant_and_gemv_match_reference_golden(cuda_device):
    layer, z = _golden("dequant_svs8")
    dl = L.prepare_layer(layer, cuda_device)
    assert dl.sub_vector_size == 8
    w = L.dequantize(dl).cpu().numpy()
    np.testing.assert_array_equal(w.view(np.uint16), z["W"].view(np.uint16))  # bit-exact vs the reference
    y = L.gemv(dl, torch.from_numpy(z["x"]).to(cuda_device)).cpu().numpy()
    assert oracle.rel_err(y, z["y64"]) <= REL_TOL


@pytest.mark.gpu
@pytest.mark.parametrize("M,K,n_out", [(16, 8, 0), (200, 520, 5), (1024, 4096, 10), (300, 14336, 3), (4096, 1024, 41)])
def test_vq8_dequant_bit_exact(cuda_device, M, K, n_out):
    ly = synthetic.random_layer_vq8(M, K, n_out, seed=M + K, shuffle_ids=True)
    dl = L.prepare_layer(ly, cuda_device)
    w = L.dequantize(dl).cpu().numpy()
    np.testing.assert_array_equal(w.view(np.uint16), oracle.dequantize_np(ly).view(np.uint16))


@pytest.mark.gpu
@pytest.mark.parametrize("M,K,n_out", [(200, 520, 5), (1024, 4096, 10), (300, 14336, 3), (4096, 4096, 40)])
@pytest.mark.parametrize("batch", [1, 3, 8, 13])
def test_vq8_gemv_matches_fp64(cuda_device, M, K, n_out, batch):
    ly = synthetic.random_layer_vq8(M, K, n_out, seed=7 * M + K)
    dl = L.prepare_layer(ly, cuda_device)
    x = synthetic.activations(batch, K, seed=batch)
    y = L.gemv(dl, torch.from_numpy(x).to(cuda_device)).cpu().numpy()
    y64 = oracle.gemv_f64(oracle.dequantize_np(ly), x)
    assert np.all(np.isfinite(y))
    assert oracle.rel_err(y, y64) <= REL_TOL


@pytest.mark.gpu
def test_vq8_strided_io_duplicate_ids_and_determinism(cuda_device):
    M, K, batch = 333, 1000, 5
    ly = synthetic.random_layer_vq8(M, K, 4, seed=11)
    ly["outlier_indices"] = torch.cat([ly["outlier_indices"], ly["outlier_indices"][:1]])
    ly["outlier_values"] = torch.cat([ly["outlier_values"], ly["outlier_values"][:1] * 2])
    dl = L.prepare_layer(ly, cuda_device)
    xs = torch.zeros(batch, K + 24, dtype=torch.float16, device=cuda_device)
    x = torch.from_numpy(synthetic.activations(batch, K, seed=2)).to(cuda_device)
    xs[:, 3:3 + K] = x                                          # odd offset: unaligned rows
    ys = torch.full((batch, M + 9), 7.0, dtype=torch.float16, device=cuda_device)
    L.gemv(dl, xs[:, 3:3 + K], out=ys[:, :M])
    y2 = L.gemv(dl, x)
    torch.cuda.synchronize()
    assert torch.equal(ys[:, :M], y2)                           # same values, strided or not
    assert torch.all(ys[:, M:] == 7.0)                          # nothing written past M
    y64 = oracle.gemv_f64(oracle.dequantize_np(ly), x.cpu().numpy())
    assert oracle.rel_err(y2.cpu().numpy(), y64) <= REL_TOL
    assert torch.equal(L.gemv(dl, x), y2)                       # deterministic


@pytest.mark.gpu
def test_vq8_rejections(cuda_device):
    trim, _ = _golden("dequant_svs8_trim")                      # K not a multiple of 8
    with pytest.raises(_lib.OpcError) as e:
        L.prepare_layer(trim, cuda_device)
    assert e.value.code == _lib.OPC_ERR_UNSUPPORTED
    dl = L.prepare_layer(synthetic.random_layer_vq8(256, 512, 2, seed=1), cuda_device)
    xb = torch.zeros(1, 512, dtype=torch.float16, device=cuda_device)
    yb = torch.zeros(1, 256, dtype=torch.float16, device=cuda_device)
    with pytest.raises(_lib.OpcError):
        C.Chain([(dl, xb, yb)])


@pytest.mark.gpu
def test_vq8_through_the_kernel_manager_raw_buffers(cuda_device):
    """The reference's call shape (metal_utils.py:202-213: codebooks, indices, input, output, M,
    K, outlier values, outlier ids, n) with sub_vector_size 8 buffers, as its Metal kernel takes."""
    from opac1ty_b200.utils import CudaKernelManager

    M, K, n = 512, 2048, 5
    ly = synthetic.random_layer_vq8(M, K, n, seed=21)
    mgr = CudaKernelManager(cuda_device)
    x = torch.from_numpy(synthetic.activations(1, K, seed=4)).to(cuda_device).reshape(K)
    y = torch.empty(M, dtype=torch.float16, device=cuda_device)
    mgr.dequant_gemv(ly["codebooks"].to(cuda_device).reshape(-1), ly["indices"].to(cuda_device).reshape(-1), x, y,
                     M, K, ly["outlier_values"].to(cuda_device), ly["outlier_indices"].to(cuda_device), n)
    y64 = oracle.gemv_f64(oracle.dequantize_np(ly), x.cpu().numpy().reshape(1, K))
    assert oracle.rel_err(y.cpu().numpy().reshape(1, M), y64) <= REL_TOL


@pytest.mark.gpu
def test_vq8_gemv_with_large_staged_x_on_two_devices(cuda_device):
    # batch 8 at K = 4096 stages 8 x 8.2 KB of x: more than the default 48 KB of dynamic shared
    # memory, so the raised limit must be in force on every device the kernel runs on.
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    M, K, batch = 512, 4096, 8
    layer = synthetic.random_layer_vq8(M, K, 4, seed=5)
    x = synthetic.activations(batch, K, seed=6)
    y64 = oracle.gemv_f64(oracle.dequantize_np(layer), x)
    for d in range(2):
        dev = torch.device("cuda", d)
        with torch.cuda.device(dev):
            dl = L.prepare_layer(layer, dev)
            y = L.gemv(dl, torch.from_numpy(x).to(dev)).cpu().numpy()
        assert oracle.rel_err(y, y64) <= REL_TOL, d


@pytest.mark.gpu
@pytest.mark.parametrize("M,K,n_out,n_tok", [(200, 520, 5, 33), (1024, 4096, 10, 512), (300, 14336, 3, 16),
                                             (4096, 1024, 41, 300), (2048, 2048, 20, 1)])
def test_vq8_gemm_matches_fp64(cuda_device, M, K, n_out, n_tok):
    # The prefill GEMM selects each 8-column chunk of the A tile (one codebook vector) by its 2-bit
    # index; every token tile size and the outlier rows' dense tiles take part.
    ly = synthetic.random_layer_vq8(M, K, n_out, seed=3 * M + K, shuffle_ids=True)
    dl = L.prepare_layer(ly, cuda_device)
    x = synthetic.activations(n_tok, K, seed=n_tok)
    y = Gm.gemm(dl, torch.from_numpy(x).to(cuda_device)).cpu().numpy()
    y64 = oracle.gemv_f64(oracle.dequantize_np(ly), x)
    assert y.shape == (n_tok, M) and np.all(np.isfinite(y))
    assert oracle.rel_err(y, y64) <= REL_TOL


@pytest.mark.gpu
def test_vq8_gemm_on_the_reference_golden_and_agrees_with_the_gemv(cuda_device):
    layer, z = _golden("dequant_svs8")
    dl = L.prepare_layer(layer, cuda_device)
    x = torch.from_numpy(z["x"]).to(cuda_device)
    y = Gm.gemm(dl, x)
    assert oracle.rel_err(y.cpu().numpy(), z["y64"]) <= REL_TOL
    assert torch.equal(y, Gm.gemm(dl, x))  # deterministic
    assert oracle.rel_err(y.cpu().numpy(), L.gemv(dl, x).cpu().numpy().astype(np.float64)) <= REL_TOL

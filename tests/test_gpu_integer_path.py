"""The batch 1..2 integer GEMV path (opc_gemv and a one-step decode chain) on inputs chosen to
stress its fixed-point forms: the reference quantizer's own output (a golden fixture made by
the reference's VectorQuantizer), centroids of one row spanning three decades, x with a 2^15
dynamic range plus fp16 subnormals, and K = 14336.  Everything within the GEMV tolerance
(norm-wise 2e-3) of the fp64 recompute of the reference's dequantize-then-matmul
(opacc1ty/export/converter.py:26-67)."""

from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import oracle
from opac1ty_b200 import layer as L
from opac1ty_b200 import synthetic
from opac1ty_b200.chain import Chain

pytestmark = pytest.mark.gpu

REL_TOL = 2e-3
GOLDEN = Path(__file__).resolve().parent / "golden"


def _chain_once(dl, x):
    xb = x.clone()
    y = torch.zeros(x.shape[0], dl.M, dtype=torch.float16, device=x.device)
    ch = Chain([(dl, xb, y)])
    ch.launch()
    torch.cuda.synchronize()
    out = y.clone()
    ch.close()
    return out


def _check_all_paths(dl, w_ref, x_np, device):
    y64 = oracle.gemv_f64(w_ref, x_np)
    for b in range(1, x_np.shape[0] + 1):
        x = torch.from_numpy(np.ascontiguousarray(x_np[:b])).to(device)
        y = L.gemv(dl, x).cpu().numpy()
        assert oracle.rel_err(y, y64[:b]) <= REL_TOL, ("gemv", b)
        if b <= 2:
            yc = _chain_once(dl, x).cpu().numpy()
            assert oracle.rel_err(yc, y64[:b]) <= REL_TOL, ("chain", b)


def test_reference_quantizer_output(cuda_device):
    z = np.load(GOLDEN / "quantized_svs1.npz")
    layer = {"type": "quantized", "shape": tuple(int(v) for v in z["shape"]),
             "codebooks": torch.from_numpy(z["codebooks"]), "indices": torch.from_numpy(z["indices"]),
             "outlier_values": torch.from_numpy(z["outlier_values"]),
             "outlier_indices": torch.from_numpy(z["outlier_indices"])}
    dl = L.prepare_layer(layer, cuda_device)
    w = L.dequantize(dl).cpu().numpy()
    np.testing.assert_array_equal(w.view(np.uint16), z["W"].view(np.uint16))
    y64 = z["y64"]
    for b in (1, 2, 3):
        x = torch.from_numpy(np.ascontiguousarray(z["x"][:b])).to(cuda_device)
        assert oracle.rel_err(L.gemv(dl, x).cpu().numpy(), y64[:b]) <= REL_TOL, b
        if b <= 2:
            assert oracle.rel_err(_chain_once(dl, x).cpu().numpy(), y64[:b]) <= REL_TOL, b


def _wide_layer(M, K, seed):
    """Random layer whose every 5th row has centroids spanning ~2^10 (a, -a, a/2^10, -a/2^11)."""
    layer = synthetic.random_layer(M, K, max(1, M // 100), seed=seed)
    cb = layer["codebooks"].numpy().copy()
    rng = synthetic.rng_for(seed + 1)
    for r in range(0, M, 5):
        a = float(rng.uniform(0.02, 0.08))
        cb[r, :, 0] = np.array([a, -a, a / 1024.0, -a / 2048.0], dtype=np.float16)
    ids = layer["outlier_indices"].numpy()
    cb[ids] = 0
    layer["codebooks"] = torch.from_numpy(cb)
    return layer


def _wide_x(batch, K, seed):
    """|x| = 2^u, u uniform in [-10, 5] (a 2^15 range), random signs, 3 % fp16 subnormals."""
    rng = synthetic.rng_for(seed)
    mag = np.exp2(rng.uniform(-10.0, 5.0, size=(batch, K)))
    sub = rng.random((batch, K)) < 0.03
    mag[sub] = rng.integers(1, 1024, size=int(sub.sum())) * 2.0 ** -24
    sign = np.where(rng.random((batch, K)) < 0.5, -1.0, 1.0)
    x = (sign * mag).astype(np.float16)
    assert np.any((np.abs(x) > 0) & (np.abs(x) < 2.0 ** -14))  # subnormals present
    return x


@pytest.mark.parametrize("M,K", [(512, 14336), (1000, 4096)])
def test_wide_centroids_wide_x_and_subnormals(cuda_device, M, K):
    layer = _wide_layer(M, K, seed=M + K)
    dl = L.prepare_layer(layer, cuda_device)
    w_ref = oracle.dequantize_np(layer)
    _check_all_paths(dl, w_ref, _wide_x(3, K, seed=K), cuda_device)


def test_x_with_a_single_dominant_value(cuda_device):
    # One value carries the scale, all others are 2^-15 of it or subnormal: the fixed-point form
    # of x keeps the dominant term exactly and the dot product stays within tolerance.
    M, K = 256, 14336
    layer = synthetic.random_layer(M, K, 2, seed=9)
    dl = L.prepare_layer(layer, cuda_device)
    rng = synthetic.rng_for(10)
    x = (rng.standard_normal((2, K)) * 2.0 ** -14).astype(np.float16)
    x[:, 777] = 1.0
    x[:, 5000] = -0.5
    _check_all_paths(dl, oracle.dequantize_np(layer), x, cuda_device)

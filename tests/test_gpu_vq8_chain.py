"""sub_vector_size 8 on the decode chain (one GPU, barrier form): the chain streams each svs-8
layer's own index units and multiplies integer forms of the selected codebook vectors (one
exponent per row) with its staged x digits, so the step is an exact integer dot product like
svs 1's.  Checked against the oracle's fp64 chain, against per-GEMV svs-8 launches (fp32
accumulation: within tolerance, not bit-equal), and on the reference quantizer's own svs-8 layer
(tests/golden/dequant_svs8.npz) tiled to K = 1024."""

from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import oracle
from opac1ty_b200 import _lib
from opac1ty_b200 import decode as D
from opac1ty_b200 import layer as L
from opac1ty_b200 import synthetic
from opac1ty_b200.chain import Chain

from test_gpu_chain import _oracle_chain

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"


def _blocks8(cfg, seed=0, frac=0.01):
    shapes = synthetic.decoder_shapes(cfg)
    return [{name: synthetic.random_layer_vq8(M, K, synthetic.n_outliers_for(M, frac), seed=seed + 50 * li + pi,
                                              shuffle_ids=True)
             for pi, (name, (M, K)) in enumerate(shapes.items())} for li in range(cfg["layers"])]


CFG = {"hidden": 1024, "intermediate": 2048, "kv": 256, "layers": 2}


@pytest.mark.parametrize("batch", [1, 2])
def test_vq8_chain_matches_oracle_and_launches(cuda_device, batch):
    bds = _blocks8(CFG)
    x = synthetic.activations(batch, CFG["hidden"], seed=5)
    ys = {}
    for use_chain in (True, False):
        st = D.DecodeStack.from_block_dicts(bds, CFG["hidden"], CFG["intermediate"], CFG["kv"], cuda_device,
                                            batch=batch, use_chain=use_chain, chain_form="barrier")
        assert (st.chain is not None) == use_chain
        st.bufs["x"].copy_(torch.from_numpy(x))
        ys[use_chain] = st.step_eager().clone().cpu().numpy()
        if use_chain:  # deterministic: a second step from the same input is bit-equal
            st.bufs["x"].copy_(torch.from_numpy(x))
            assert np.array_equal(st.step_eager().cpu().numpy(), ys[True])
    y64 = _oracle_chain(x, bds, CFG)
    assert oracle.rel_err(ys[True], y64) <= 5e-3
    assert oracle.rel_err(ys[False], y64) <= 5e-3


def test_vq8_chain_on_the_reference_quantizers_layer(cuda_device):
    g = np.load(GOLDEN / "dequant_svs8.npz")
    reps = 1024 // g["W"].shape[1]                      # 64 columns -> K = 1024
    layer = {"type": "quantized", "shape": (g["W"].shape[0], 1024),
             "codebooks": torch.from_numpy(g["codebooks"]),
             "indices": torch.from_numpy(np.tile(g["indices"], (1, reps))),
             "outlier_values": torch.from_numpy(np.tile(g["outlier_values"], (1, reps))),
             "outlier_indices": torch.from_numpy(g["outlier_indices"])}
    W = oracle.dequantize_np(layer)
    assert np.array_equal(W, np.tile(g["W"], (1, reps)))  # the tiled layer is the golden matrix tiled
    dl = L.prepare_layer(layer, cuda_device)
    for batch in (1, 2):
        x = torch.from_numpy(np.tile(g["x"][:batch], (1, reps))).to(cuda_device)
        y = torch.empty(batch, dl.M, dtype=torch.float16, device=cuda_device)
        ch = Chain([(dl, x, y)], form="barrier")
        ch.launch()
        torch.cuda.synchronize()
        y64 = oracle.gemv_f64(W, x.cpu().numpy())
        assert oracle.rel_err(y.cpu().numpy(), y64) <= 2e-3
        ch.close()


def test_vq8_chain_needs_k_multiple_of_1024(cuda_device):
    ly = synthetic.random_layer_vq8(64, 512, 1, seed=3)
    dl = L.prepare_layer(ly, cuda_device)
    x = torch.zeros(1, 512, dtype=torch.float16, device=cuda_device)
    y = torch.empty(1, 64, dtype=torch.float16, device=cuda_device)
    with pytest.raises(_lib.OpcError, match="multiple of 1024"):
        Chain([(dl, x, y)], form="barrier")

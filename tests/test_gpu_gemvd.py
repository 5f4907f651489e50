"""The single-launch integer GEMV (gemvd_kernel, what opc_gemv runs for batch 1..2).

Every warp takes a contiguous range of units, and row tiles shared by several warps (of one CTA
or of several) are summed with count-carrying int64 atomics in the workspace.  The partial sums
are exact integers, so the result does not depend on the partition: the rows of a batch-2 call
equal two batch-1 calls (each batch row has its own x scale), a one-step decode chain (another
partition of the same arithmetic), and a repeated call (the accumulators clear themselves), all
bit for bit.  Shapes: a single weight, ragged M and K (x read element-wise), more than one
outlier tile, and Llama-3.1-8B projections whose tiles are split over many warps and CTAs."""

import numpy as np
import pytest
import torch

from oracle import oracle
from opac1ty_b200 import layer as L, synthetic
from opac1ty_b200.chain import Chain

pytestmark = pytest.mark.gpu
REL_TOL = 2e-3


@pytest.mark.parametrize("M,K,n_out", [(1, 1, 0), (17, 37, 2), (130, 1000, 17), (4096, 4096, 40),
                                       (28672, 4096, 286), (4096, 14336, 40)])
def test_partitions_agree_bit_for_bit(cuda_device, M, K, n_out):
    layer = synthetic.random_layer(M, K, n_out, seed=M + K)
    dl = L.prepare_layer(layer, cuda_device)
    x = synthetic.activations(2, K, seed=K)
    xt = torch.from_numpy(x).to(cuda_device)
    y2 = L.gemv(dl, xt).cpu().numpy()
    y1 = np.stack([L.gemv(dl, xt[b:b + 1]).cpu().numpy()[0] for b in range(2)])
    assert np.array_equal(y2.view(np.uint16), y1.view(np.uint16)), "batch-2 rows differ from batch-1 calls"
    again = L.gemv(dl, xt).cpu().numpy()
    assert np.array_equal(again.view(np.uint16), y2.view(np.uint16)), "a repeated call differs"
    yc = torch.empty(2, M, dtype=torch.float16, device=cuda_device)
    ch = Chain([(dl, xt, yc)], form="barrier")
    ch.launch()
    torch.cuda.synchronize()
    ch.close()
    assert np.array_equal(yc.cpu().numpy().view(np.uint16), y2.view(np.uint16)), "the decode chain differs"
    if M * K <= 1 << 24:  # the fp64 recompute of the larger shapes is covered by the GEMV tests
        assert oracle.rel_err(y2, oracle.gemv_f64(oracle.dequantize_np(layer), x)) <= REL_TOL

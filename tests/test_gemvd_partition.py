"""The unit partition of the single-launch GEMV (opac1ty_b200/csrc/opc_gemvd.cuh), restated on the
CPU: warp w of NW active warps takes units [w U / NW, (w+1) U / NW), the warp holding unit u is
((u + 1) NW - 1) / U, and a row tile's contributor count is the difference of the holders of
its first and last unit plus one.  The kernel completes a shared row when exactly that many
count-carrying additions have arrived, so the count must equal the number of warps whose ranges
meet the tile, for every shape and grid the host can choose (NW = min(grid * 16, U), grid =
min(SMs, ceil(U / 16)), 32-bit products below 2^32)."""

import numpy as np
import pytest

from opac1ty_b200 import layer as L

SMS = 148
WARPS = 16


def _ranges(U, NW):
    w = np.arange(NW + 1, dtype=np.int64)
    return (w * U) // NW


def _warp_of(u, U, NW):
    return ((u + 1) * NW - 1) // U


def _segments(Up, KT, U, KO):
    s = [(b, b + KT) for b in range(0, Up, KT)]
    s += [(b, b + KO) for b in range(Up, U, KO)]
    return s


@pytest.mark.parametrize("M,K,n_out", [(1, 1, 0), (17, 37, 2), (130, 1000, 17), (4096, 4096, 40), (6144, 4096, 60),
                                       (28672, 4096, 286), (4096, 14336, 40), (57344, 8192, 573), (8192, 28672, 81),
                                       (128256, 4096, 0)])
def test_contributor_counts_match_the_ranges(M, K, n_out):
    plan = L.plan_layer(M, K, n_out, 1)
    KT, KO = plan.k_units, plan.outlier_k_units
    Up, U = plan.packed_units, plan.total_units
    assert Up == plan.row_tiles * KT and U == Up + plan.outlier_tiles * KO
    grid = min(SMS, max(1, -(-U // WARPS)))
    NW = min(grid * WARPS, U)
    assert NW * U < 2 ** 32  # the host's condition for this kernel
    bounds = _ranges(U, NW)
    assert (np.diff(bounds) >= 1).all(), "an active warp without units"
    for sb, se in _segments(Up, KT, U, KO):
        meets = int(np.sum((bounds[:-1] < se) & (bounds[1:] > sb)))
        need = _warp_of(se - 1, U, NW) - _warp_of(sb, U, NW) + 1
        assert need == meets, (sb, se)
        assert 1 <= need <= 4095
        whole = any(bounds[w] <= sb and se <= bounds[w + 1] for w in range(_warp_of(sb, U, NW), _warp_of(sb, U, NW) + 1))
        assert whole == (need == 1)


@pytest.mark.parametrize("seed", range(4))
def test_random_unit_counts(seed):
    rng = np.random.default_rng(seed)
    for U in rng.integers(1, 400_000, size=200):
        U = int(U)
        grid = min(SMS, max(1, -(-U // WARPS)))
        NW = min(grid * WARPS, U)
        bounds = _ranges(U, NW)
        assert bounds[0] == 0 and bounds[-1] == U and (np.diff(bounds) >= 1).all()
        for u in rng.integers(0, U, size=50):
            w = _warp_of(int(u), U, NW)
            assert bounds[w] <= u < bounds[w + 1]

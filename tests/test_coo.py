"""Element-wise (COO) outliers without a GPU: the quantizer's element mode, the .bf2 layer type the
reference reserves for them (format/header.py:57-60), the oracle's dequant semantics, and the
host-side row compression (opc_coo_build) against numpy."""

import ctypes

import numpy as np
import pytest
import torch

from oracle import oracle
from opac1ty_b200 import _lib, synthetic
from opac1ty_b200.format import BF2Reader, BF2Writer
from opac1ty_b200.quantize import QuantizeConfig, VectorQuantizer


def test_quantizer_element_mode_keeps_the_largest_weights_exactly():
    w = torch.from_numpy(synthetic.student_t_weights(96, 128, seed=3)).float()
    q = VectorQuantizer(QuantizeConfig(sub_vector_size=1, outlier_fraction=0.01, outlier_mode="element",
                                       codebook_iters=5))
    r = q.quantize_layer(w)
    assert r["type"] == "sparse_outlier"
    pos = r["outlier_indices"].numpy()
    vals = r["outlier_values"].numpy()
    k = int(96 * 128 * 0.01)
    assert pos.shape == (k, 2) and vals.dtype == np.float16
    # the selected weights are the k of largest magnitude
    a = w.abs().numpy()
    thr = np.sort(a.reshape(-1))[-k]
    assert (a[pos[:, 0], pos[:, 1]] >= thr).all()
    assert np.array_equal(vals, w.numpy()[pos[:, 0], pos[:, 1]].astype(np.float16))
    # row-major order, and the dequantized matrix holds them exactly
    assert np.array_equal(pos, pos[np.lexsort((pos[:, 1], pos[:, 0]))])
    W = oracle.dequantize_np(r)
    assert np.array_equal(W[pos[:, 0], pos[:, 1]], vals)
    # the codebooks fit the clipped rows: no centroid beyond the largest non-outlier magnitude
    mask = np.zeros_like(a, dtype=bool)
    mask[pos[:, 0], pos[:, 1]] = True
    rest = np.where(mask, 0, a).max(axis=1)
    assert (np.abs(r["codebooks"].float().numpy()).max(axis=(1, 2)) <= rest * (1 + 2 ** -10) + 1e-6).all()


def test_quantizer_element_mode_zero_fraction_has_no_entries():
    w = torch.from_numpy(synthetic.student_t_weights(80, 96, seed=4)).float()
    r = VectorQuantizer(QuantizeConfig(sub_vector_size=1, outlier_fraction=0.0, outlier_mode="element",
                                       codebook_iters=3)).quantize_layer(w)
    assert r["outlier_values"].numel() == 0 and r["outlier_indices"].shape == (0, 2)


@pytest.mark.parametrize("svs", [1, 8])
def test_sparse_layer_round_trips_through_bf2(tmp_path, svs):
    sp = synthetic.random_layer_sparse(64, 256, 0.02, seed=5, svs=svs, duplicates=3)
    after = synthetic.random_layer(32, 128, 2, seed=6)
    p = tmp_path / "s.bf2"
    BF2Writer(str(p)).write({"a": sp, "b": after}, {"architecture": "t"}, {"bits": 2}, progress=False, checksum=True)
    with BF2Reader(str(p)) as r:
        assert r.checksum_ok
        fmt = r.layer_format("a")
        assert int(fmt.layer_type) == 1 and fmt.nnz == len(sp["outlier_values"]) and fmt.n_outliers == 0
        a = r.load_layer("a")
        assert a["type"] == "sparse_outlier"
        for k in ("codebooks", "indices", "outlier_values", "outlier_indices"):
            assert np.array_equal(np.asarray(a[k]), np.asarray(sp[k])), k
        b = r.load_layer("b")  # the layer after it is found at the right offset
        assert np.array_equal(np.asarray(b["indices"]), np.asarray(after["indices"]))
    assert np.array_equal(oracle.dequantize_np(a), oracle.dequantize_np(sp))


def test_oracle_last_entry_of_a_repeated_position_wins():
    sp = synthetic.random_layer_sparse(32, 128, 0.0, seed=8)
    sp["outlier_indices"] = torch.tensor([[3, 5], [3, 5], [0, 0]])
    sp["outlier_values"] = torch.tensor([1.0, -2.0, 4.0], dtype=torch.float16)
    W = oracle.dequantize_np(sp)
    assert W[3, 5] == np.float16(-2.0) and W[0, 0] == np.float16(4.0)


def _build(layer):
    cb = np.ascontiguousarray(layer["codebooks"].numpy().astype(np.float16))
    idx = np.ascontiguousarray(layer["indices"].numpy().astype(np.uint8))
    pos = np.ascontiguousarray(layer["outlier_indices"].numpy().astype(np.int64).reshape(-1, 2))
    vals = np.ascontiguousarray(layer["outlier_values"].numpy().astype(np.float16))
    M, K = layer["shape"]
    n = len(pos)
    row_ptr = np.zeros(M + 1, np.int32)
    cols = np.zeros(max(n, 1), np.int32)
    vout = np.zeros(max(n, 1), np.float16)
    delta = np.zeros(max(n, 1), np.float32)
    nnz = ctypes.c_int64()
    p = lambda a: a.ctypes.data_as(ctypes.c_void_p)
    rc = _lib.load().opc_coo_build(M, K, cb.shape[2], p(cb), p(idx), p(pos), p(vals), n, p(row_ptr), p(cols), p(vout),
                                   p(delta), ctypes.byref(nnz))
    return rc, row_ptr, cols[:nnz.value], vout[:nnz.value], delta[:nnz.value]


@pytest.mark.parametrize("svs", [1, 8])
def test_coo_build_matches_numpy(svs):
    sp = synthetic.random_layer_sparse(48, 256, 0.03, seed=9, svs=svs, duplicates=5)
    rc, row_ptr, cols, vals, delta = _build(sp)
    assert rc == 0
    # numpy restatement: last entry per position, sorted by (row, col)
    pos = sp["outlier_indices"].numpy()
    v = sp["outlier_values"].numpy()
    last = {}
    for j, (r, c) in enumerate(pos):
        last[(int(r), int(c))] = j
    keys = sorted(last)
    assert len(cols) == len(keys)
    W0 = oracle.dequantize_np(dict(sp, type="quantized", outlier_values=None, outlier_indices=None))
    for i, (r, c) in enumerate(keys):
        assert row_ptr[r] <= i < row_ptr[r + 1] and cols[i] == c
        assert vals[i] == v[last[(r, c)]]
        assert delta[i] == np.float32(v[last[(r, c)]]) - np.float32(W0[r, c])
    assert row_ptr[0] == 0 and row_ptr[-1] == len(keys) and (np.diff(row_ptr) >= 0).all()


def test_coo_build_rejects_out_of_range_positions():
    sp = synthetic.random_layer_sparse(16, 128, 0.01, seed=10)
    sp["outlier_indices"] = torch.tensor([[16, 0]])
    sp["outlier_values"] = torch.tensor([1.0], dtype=torch.float16)
    rc, *_ = _build(sp)
    assert rc == _lib.OPC_ERR_INVALID
    assert "outside" in _lib.load().opc_last_error().decode()

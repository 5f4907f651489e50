"""Pin the CPU oracle to fixtures produced by the reference implementation itself
(tests/golden/make_golden.py runs opacc1ty's dequantize_layer / quantize_layer / BF2Writer)."""

import hashlib
import json
from pathlib import Path

import numpy as np
import pytest

from oracle import oracle
from opac1ty_b200 import synthetic

GOLDEN = Path(__file__).resolve().parent / "golden"
CASES = ["dequant_svs1", "dequant_svs8", "dequant_svs8_trim", "quantized_svs1"]


def load_case(name):
    z = np.load(GOLDEN / f"{name}.npz")
    layer = {"type": "quantized", "shape": tuple(int(v) for v in z["shape"]), "codebooks": z["codebooks"],
             "indices": z["indices"], "outlier_values": z["outlier_values"] if "outlier_values" in z else None,
             "outlier_indices": z["outlier_indices"] if "outlier_indices" in z else None}
    return layer, z


@pytest.mark.parametrize("name", CASES)
def test_numpy_dequant_matches_reference(name):
    layer, z = load_case(name)
    w = oracle.dequantize_np(layer)
    assert w.shape == z["W"].shape
    assert np.array_equal(w.view(np.uint16), z["W"].view(np.uint16))


@pytest.mark.parametrize("name", CASES)
def test_c_dequant_matches_reference(name):
    layer, z = load_case(name)
    w = oracle.dequantize_c(layer)
    assert np.array_equal(w.view(np.uint16), z["W"].view(np.uint16))


@pytest.mark.parametrize("name", CASES)
def test_gemv_f64_matches_reference_matmul(name):
    layer, z = load_case(name)
    y64 = oracle.gemv_f64(z["W"], z["x"])
    np.testing.assert_allclose(y64, z["y64"], rtol=1e-12, atol=1e-12)
    # the reference's own fp32 torch matmul is within fp32 rounding of the fp64 recompute
    assert oracle.rel_err(z["y32"], y64) < 1e-5


def test_cpu_baseline_port_matches_reference():
    for name in ["dequant_svs1", "quantized_svs1"]:
        layer, z = load_case(name)
        y = oracle.gemv_cpu(layer, z["x"], threads=2)
        assert oracle.rel_err(y, z["y64"]) < 2e-3


def test_reference_quantizer_fixture_properties():
    """The reference quantizer zeroes outlier rows before k-means and keeps them as fp16 rows."""
    layer, z = load_case("quantized_svs1")
    inp = np.load(GOLDEN / "quantized_svs1_input.npz")
    mask = inp["outlier_mask"]
    ids = z["outlier_indices"]
    assert z["outlier_indices"].dtype == np.int64  # torch.where -> int64, as the reference writes
    assert np.array_equal(np.where(mask)[0], ids)
    assert 3 in ids  # the planted outlier row
    np.testing.assert_array_equal(z["outlier_values"], inp["weight"][ids].astype(np.float16))


def test_config0_pin():
    """4096x4096 layer with 40 outlier rows (seeded): the oracle reproduces the SHA-256 of the
    reference's dequantize_layer output and the fp64 GEMV."""
    pin_path = GOLDEN / "config0_pin.json"
    if not pin_path.exists():
        pytest.skip("config-0 pin not generated")
    pin = json.loads(pin_path.read_text())
    layer = synthetic.random_layer(4096, 4096, 40, seed=2024)
    w = oracle.dequantize_np(layer)
    assert hashlib.sha256(np.ascontiguousarray(w).tobytes()).hexdigest() == pin["W_sha256"]
    assert hashlib.sha256(np.ascontiguousarray(oracle.dequantize_c(layer)).tobytes()).hexdigest() == pin["W_sha256"]
    x = synthetic.activations(1, 4096, seed=2025)
    y = np.load(GOLDEN / "config0_y.npz")
    np.testing.assert_allclose(oracle.gemv_f64(w, x), y["y64"], rtol=1e-12, atol=1e-12)


def test_oracle_rejects_bad_index():
    layer, _ = load_case("dequant_svs1")
    idx = np.array(layer["indices"]).copy()
    idx[0, 0] = 4
    layer["indices"] = idx
    with pytest.raises(IndexError):
        oracle.dequantize_c(layer)
    with pytest.raises(IndexError):
        oracle.dequantize_np(layer)


def test_fp16_conversions_exhaustive():
    lib = oracle.load()
    hs = np.arange(0, 65536, 3, dtype=np.uint16)
    f = np.array([lib.oracle_half_to_float(int(h)) for h in hs], dtype=np.float32)
    ref = hs.view(np.float16).astype(np.float32)
    assert np.all((f == ref) | (np.isnan(f) & np.isnan(ref)))
    xs = np.random.default_rng(0).standard_normal(5000).astype(np.float32) * np.float32(300)
    got = np.array([lib.oracle_float_to_half(float(v)) for v in xs], dtype=np.uint16)
    assert np.array_equal(got, xs.astype(np.float16).view(np.uint16))

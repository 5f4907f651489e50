"""The C ABI without a GPU: the library loads, exports every entry point declared in
include/opc_b200.h, and its host-side logic (planning, validation, errors) behaves."""

import ctypes
import re
from pathlib import Path

import pytest

from opac1ty_b200 import _lib

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "opc_b200.h"


def declared_functions():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(opc_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    names = declared_functions()
    assert len(names) >= 10
    for n in names:
        assert hasattr(lib, n), f"{n} declared in opc_b200.h but not exported"
    assert set(names) == set(_lib.PROTOTYPES), "ctypes prototypes out of sync with the header"


def test_version_and_no_error():
    assert _lib.version().startswith("opc_b200 ")
    assert "abi 1" in _lib.version()


def test_plan_shapes():
    from opac1ty_b200.layer import plan_layer

    p = plan_layer(4096, 4096, 40)
    assert (p.row_tiles, p.k_units, p.outlier_tiles, p.outlier_k_units) == (256, 32, 3, 256)
    assert p.packed_units == 8192 and p.total_units == 8192 + 3 * 256
    # packed units + int8 outlier units + fp16 outlier units + row-major outlier rows (3*16 x 4096
    # fp16); split fp16 + integer codebooks
    assert p.units_bytes == (8192 + 2 * 3 * 256) * 512 + 48 * 4096 * 2
    assert p.codebook_bytes == 4096 * (8 + 16)
    assert p.outlier_rows_bytes == 3 * 16 * 8
    p = plan_layer(17, 37, 2)
    assert (p.M_pad, p.K_pad, p.row_tiles, p.k_units) == (32, 128, 2, 1)


def test_plan_rejects_bad_arguments():
    from opac1ty_b200.layer import plan_layer

    with pytest.raises(_lib.OpcError) as e:
        plan_layer(0, 16, 0)
    assert e.value.code == _lib.OPC_ERR_INVALID
    with pytest.raises(_lib.OpcError) as e:
        plan_layer(16, 16, 17)
    assert e.value.code == _lib.OPC_ERR_INVALID
    with pytest.raises(_lib.OpcError) as e:
        plan_layer(16, 64, 0, sub_vector_size=4)
    assert e.value.code == _lib.OPC_ERR_UNSUPPORTED
    assert "sub_vector_size" in _lib.last_error()
    with pytest.raises(_lib.OpcError) as e:
        plan_layer(16, 60, 0, sub_vector_size=8)   # K not a multiple of 8
    assert e.value.code == _lib.OPC_ERR_UNSUPPORTED


def test_plan_svs8_sizes():
    from opac1ty_b200.layer import plan_layer

    p = plan_layer(40, 520, 3, sub_vector_size=8)
    assert (p.row_tiles, p.M_pad, p.k_units, p.K_pad) == (3, 48, 3, 768)
    assert p.units_bytes == 3 * 3 * 128 + 16 * 768 * 2     # index units, then 16 outlier slots
    assert p.codebook_bytes == 48 * 64
    assert p.tile_mask_bytes == 3 * 2


def test_count_distinct_ids():
    lib = _lib.load()
    arr = (ctypes.c_int64 * 6)(5, 3, 5, 9, 3, 1)
    assert lib.opc_count_distinct_ids(arr, 6) == 4
    assert lib.opc_count_distinct_ids(None, 0) == 0


def test_gemv_rejects_null_layer_without_touching_a_device():
    lib = _lib.load()
    rc = lib.opc_gemv(None, None, 0, None, 0, 1, None, 0, None)
    assert rc == _lib.OPC_ERR_INVALID
    assert "invalid layer plan" in _lib.last_error()


def test_device_info_without_gpu_fails_cleanly():
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    lib = _lib.load()
    props = _lib.DeviceProps()
    rc = lib.opc_device_info(0, ctypes.byref(props))
    assert rc in (_lib.OPC_ERR_CUDA, _lib.OPC_ERR_INVALID)


def test_product_does_not_import_the_oracle():
    for p in (ROOT / "opac1ty_b200").rglob("*.py"):
        src = p.read_text()
        assert "import oracle" not in src and "from oracle" not in src, p


def test_metal_manager_raises_and_cuda_manager_mirrors_methods():
    from opac1ty_b200.utils import CudaKernelManager, MetalKernelManager

    with pytest.raises(RuntimeError):
        MetalKernelManager()
    for m in ("compile_kernels", "load_library", "dequant_gemv", "dequant_gemm", "prepare_layer"):
        assert callable(getattr(CudaKernelManager, m))


def test_gemm_crossover_setting_is_validated_and_kept():
    lib = _lib.load()
    old = lib.opc_gemm_crossover()
    assert old == 8  # the measured default: the GEMM wins from batch 16 on every 8B and 70B projection
    try:
        assert lib.opc_set_gemm_crossover(65) == _lib.OPC_ERR_INVALID
        assert "crossover" in _lib.last_error()
        assert lib.opc_set_gemm_crossover(64) == _lib.OPC_OK
        assert lib.opc_gemm_crossover() == 64
    finally:
        lib.opc_set_gemm_crossover(old)

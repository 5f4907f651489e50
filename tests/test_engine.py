"""The engine API (include/opc_engine.h) without a GPU: every declared function is exported, the
constants match the reference's header, and file errors surface through bf_engine_get_error
before any device work (runtime/src/bf2_format.c:151-225 keeps the handle and sets the error)."""

import re
from pathlib import Path

import numpy as np
import pytest

from opac1ty_b200 import engine as E

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "opc_engine.h"


def declared():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(bf_[a-z0-9_]+)\s*\(", text)))


def test_every_declared_function_is_exported_and_bound():
    names = declared()
    assert "bf_engine_forward_step" in names and "bf_engine_create" in names
    assert set(names) == set(E.PROTOTYPES)
    L = E.lib()
    for n in names:
        assert hasattr(L, n)


def test_constants_and_version():
    d = E.default_sampling()
    assert (d.temperature, d.top_p, d.top_k, d.repetition_penalty, d.seed) == (1.0, 0.0, 0, 1.0, 0)
    assert E.lib().bf_version().decode().startswith("opc_b200 engine")
    assert E.lib().bf_has_metal_gpu() == 0


def _error_of(path) -> str:
    L = E.lib()
    h = L.bf_engine_create(str(path).encode())
    assert h
    try:
        err = L.bf_engine_get_error(h)
        assert err, "a failed load must leave an error on the handle"
        # every compute call on a failed handle returns -1
        out = np.zeros(4, dtype=np.float32)
        assert L.bf_engine_forward_step(h, 0, out.ctypes.data_as(E._F32P), 4) == -1
        return err.decode()
    finally:
        L.bf_engine_destroy(h)


def test_missing_file(tmp_path):
    assert "Cannot open file" in _error_of(tmp_path / "nope.bf2")


def test_bad_magic(tmp_path):
    p = tmp_path / "x.bf2"
    p.write_bytes(b"NOPE" + bytes(60))
    assert "bad magic" in _error_of(p)


def test_null_path_returns_null():
    assert not E.lib().bf_engine_create(None)


def test_model_without_embedding_is_rejected_after_parsing(tmp_path):
    # the reference-written file (int64 outlier ids) parses; it holds no embedding
    golden = ROOT / "tests" / "golden" / "ref_int64.bf2"
    if not golden.exists():
        pytest.skip("golden file absent")
    assert "model.embed_tokens.weight" in _error_of(golden)


def test_checksum_mismatch_is_detected(tmp_path):
    from engine_model import build

    p = tmp_path / "m.bf2"
    build(p, hidden=128, heads=2, kv_heads=1, n_layers=1, inter=256, vocab=160, checksum=True)
    data = bytearray(p.read_bytes())
    data[len(data) // 2] ^= 0x55
    p.write_bytes(bytes(data))
    assert "checksum mismatch" in _error_of(p)


def test_valid_model_parses_up_to_the_device(tmp_path):
    """Without a GPU a well-formed model gets through parsing and fails at the first CUDA call."""
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    from engine_model import build

    p = tmp_path / "m.bf2"
    build(p, hidden=128, heads=2, kv_heads=1, n_layers=1, inter=256, vocab=160, checksum=True)
    assert "cudaSetDevice" in _error_of(p)


@pytest.mark.parametrize("cut", [8, 20, 0.25, 0.5, 0.75, 0.999, -1])
def test_truncated_file_is_rejected_while_parsing(tmp_path, cut):
    """A file cut short anywhere -- in the file header, a layer header or a payload -- is refused
    by the parser with an error on the handle, before any device work."""
    from engine_model import build

    p = tmp_path / "m.bf2"
    build(p, hidden=128, heads=2, kv_heads=1, n_layers=1, inter=256, vocab=160, checksum=False)
    data = p.read_bytes()
    n = len(data) + cut if isinstance(cut, int) and cut < 0 else (cut if isinstance(cut, int) else int(len(data) * cut))
    p.write_bytes(data[:n])
    err = _error_of(p)
    assert "cudaSetDevice" not in err and "CUDA" not in err, err


def _first_layer_header(data: bytes) -> int:
    import struct

    pos = 12
    pos += 8 + struct.unpack_from("<I", data, pos)[0]   # model JSON (length written twice)
    pos += 4 + struct.unpack_from("<I", data, pos)[0]   # quantize JSON
    return pos + 4                                      # layer count


@pytest.mark.parametrize("field,offset,width,value", [
    ("nnz", 51, 8, 2 ** 62), ("nnz", 51, 8, 2 ** 64 - 1), ("nnz", 51, 8, 10 ** 12),
    ("n_groups", 11, 4, 0x7FFFFFFF), ("n_groups", 11, 4, 0xFFFFFFFF),
    ("in_features", 7, 4, 0x7FFFFFFF), ("in_features", 7, 4, 0xFFFFFFFF), ("out_features", 3, 4, 0xFFFFFFFF)])
def test_oversized_layer_fields_are_refused(tmp_path, field, offset, width, value):
    """Layer header fields that describe more bytes than the file holds (or sizes past 2^31) are
    refused while parsing; sizes are summed without wrapping around, so no field value makes the
    loader read outside the mapped file.  The first layer of this model has element-wise
    outliers, so its header carries the entry count (u64)."""
    from engine_model import build

    p = tmp_path / "m.bf2"
    build(p, hidden=128, heads=2, kv_heads=1, n_layers=1, inter=256, vocab=160, element=True, checksum=False)
    data = bytearray(p.read_bytes())
    h = _first_layer_header(bytes(data))
    assert data[h + 2] == 1  # a sparse_outlier layer
    data[h + offset:h + offset + width] = value.to_bytes(width, "little")
    p.write_bytes(bytes(data))
    err = _error_of(p)
    assert "truncated" in err or "invalid" in err, (field, err)

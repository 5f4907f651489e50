"""The .bf2 format: the reference's format tests restated (tests/test_format.py of opacc1ty),
plus byte-level parity with files written by the reference writer and the int64-id fix."""

import json
from pathlib import Path

import numpy as np
import pytest
import torch

from opac1ty_b200.format import HEADER_SIZE, MAGIC, BF2Header, BF2Reader, BF2Writer, LayerFormat, LayerType

GOLDEN = Path(__file__).resolve().parent / "golden"


def test_layer_format_pack_unpack():
    fmt = LayerFormat(name="test.layer", layer_type=LayerType.QUANTIZED, out_features=512, in_features=512,
                      n_groups=64, codebook_entries=4, sub_vector_size=8, n_outliers=5, cb_offset=128,
                      idx_offset=1024, out_val_offset=2048, out_idx_offset=4096)
    packed = fmt.pack()
    assert len(packed) == HEADER_SIZE == 64
    u = LayerFormat.unpack(packed)
    assert (u.out_features, u.in_features, u.layer_type, u.n_groups, u.n_outliers) == (512, 512, LayerType.QUANTIZED, 64, 5)
    assert (u.cb_offset, u.idx_offset, u.out_val_offset, u.out_idx_offset) == (128, 1024, 2048, 4096)


def test_header_pack_unpack():
    h = BF2Header(version=1, model_config={"architecture": "llama", "hidden_size": 4096},
                  quantize_config={"bits": 2}, layer_count=42)
    packed = h.pack()
    assert packed[:4] == MAGIC
    u, consumed = BF2Header.unpack(packed)
    assert consumed == len(packed)
    assert (u.version, u.model_config["architecture"], u.quantize_config["bits"], u.layer_count) == (1, "llama", 2, 42)


def test_header_rejects_bad_magic_and_truncation():
    with pytest.raises(ValueError):
        BF2Header.unpack(b"XXXX" + b"\0" * 40)
    with pytest.raises(ValueError):
        BF2Header.unpack(BF2Header(model_config={"a": 1}).pack()[:18])


def _layers():
    g = np.random.default_rng(3)
    return {
        "embed.weight": {"type": "fp16_passthrough", "shape": (320, 64),
                         "data": torch.from_numpy(g.standard_normal((320, 64)).astype(np.float16))},
        "layer.0.q_proj.weight": {
            "type": "quantized", "shape": (96, 128),
            "codebooks": torch.from_numpy(g.standard_normal((96, 4, 1)).astype(np.float16)),
            "indices": torch.from_numpy(g.integers(0, 4, (96, 128), dtype=np.uint8)),
            "outlier_values": torch.from_numpy(g.standard_normal((3, 128)).astype(np.float16)),
            "outlier_indices": torch.tensor([1, 50, 95], dtype=torch.int64)},
        "layer.0.k_proj.weight": {
            "type": "quantized", "shape": (64, 128),
            "codebooks": torch.from_numpy(g.standard_normal((64, 4, 8)).astype(np.float16)),
            "indices": torch.from_numpy(g.integers(0, 4, (64, 16), dtype=np.uint8)),
            "outlier_values": None, "outlier_indices": None},
    }


def test_roundtrip_values(tmp_path):
    layers = _layers()
    p = tmp_path / "m.bf2"
    BF2Writer(str(p)).write(layers, {"architecture": "test", "hidden_size": 128}, {"bits": 2}, progress=False)
    with BF2Reader(str(p)) as r:
        assert r.model_config["architecture"] == "test" and r.quantize_config["bits"] == 2
        assert r.layer_names() == list(layers)
        e = r.load_layer("embed.weight")
        assert e["type"] == "fp16_passthrough" and torch.equal(e["data"], layers["embed.weight"]["data"])
        q = r.load_layer("layer.0.q_proj.weight")
        src = layers["layer.0.q_proj.weight"]
        assert torch.equal(q["codebooks"], src["codebooks"]) and torch.equal(q["indices"], src["indices"])
        assert torch.equal(q["outlier_values"], src["outlier_values"])
        assert q["outlier_indices"].tolist() == [1, 50, 95]  # values survive (the reference checks shapes only)
        k = r.load_layer("layer.0.k_proj.weight")
        assert tuple(k["codebooks"].shape) == (64, 4, 8) and "outlier_values" not in k


def test_writer_is_byte_identical_to_reference_writer(tmp_path):
    """Reading the reference writer's int32-id file and writing it back reproduces every byte."""
    src = GOLDEN / "ref_int32.bf2"
    with BF2Reader(str(src)) as r:
        layers = {n: r.load_layer(n) for n in r.layer_names()}
        mcfg, qcfg = r.model_config, r.quantize_config
    out = tmp_path / "rewritten.bf2"
    BF2Writer(str(out)).write(layers, mcfg, qcfg, progress=False)
    assert out.read_bytes() == src.read_bytes()


def test_reader_accepts_int64_ids_written_by_reference():
    """The reference writes int64 ids (torch.where) but reads int32, so its own reader misreads
    every layer after an outlier layer; this reader detects the id width per layer."""
    with BF2Reader(str(GOLDEN / "ref_int64.bf2")) as r64, BF2Reader(str(GOLDEN / "ref_int32.bf2")) as r32:
        assert r64.layer_names() == r32.layer_names()
        for n in r32.layer_names():
            a, b = r64.load_layer(n), r32.load_layer(n)
            for key in b:
                if isinstance(b[key], torch.Tensor):
                    assert torch.equal(a[key], b[key]), (n, key)
    readback = json.loads((GOLDEN / "ref_int64_readback.json").read_text())
    assert any(not v.get("ok", True) for v in readback.values()), "the reference reader should fail on this file"


def test_truncated_file_rejected(tmp_path):
    data = (GOLDEN / "ref_int32.bf2").read_bytes()
    p = tmp_path / "trunc.bf2"
    p.write_bytes(data[: len(data) - 100])
    with pytest.raises(ValueError):
        BF2Reader(str(p))


def test_file_size_much_smaller_than_fp16(tmp_path):
    layers = {}
    g = np.random.default_rng(0)
    for i in range(8):
        layers[f"model.layers.{i}.self_attn.q_proj.weight"] = {
            "type": "quantized", "shape": (256, 256),
            "codebooks": torch.from_numpy(g.standard_normal((256, 4, 8)).astype(np.float16)),
            "indices": torch.from_numpy(g.integers(0, 4, (256, 32), dtype=np.uint8)),
            "outlier_values": None, "outlier_indices": None}
    p = tmp_path / "big.bf2"
    BF2Writer(str(p)).write(layers, {"architecture": "llama"}, {"bits": 2}, progress=False)
    assert p.stat().st_size < 8 * 256 * 256 * 2 * 0.3


def test_xxh64_known_answers():
    from opac1ty_b200.format import xxh64

    # published XXH64 values (seed 0)
    assert xxh64(b"") == 0xEF46DB3751D8E999
    assert xxh64(b"a") == 0xD24EC4F1A98C6E5B
    assert xxh64(b"abc") == 0x44BC2CF5AD770999
    assert xxh64(b"Nobody inspects the spammish repetition") == 0xFBCEA83C8A378BF1
    data = np.arange(1000, dtype=np.uint8)
    assert xxh64(data) == xxh64(data.tobytes()) and xxh64(data, seed=1) != xxh64(data)


def test_checksum_trailer_roundtrip_and_corruption(tmp_path):
    from opac1ty_b200.format import CHECKSUM_BYTES, FLAG_CHECKSUM, xxh64

    plain, summed = tmp_path / "plain.bf2", tmp_path / "summed.bf2"
    BF2Writer(str(plain)).write(_layers(), {"m": 1}, {"q": 2}, progress=False)
    BF2Writer(str(summed)).write(_layers(), {"m": 1}, {"q": 2}, progress=False, checksum=True)
    a, b = plain.read_bytes(), summed.read_bytes()
    # same layers at the same offsets; only the flags word and the 8-byte trailer differ
    assert len(b) == len(a) + CHECKSUM_BYTES
    assert b[:8] == a[:8] and b[12:len(a)] == a[12:]
    assert int.from_bytes(b[8:12], "little") == FLAG_CHECKSUM
    assert int.from_bytes(b[len(a):], "little") == xxh64(b[:len(a)])
    with BF2Reader(str(summed)) as r, BF2Reader(str(plain)) as rp:
        assert r.has_checksum and r.checksum_ok and not rp.has_checksum
        for name in rp.layer_names():
            x, y = r.load_layer(name), rp.load_layer(name)
            for k in x:
                if isinstance(x[k], torch.Tensor):
                    assert torch.equal(x[k], y[k]), (name, k)
    bad = bytearray(b)
    bad[len(a) // 2] ^= 0x10
    (tmp_path / "bad.bf2").write_bytes(bytes(bad))
    with pytest.raises(ValueError, match="checksum mismatch"):
        BF2Reader(str(tmp_path / "bad.bf2"))
    with BF2Reader(str(tmp_path / "bad.bf2"), verify_checksum=False) as r:   # opt out: still readable
        assert r.checksum_ok is None and len(r.layer_names()) == 3

"""The device-format cache (opac1ty_b200.devcache) without a GPU: layers built from CPU tensors
of the sizes the library's plans give go through save_layers / load_layers unchanged; a cache of
another library build, or whose buffers do not match the plan of its shape, is refused; the key
follows the .bf2 file's bytes."""

import numpy as np
import pytest
import torch

from opac1ty_b200 import devcache, synthetic
from opac1ty_b200 import layer as L
from opac1ty_b200.format import BF2Writer

CPU = torch.device("cpu")


def _fake_layer(M, K, n_out, svs, seed, name, coo=False):
    plan = L.plan_layer(M, K, n_out, svs)
    g = np.random.default_rng(seed)
    units = torch.from_numpy(g.integers(0, 256, plan.units_bytes, dtype=np.uint8))
    codebooks = torch.from_numpy(g.integers(0, 256, plan.codebook_bytes, dtype=np.uint8))
    tile_mask = torch.from_numpy(g.integers(-2 ** 15, 2 ** 15, plan.tile_mask_bytes // 2, dtype=np.int16))
    orows = torch.from_numpy(g.integers(-1, M, plan.outlier_rows_bytes // 4, dtype=np.int32))
    part = None
    if coo:
        nnz = 7
        row_ptr = torch.from_numpy(np.sort(g.integers(0, nnz + 1, M + 1)).astype(np.int32))
        row_ptr[0], row_ptr[-1] = 0, nnz
        part = L.CooPart(row_ptr, torch.from_numpy(g.integers(0, K, nnz, dtype=np.int32)),
                         torch.from_numpy(g.standard_normal(nnz).astype(np.float16)),
                         torch.from_numpy(g.standard_normal(nnz).astype(np.float32)))
    return L.DeviceLayer(plan, units, codebooks, tile_mask, orows, CPU, name, part)


def _same(a: L.DeviceLayer, b: L.DeviceLayer):
    assert bytes(a.plan) == bytes(b.plan) and a.name == b.name
    for k in ("units", "codebooks", "tile_mask", "outlier_rows"):
        assert torch.equal(getattr(a, k), getattr(b, k)), k
    assert (a.coo is None) == (b.coo is None)
    if a.coo is not None:
        for k in ("row_ptr", "cols", "values", "delta"):
            assert torch.equal(getattr(a.coo, k), getattr(b.coo, k)), k


def test_round_trip(tmp_path):
    layers = {"a.q_proj": _fake_layer(4096, 4096, 40, 1, 1, "a.q_proj"),
              "b.down": _fake_layer(130, 1000, 0, 1, 2, "b.down", coo=True),
              "c.vq8": _fake_layer(64, 1024, 1, 8, 3, "c.vq8")}
    p = tmp_path / "c.npz"
    devcache.save_layers(layers, p)
    back = devcache.load_layers(p, CPU)
    assert list(back) == list(layers)
    for k in layers:
        _same(layers[k], back[k])
    assert not list(tmp_path.glob("*.tmp*")), "temporary file left behind"


def test_other_build_is_refused(tmp_path, monkeypatch):
    p = tmp_path / "c.npz"
    monkeypatch.setattr(devcache, "_build_tag", lambda: "v0-other-build")
    devcache.save_layers({"x": _fake_layer(32, 256, 1, 1, 4, "x")}, p)
    monkeypatch.undo()
    with pytest.raises(devcache.CacheMismatch, match="build"):
        devcache.load_layers(p, CPU)


def test_buffers_must_match_the_plan(tmp_path):
    dl = _fake_layer(32, 256, 1, 1, 5, "x")
    dl.units = dl.units[:-16]  # a truncated buffer
    p = tmp_path / "c.npz"
    devcache.save_layers({"x": dl}, p)
    with pytest.raises(devcache.CacheMismatch, match="units"):
        devcache.load_layers(p, CPU)


@pytest.mark.parametrize("content", [b"garbage", b"PK\x03\x04" + b"\x00" * 40])
def test_unreadable_cache_file_raises_what_the_loader_catches(tmp_path, content):
    import zipfile

    p = tmp_path / "c.npz"
    p.write_bytes(content)
    with pytest.raises((devcache.CacheMismatch, KeyError, ValueError, OSError, EOFError, zipfile.BadZipFile)):
        devcache.load_layers(p, CPU)


def test_key_follows_the_file(tmp_path):
    a, b = tmp_path / "a.bf2", tmp_path / "b.bf2"
    for path, seed in ((a, 1), (b, 2)):
        BF2Writer(str(path)).write({"l": synthetic.random_layer(32, 128, 1, seed=seed)}, {"architecture": "t"},
                                   {"bits": 2}, progress=False)
    ka, kb = devcache.bf2_key(a), devcache.bf2_key(b)
    assert ka != kb and ka == devcache.bf2_key(a)
    data = bytearray(a.read_bytes())
    data[-1] ^= 1
    a.write_bytes(bytes(data))
    assert devcache.bf2_key(a) != ka


def test_loading_a_model_needs_a_gpu(tmp_path):
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    p = tmp_path / "m.bf2"
    BF2Writer(str(p)).write({"l": synthetic.random_layer(32, 128, 1, seed=1)}, {"architecture": "t"}, {"bits": 2},
                            progress=False)
    with pytest.raises(RuntimeError, match="CUDA"):
        devcache.load_bf2_layers(p, cache_dir=str(tmp_path))

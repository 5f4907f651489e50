"""Row-sharded tensor parallelism: shard geometry, shard contents and the sharded decode chain.

CPU only: the chain logic (opac1ty_b200.tp.tp_chain_step) runs with the oracle's GEMV (fp64
dot product rounded to fp16) and gloo all-gathers on two spawned ranks, and must reproduce the
unsharded chain bit for bit (each output row is computed from the same row and the same x).
"""

import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from oracle import oracle
from opac1ty_b200 import decode as D
from opac1ty_b200 import synthetic, tp


def test_shard_bounds_cover_rows():
    for M in (1, 15, 16, 17, 1024, 6144, 28672, 1000):
        for world in (1, 2, 3, 4, 8):
            b = tp.shard_bounds(M, world)
            S = tp.shard_rows_count(M, world)
            assert S % 16 == 0 and S * world >= M
            assert b[0][0] == 0 and b[-1][1] == M
            for (a0, a1), (c0, c1) in zip(b, b[1:]):
                assert a1 == c0
            assert all(r1 - r0 <= S for r0, r1 in b)
    assert tp.shard_rows_count(6144, 8) == 768
    assert tp.shard_rows_count(28672, 8) == 3584


@pytest.mark.parametrize("world", [2, 3, 8])
def test_shards_dequantize_to_full(world):
    M, K = 200, 96
    ly = synthetic.random_layer(M, K, 9, seed=5, shuffle_ids=True)
    # add a repeated id (last occurrence wins) and an outlier in the last row
    oi = torch.cat([ly["outlier_indices"], torch.tensor([int(ly["outlier_indices"][0]), M - 1])])
    ov = torch.cat([ly["outlier_values"], ly["outlier_values"][:1] * 2, ly["outlier_values"][1:2] * 3])
    ly["outlier_indices"], ly["outlier_values"] = oi, ov
    full = oracle.dequantize_np(ly)
    parts = []
    for r0, r1 in tp.shard_bounds(M, world):
        sh = tp.shard_layer(ly, r0, r1)
        assert tuple(sh["shape"]) == (r1 - r0, K)
        if sh["outlier_indices"] is not None:
            ids = np.asarray(sh["outlier_indices"])
            assert ids.min() >= 0 and ids.max() < r1 - r0
        parts.append(oracle.dequantize_np(sh) if r1 > r0 else np.zeros((0, K), np.float16))
    np.testing.assert_array_equal(np.concatenate(parts).view(np.uint16), full.view(np.uint16))


def test_gathered_view_layout():
    world, batch, S, M = 3, 2, 16, 40
    g = torch.arange(world * batch * S, dtype=torch.float32)
    v = tp.gathered_view(g, world, batch, S, M)
    assert tuple(v.shape) == (batch, M)
    for b in range(batch):
        for r in range(M):
            rank, i = divmod(r, S)
            assert v[b, r] == g[(rank * batch + b) * S + i]


# --- two-rank chain over gloo -------------------------------------------------------------

CFG = {"hidden": 64, "intermediate": 96, "kv": 16, "layers": 2}


def _block_dicts(cfg):
    shapes = synthetic.decoder_shapes(cfg)
    out = []
    for li in range(cfg["layers"]):
        bd = {}
        for pi, (name, (M, K)) in enumerate(shapes.items()):
            bd[name] = synthetic.random_layer(M, K, synthetic.n_outliers_for(M, 0.05), seed=100 * li + pi)
        out.append({"qkv": D.concat_rows([bd["q_proj"], bd["k_proj"], bd["v_proj"]]), "o": bd["o_proj"],
                    "gate_up": D.concat_rows([bd["gate_proj"], bd["up_proj"]]), "down": bd["down_proj"]})
    return out


def _cpu_gemv(layer, x, out):
    w = oracle.dequantize_np(layer)
    y = oracle.gemv_f64(w, x.numpy()).astype(np.float16)
    out.copy_(torch.from_numpy(y.reshape(out.shape)))


def _reference_chain(x, blocks_full, cfg):
    cur = x
    h, f = cfg["hidden"], cfg["intermediate"]
    for blk in blocks_full:
        for name in ("qkv", "o", "gate_up", "down"):
            inp = cur[:, :h] if name == "o" else cur[:, :f] if name == "down" else cur
            w = oracle.dequantize_np(blk[name])
            cur = torch.from_numpy(oracle.gemv_f64(w, inp.contiguous().numpy()).astype(np.float16))
    return cur


def _rank_main(rank, world, port, batch, result_path):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        blocks_full = _block_dicts(CFG)
        blocks = []
        for blk in blocks_full:
            sb = {}
            for name, ly in blk.items():
                M = int(ly["shape"][0])
                r0, r1 = tp.shard_bounds(M, world)[rank]
                sb[name] = tp._alloc_proj(tp.shard_layer(ly, r0, r1), M, r1 - r0, world, batch, "cpu")
            blocks.append(sb)

        def all_gather(out, inp):
            chunks = list(out.view(world, -1).unbind(0))
            dist.all_gather(chunks, inp.reshape(-1).contiguous())
            out.view(world, -1).copy_(torch.stack(chunks))

        x = torch.from_numpy(synthetic.activations(batch, CFG["hidden"], seed=7))
        y = tp.tp_chain_step(x, blocks, CFG["hidden"], CFG["intermediate"], world, _cpu_gemv, all_gather)
        if rank == 0:
            ref = _reference_chain(x, blocks_full, CFG)
            np.save(result_path, np.stack([y.numpy(), ref.numpy()]))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("batch", [1, 3])
def test_tp_chain_two_ranks_matches_unsharded(tmp_path, batch):
    world = 2
    out = tmp_path / "res.npy"
    mp.start_processes(_rank_main, args=(world, _free_port(), batch, str(out)), nprocs=world, join=True,
                       start_method="spawn")
    y, ref = np.load(out)
    assert y.shape == (batch, CFG["hidden"])
    np.testing.assert_array_equal(y.view(np.uint16), ref.view(np.uint16))


def test_chain_region_layout():
    rows = [6144, 4096, 28672, 4096, 200]
    offs, lds, soff, total = tp.chain_region_layout(rows, 2, 1000)
    assert lds == [6144, 4096, 28672, 4096, 200]
    assert all(o % 256 == 0 for o in offs) and soff % 256 == 0 and total % 256 == 0
    ends = [o + 2 * 2 * ld for o, ld in zip(offs, lds)]
    assert all(e <= n for e, n in zip(ends, offs[1:] + [soff]))   # outputs never overlap
    assert total >= soff + 1000
    _, lds2, _, _ = tp.chain_region_layout([13, 17], 1, 0)
    assert lds2 == [16, 24]                                       # 16-byte rows
    with pytest.raises(ValueError):
        tp.chain_region_layout([0], 1, 0)

"""Row-sharded decode chain on 2 (and 4, 8) GPUs, checked against the oracle's unsharded chain: the NCCL
form (GEMV + all-gather per projection) and the fused form (TPChain: one kernel per rank, rows
stored into every rank's activations over NVLink), which must equal the NCCL form bit for bit.

Runs as two spawned ranks (one per GPU) with a short process-group timeout; skipped on
machines with fewer than two GPUs.  The CPU form of the same chain logic is tests/test_tp.py.
"""

import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from oracle import oracle
from opac1ty_b200 import decode as D
from opac1ty_b200 import synthetic

CFG = {"hidden": 512, "intermediate": 1024, "kv": 128, "layers": 2}
TOL = 1e-2  # norm-wise, after 8 chained fp16 GEMVs


def _fused_blocks():
    shapes = synthetic.decoder_shapes(CFG)
    out = []
    for li in range(CFG["layers"]):
        bd = {name: synthetic.random_layer(M, K, synthetic.n_outliers_for(M, 0.01), seed=300 * li + pi)
              for pi, (name, (M, K)) in enumerate(shapes.items())}
        out.append({"qkv": D.concat_rows([bd["q_proj"], bd["k_proj"], bd["v_proj"]]), "o": bd["o_proj"],
                    "gate_up": D.concat_rows([bd["gate_proj"], bd["up_proj"]]), "down": bd["down_proj"]})
    return out


def _oracle_chain(x, fused):
    cur = x.astype(np.float16)
    h, f = CFG["hidden"], CFG["intermediate"]
    for blk in fused:
        for name in ("qkv", "o", "gate_up", "down"):
            inp = cur[:, :h] if name == "o" else cur[:, :f] if name == "down" else cur
            y64 = oracle.gemv_f64(oracle.dequantize_np(blk[name]), np.ascontiguousarray(inp))
            cur = y64.astype(np.float16)
    return y64


def _rank(rank, world, port, batch, out_path):
    import torch.distributed as dist

    from opac1ty_b200 import tp

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        fused = _fused_blocks()
        st = tp.TPDecodeStack.from_fused_blocks(fused, CFG, rank, world, dev, batch)
        x = synthetic.activations(batch, CFG["hidden"], seed=11)
        st.bufs["x"].copy_(torch.from_numpy(x))
        y = st.step_eager().cpu().numpy()
        torch.cuda.synchronize()
        if rank == 0:
            np.save(out_path, y)
            np.save(out_path + ".x.npy", x)
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
@pytest.mark.parametrize("batch", [1, 2])
def test_tp2_chain_matches_oracle(tmp_path, batch):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    out = str(tmp_path / "y.npy")
    mp.start_processes(_rank, args=(2, port, batch, out), nprocs=2, join=True, start_method="spawn")
    y = np.load(out)
    x = np.load(out + ".x.npy")
    y64 = _oracle_chain(x, _fused_blocks())
    assert oracle.rel_err(y, y64) <= TOL


def _rank_fused(rank, world, port, batch, out_path):
    """The same sharded step through TPChain (one kernel per rank, peer stores, no NCCL in the
    step) against the NCCL form on the same shards, over three chained steps."""
    import ctypes

    import torch.distributed as dist

    from opac1ty_b200 import _lib, tp

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        fused = _fused_blocks()
        st = tp.TPDecodeStack.from_fused_blocks(fused, CFG, rank, world, dev, batch)
        x = torch.from_numpy(synthetic.activations(batch, CFG["hidden"], seed=11)).to(dev)
        st.bufs["x"].copy_(x)
        ref = [st.step_eager().clone() for _ in range(3)]
        st.bufs["x"].copy_(x)
        st.enable_chain()
        got = [st.step_eager().clone() for _ in range(3)]
        torch.cuda.synchronize()
        same = [bool(torch.equal(a, b)) for a, b in zip(ref, got)]
        code = ctypes.c_int32(-1)
        _lib.check(_lib.load().opc_take_device_error(rank, ctypes.byref(code)))
        st.close()
        flags = torch.tensor([int(all(same)), code.value], device=dev)
        allf = [torch.zeros_like(flags) for _ in range(world)]
        dist.all_gather(allf, flags)
        if rank == 0:
            np.save(out_path, got[0].cpu().numpy())
            np.save(out_path + ".x.npy", x.cpu().numpy())
            np.save(out_path + ".flags.npy", torch.stack(allf).cpu().numpy())
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
@pytest.mark.parametrize("world,batch", [(2, 1), (2, 2), (4, 1), (8, 2)])
def test_tp_fused_chain_equals_nccl_and_oracle(tmp_path, world, batch):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    out = str(tmp_path / "yf.npy")
    mp.start_processes(_rank_fused, args=(world, port, batch, out), nprocs=world, join=True, start_method="spawn")
    flags = np.load(out + ".flags.npy")
    assert flags[:, 0].all(), f"fused chain differs from the NCCL form on some rank: {flags}"
    assert (flags[:, 1] == 0).all(), f"device errors: {flags}"
    y = np.load(out)
    y64 = _oracle_chain(np.load(out + ".x.npy"), _fused_blocks())
    assert oracle.rel_err(y, y64) <= TOL

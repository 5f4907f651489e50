"""Decode chain on one persistent kernel (opc_chain_*), barrier form: bit-identical to per-GEMV
launches (both accumulate exactly in integers at batch 1..2, with the same fixed-point x) and
within 2e-3 of the oracle's fp64 chain.  The dataflow form is tested in test_gpu_chain_dataflow.py."""

import numpy as np
import pytest
import torch

from oracle import oracle
from opac1ty_b200 import decode as D
from opac1ty_b200 import layer as L
from opac1ty_b200 import synthetic


def _blocks(cfg, n_out_frac=0.01, seed=0):
    shapes = synthetic.decoder_shapes(cfg)
    out = []
    for li in range(cfg["layers"]):
        bd = {name: synthetic.random_layer(M, K, synthetic.n_outliers_for(M, n_out_frac), seed=seed + 50 * li + pi,
                                           shuffle_ids=True)
              for pi, (name, (M, K)) in enumerate(shapes.items())}
        out.append(bd)
    return out


def _oracle_chain(x, block_dicts, cfg):
    cur = x.astype(np.float16)
    h, f = cfg["hidden"], cfg["intermediate"]
    y64 = None
    for bd in block_dicts:
        qkv = D.concat_rows([bd["q_proj"], bd["k_proj"], bd["v_proj"]])
        gu = D.concat_rows([bd["gate_proj"], bd["up_proj"]])
        for ly, take in ((qkv, None), (bd["o_proj"], h), (gu, None), (bd["down_proj"], f)):
            inp = cur if take is None else cur[:, :take]
            if ly is bd["o_proj"]:
                inp = cur[:, :h]
            y64 = oracle.gemv_f64(oracle.dequantize_np(ly), np.ascontiguousarray(inp))
            cur = y64.astype(np.float16)
    return y64


CFGS = [
    {"hidden": 512, "intermediate": 1024, "kv": 128, "layers": 2},
    {"hidden": 200, "intermediate": 328, "kv": 40, "layers": 3},   # ragged: tiles and k blocks cut
]


@pytest.mark.gpu
@pytest.mark.parametrize("cfg", CFGS)
@pytest.mark.parametrize("batch", [1, 2])
def test_chain_equals_launches_and_oracle(cuda_device, cfg, batch):
    bds = _blocks(cfg)
    x = synthetic.activations(batch, cfg["hidden"], seed=21)
    outs = []
    for use_chain in (True, False):
        st = D.DecodeStack.from_block_dicts(bds, cfg["hidden"], cfg["intermediate"], cfg["kv"], cuda_device,
                                            batch=batch, use_chain=use_chain,
                                            chain_form="barrier")
        assert (st.chain is not None) == use_chain
        st.bufs["x"].copy_(torch.from_numpy(x))
        y = st.step_eager().clone()
        inter = {k: v.clone() for k, v in st.bufs.items()}
        torch.cuda.synchronize()
        outs.append((y, inter))
    (yc, ic), (yl, il) = outs
    assert torch.equal(yc, yl)
    for k in ic:  # every intermediate buffer (outlier rows included) matches too
        assert torch.equal(ic[k], il[k]), k
    y64 = _oracle_chain(x, bds, cfg)
    assert oracle.rel_err(yc.cpu().numpy(), y64) <= 5e-3


@pytest.mark.gpu
def test_chain_repeated_launches_and_graph(cuda_device):
    cfg = CFGS[0]
    bds = _blocks(cfg, seed=7)
    st = D.DecodeStack.from_block_dicts(bds, cfg["hidden"], cfg["intermediate"], cfg["kv"], cuda_device,
                                        chain_form="barrier")
    x = torch.from_numpy(synthetic.activations(1, cfg["hidden"], seed=3)).to(cuda_device)
    st.bufs["x"].copy_(x)
    y1 = st.step_eager().clone()
    st.bufs["x"].copy_(x)
    st.capture()
    st.bufs["x"].copy_(x)
    y2 = st.step().clone()
    torch.cuda.synchronize()
    assert torch.equal(y1, y2)
    from opac1ty_b200 import _lib
    import ctypes
    code = ctypes.c_int32(-1)
    _lib.check(_lib.load().opc_take_device_error(0, ctypes.byref(code)))
    assert code.value == 0


@pytest.mark.gpu
def test_chain_rejects_unlinked_steps(cuda_device):
    from opac1ty_b200.chain import Chain
    from opac1ty_b200 import _lib

    a = L.prepare_layer(synthetic.random_layer(64, 64, 1, seed=1), cuda_device)
    b = L.prepare_layer(synthetic.random_layer(64, 64, 1, seed=2), cuda_device)
    x = torch.zeros(1, 64, dtype=torch.float16, device=cuda_device)
    y1 = torch.zeros_like(x)
    y2 = torch.zeros_like(x)
    with pytest.raises(_lib.OpcError):
        Chain([(a, x, y1), (b, x, y2)])   # step 1 must read step 0's output
    with pytest.raises(_lib.OpcError):
        Chain([(a, x, y1), (b, x, y2)], form="dataflow")


def _blocks_8b(n_blocks, seed):
    """Llama-3.1-8B projection shapes (the benchmark's), numpy-generated so the oracle can run them."""
    cfg = dict(synthetic.LLAMA_8B, layers=n_blocks)
    return cfg, _blocks(cfg, seed=seed)


@pytest.mark.gpu
@pytest.mark.parametrize("batch", [1, 2])
def test_chain_at_llama8b_shapes(cuda_device, batch):
    # The benchmark's shapes: K = 14336 on the down projection forces two ring stages, and at
    # batch 2 the staged x (2 x 14336 values) selects the 8-chunk staging instance of the kernel.
    cfg, bds = _blocks_8b(2, seed=100 + batch)
    x = synthetic.activations(batch, cfg["hidden"], seed=31 + batch)
    outs = []
    for use_chain in (True, False):
        st = D.DecodeStack.from_block_dicts(bds, cfg["hidden"], cfg["intermediate"], cfg["kv"], cuda_device,
                                            batch=batch, use_chain=use_chain,
                                            chain_form="barrier")
        assert (st.chain is not None) == use_chain
        st.bufs["x"].copy_(torch.from_numpy(x))
        y = st.step_eager().clone()
        inter = {k: v.clone() for k, v in st.bufs.items()}
        torch.cuda.synchronize()
        outs.append((y, inter))
        del st
    (yc, ic), (yl, il) = outs
    assert torch.equal(yc, yl)
    for k in ic:
        assert torch.equal(ic[k], il[k]), k
    y64 = _oracle_chain(x, bds, cfg)
    assert oracle.rel_err(yc.cpu().numpy(), y64) <= 5e-3

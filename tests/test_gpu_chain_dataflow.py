"""Decode chain, dataflow form (opc_chain_create_ex with OPC_CHAIN_FORM_DATAFLOW, batch 1):
steps exchange fixed-point digits whose scale is fixed in advance from a norm bound, staged per
128-column block.  Checked against the oracle's fp64 chain (the reference's dequantize-then-matmul,
opacc1ty/export/converter.py:26-67, rounded to fp16 between steps), against the barrier form
within the GEMV tolerance, for determinism over repeated launches and CUDA-graph replay, and at
the benchmark's Llama-3.1-8B shapes."""

import ctypes

import numpy as np
import pytest
import torch

from oracle import oracle
from opac1ty_b200 import _lib
from opac1ty_b200 import decode as D
from opac1ty_b200 import layer as L
from opac1ty_b200 import synthetic
from opac1ty_b200.chain import Chain

from test_gpu_chain import CFGS, _blocks, _oracle_chain

pytestmark = pytest.mark.gpu

REL_TOL = 2e-3


def _device_error():
    code = ctypes.c_int32(-1)
    _lib.check(_lib.load().opc_take_device_error(0, ctypes.byref(code)))
    return code.value


def _run(bds, cfg, x, dev, form, launches=1):
    st = D.DecodeStack.from_block_dicts(bds, cfg["hidden"], cfg["intermediate"], cfg["kv"], dev, batch=1,
                                        chain_form=form)
    assert st.chain is not None and st.chain.form == form
    outs = []
    for _ in range(launches):
        st.bufs["x"].copy_(torch.from_numpy(x))
        y = st.step_eager().clone()
        outs.append((y, {k: v.clone() for k, v in st.bufs.items()}))
    torch.cuda.synchronize()
    return outs


@pytest.mark.parametrize("cfg", CFGS)
def test_dataflow_against_oracle_and_barrier_form(cuda_device, cfg):
    bds = _blocks(cfg, seed=3)
    x = synthetic.activations(1, cfg["hidden"], seed=22)
    (yd, idf), = _run(bds, cfg, x, cuda_device, "dataflow")
    (yb, ib), = _run(bds, cfg, x, cuda_device, "barrier")
    assert _device_error() == 0
    y64 = _oracle_chain(x, bds, cfg)
    assert oracle.rel_err(yd.cpu().numpy(), y64) <= 5e-3
    # every intermediate output agrees with the barrier form within the GEMV tolerance
    for k in idf:
        a, b = idf[k].double().cpu().numpy(), ib[k].double().cpu().numpy()
        assert oracle.rel_err(a, b) <= REL_TOL, k


def test_dataflow_repeated_launches_and_graph_are_identical(cuda_device):
    cfg = CFGS[0]
    bds = _blocks(cfg, seed=8)
    x = synthetic.activations(1, cfg["hidden"], seed=5)
    outs = _run(bds, cfg, x, cuda_device, "dataflow", launches=5)
    for y, _ in outs[1:]:
        assert torch.equal(y, outs[0][0])
    st = D.DecodeStack.from_block_dicts(bds, cfg["hidden"], cfg["intermediate"], cfg["kv"], cuda_device,
                                        chain_form="dataflow")
    xt = torch.from_numpy(x).to(cuda_device)
    st.bufs["x"].copy_(xt)
    st.step_eager()
    st.capture()
    for _ in range(3):
        st.bufs["x"].copy_(xt)
        y = st.step().clone()
        torch.cuda.synchronize()
        assert torch.equal(y, outs[0][0])
    assert _device_error() == 0


@pytest.mark.parametrize("M,K", [(256, 1024), (1000, 4096), (512, 14336)])
def test_dataflow_single_step_against_fp64(cuda_device, M, K):
    layer = synthetic.random_layer(M, K, max(1, M // 100), seed=M ^ K, shuffle_ids=True)
    dl = L.prepare_layer(layer, cuda_device)
    x = torch.from_numpy(synthetic.activations(1, K, seed=K)).to(cuda_device)
    y = torch.zeros(1, M, dtype=torch.float16, device=cuda_device)
    ch = Chain([(dl, x, y)], form="dataflow")
    for _ in range(2):
        ch.launch()
        torch.cuda.synchronize()
        y64 = oracle.gemv_f64(oracle.dequantize_np(layer), x.cpu().numpy())
        assert oracle.rel_err(y.cpu().numpy(), y64) <= REL_TOL
    ch.close()


def test_dataflow_at_llama8b_shapes(cuda_device):
    cfg = dict(synthetic.LLAMA_8B, layers=2)
    bds = _blocks(cfg, seed=300)
    x = synthetic.activations(1, cfg["hidden"], seed=41)
    (yd, idf), = _run(bds, cfg, x, cuda_device, "dataflow")
    (yb, ib), = _run(bds, cfg, x, cuda_device, "barrier")
    y64 = _oracle_chain(x, bds, cfg)
    assert oracle.rel_err(yd.cpu().numpy(), y64) <= 5e-3
    for k in idf:
        assert oracle.rel_err(idf[k].double().cpu().numpy(), ib[k].double().cpu().numpy()) <= REL_TOL, k
    assert _device_error() == 0


def test_dataflow_trace_and_rejections(cuda_device):
    cfg = CFGS[0]
    bds = _blocks(cfg, seed=9)
    st = D.DecodeStack.from_block_dicts(bds, cfg["hidden"], cfg["intermediate"], cfg["kv"], cuda_device,
                                        chain_form="dataflow")
    tr = st.chain.enable_trace()
    st.step_eager()
    torch.cuda.synchronize()
    t = tr.cpu().numpy()
    assert (t[:, :, 2] > 0).all() and (t[:, :, 3] >= t[:, :, 2]).all()   # consumer stamps every step
    assert (t[1:, :, 1] > 0).all()                                           # staging stamps, steps >= 1
    st.chain.disable_trace()
    # batch 2 is the barrier form's
    a = L.prepare_layer(synthetic.random_layer(64, 64, 1, seed=1), cuda_device)
    x2 = torch.zeros(2, 64, dtype=torch.float16, device=cuda_device)
    y2 = torch.zeros(2, 64, dtype=torch.float16, device=cuda_device)
    with pytest.raises(_lib.OpcError) as e:
        Chain([(a, x2, y2)], form="dataflow")
    assert e.value.code == _lib.OPC_ERR_UNSUPPORTED
    assert Chain([(a, x2, y2)]).form == "barrier"


def test_dataflow_overflowing_output_is_reported(cuda_device):
    # outputs beyond the fp16 range become infinite; the next step cannot take them as digits, so
    # the kernel clamps them and records device error 5 (the per-launch path gives inf likewise)
    M = K = 256
    layer = synthetic.random_layer(M, K, 0, seed=4)
    layer["codebooks"] = torch.full((M, 4, 1), 60.0, dtype=torch.float16)
    a = L.prepare_layer(layer, cuda_device)
    b = L.prepare_layer(synthetic.random_layer(M, K, 0, seed=5), cuda_device)
    x = torch.full((1, K), 100.0, dtype=torch.float16, device=cuda_device)
    y1 = torch.zeros(1, M, dtype=torch.float16, device=cuda_device)
    y2 = torch.zeros(1, M, dtype=torch.float16, device=cuda_device)
    assert _device_error() == 0
    ch = Chain([(a, x, y1), (b, y1, y2)], form="dataflow")
    ch.launch()
    torch.cuda.synchronize()
    assert torch.isinf(y1).all()
    assert _device_error() == 5
    ch.close()

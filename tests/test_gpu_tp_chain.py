"""Row-sharded decode chain (opc_chain_create_tp) on ONE GPU.

* world = 1 through the sharded API (CUDA IPC region, info exchange, create) equals the one-GPU
  chain bit for bit.
* Failure detection without a GPU fault: rank 0 of a 2-rank chain is launched alone; rank 1's
  region is a second local buffer that no kernel writes, so rank 0's first cross-rank wait runs
  out (bounded, 2 s).  The launch records device error 3 and poisons the chain; the next launch
  records error 4 and does nothing.  Only one kernel ever runs: no two waiting kernels share the
  GPU.

The 2-GPU form (one process per GPU) is in test_gpu_tp.py.
"""

import ctypes

import pytest
import torch

from opac1ty_b200 import _lib
from opac1ty_b200 import decode as D
from opac1ty_b200 import synthetic
from opac1ty_b200 import tp

CFGS = [
    {"hidden": 512, "intermediate": 1024, "kv": 128, "layers": 2},
    {"hidden": 200, "intermediate": 328, "kv": 40, "layers": 2},   # ragged: tiles and k blocks cut
]


def _blocks(cfg, seed=0):
    shapes = synthetic.decoder_shapes(cfg)
    out = []
    for li in range(cfg["layers"]):
        out.append({name: synthetic.random_layer(M, K, synthetic.n_outliers_for(M, 0.02), seed=seed + 50 * li + pi,
                                                 shuffle_ids=True)
                    for pi, (name, (M, K)) in enumerate(shapes.items())})
    return out


def _fused(bd):
    return {"qkv": D.concat_rows([bd["q_proj"], bd["k_proj"], bd["v_proj"]]), "o": bd["o_proj"],
            "gate_up": D.concat_rows([bd["gate_proj"], bd["up_proj"]]), "down": bd["down_proj"]}


def _take_error():
    code = ctypes.c_int32(-1)
    _lib.check(_lib.load().opc_take_device_error(torch.cuda.current_device(), ctypes.byref(code)))
    return code.value


@pytest.mark.gpu
@pytest.mark.parametrize("cfg", CFGS)
@pytest.mark.parametrize("batch", [1, 2])
def test_tp_chain_world1_equals_chain(cuda_device, cfg, batch):
    bds = _blocks(cfg, seed=3)
    x = torch.from_numpy(synthetic.activations(batch, cfg["hidden"], seed=8)).to(cuda_device)
    ref = D.DecodeStack.from_block_dicts(bds, cfg["hidden"], cfg["intermediate"], cfg["kv"], cuda_device, batch=batch)
    assert ref.chain is not None
    st = tp.TPDecodeStack.from_fused_blocks([_fused(bd) for bd in bds], cfg, 0, 1, cuda_device, batch)
    st.enable_chain(all_gather_obj=lambda o: [o], barrier=lambda: None)
    ref.bufs["x"].copy_(x)
    st.bufs["x"].copy_(x)
    for _ in range(3):  # chained steps: epochs advance, flags are never cleared
        yr = ref.step_eager().clone()
        yt = st.step_eager().clone()
        torch.cuda.synchronize()
        assert torch.equal(yr, yt)
    # every intermediate output equals the one-GPU chain's buffer of the same step
    want = [ref.bufs["qkv"], ref.bufs["o"], ref.bufs["gu"], ref.bufs["x"]]
    for a, b in zip(st.chain.outputs[-4:], want):
        assert torch.equal(a, b[:, :a.shape[1]])
    assert _take_error() == 0
    st.close()


@pytest.mark.gpu
def test_tp_chain_graph_replay(cuda_device):
    cfg = CFGS[0]
    bds = _blocks(cfg, seed=11)
    st = tp.TPDecodeStack.from_fused_blocks([_fused(bd) for bd in bds], cfg, 0, 1, cuda_device, 1)
    st.enable_chain(all_gather_obj=lambda o: [o], barrier=lambda: None)
    x = torch.from_numpy(synthetic.activations(1, cfg["hidden"], seed=2)).to(cuda_device)
    st.bufs["x"].copy_(x)
    y1 = st.step_eager().clone()
    y2 = st.step_eager().clone()
    st.bufs["x"].copy_(x)
    st.capture()
    st.bufs["x"].copy_(x)
    st.step()
    g1 = st.bufs["x"].clone()
    st.step()
    g2 = st.bufs["x"].clone()
    torch.cuda.synchronize()
    assert torch.equal(g1, y1) and torch.equal(g2, y2)
    assert _take_error() == 0
    st.close()


def _rank_region(stack, batch, world, arr):
    """Fill `arr` with a rank's steps (x of step 0 = the last step's output, as TPChain does)
    inside a freshly allocated region; returns (region pointer, its bytes, scratch offset)."""
    lib = _lib.load()
    projs = [blk[name] for blk in stack.blocks for name in tp.PROJ_ORDER]
    n = len(projs)
    _, lds, _, _ = tp.chain_region_layout([p.M for p in projs], batch, 0)
    for j, p in enumerate(projs):
        arr[j].layer = ctypes.pointer(p.layer.c_layer)
        arr[j].ldy = lds[j]
    scratch = ctypes.c_size_t(0)
    _lib.check(lib.opc_chain_tp_scratch_bytes(arr, n, batch, world, ctypes.byref(scratch)))
    offs, lds, soff, total = tp.chain_region_layout([p.M for p in projs], batch, scratch.value)
    ptr = ctypes.c_void_p()
    handle = (ctypes.c_ubyte * _lib.OPC_PEER_HANDLE_BYTES)()
    _lib.check(lib.opc_peer_alloc(total, ctypes.byref(ptr), handle))
    for j in range(n):
        arr[j].y = ptr.value + offs[j]
        arr[j].x = ptr.value + offs[j - 1]
        arr[j].ldx = lds[j - 1]
    return ptr, total, soff


def _info(arr, n, batch, world, ptr, total, soff):
    lib = _lib.load()
    need = ctypes.c_size_t(0)
    _lib.check(lib.opc_chain_tp_info(arr, n, batch, world, ptr.value, total, soff, None, ctypes.byref(need)))
    info = (ctypes.c_ubyte * need.value)()
    _lib.check(lib.opc_chain_tp_info(arr, n, batch, world, ptr.value, total, soff, info, ctypes.byref(need)))
    return info


@pytest.mark.gpu
def test_tp_chain_barrier_times_out_without_peer(cuda_device):
    cfg = CFGS[0]
    world, batch = 2, 1
    fused = [_fused(bd) for bd in _blocks(cfg, seed=5)[:1]]
    stacks = [tp.TPDecodeStack.from_fused_blocks(fused, cfg, r, world, cuda_device, batch) for r in range(world)]
    lib = _lib.load()
    n = 4
    regions, infos, keep = [], [], []
    try:
        for r in range(world):
            arr = (_lib.ChainStep * n)()
            ptr, total, soff = _rank_region(stacks[r], batch, world, arr)
            regions.append(ptr)
            infos.append(_info(arr, n, batch, world, ptr, total, soff))
            keep.append(arr)
        assert _take_error() == 0
        rptrs = (ctypes.c_void_p * world)(*[p.value for p in regions])
        iptrs = (ctypes.c_void_p * world)(*[ctypes.addressof(i) for i in infos])
        h = ctypes.c_void_p()
        _lib.check(lib.opc_chain_create_tp(keep[0], n, batch, 0, world, rptrs, iptrs, ctypes.byref(h)))
        try:
            stream = torch.cuda.current_stream(cuda_device).cuda_stream
            _lib.check(lib.opc_chain_launch(h, stream))
            torch.cuda.synchronize()
            assert _take_error() == 3          # cross-rank barrier gave up
            _lib.check(lib.opc_chain_launch(h, stream))
            torch.cuda.synchronize()
            assert _take_error() == 4          # poisoned: refused without work
        finally:
            lib.opc_chain_destroy(h)
    finally:
        for p in regions:
            lib.opc_peer_free(p)


@pytest.mark.gpu
def test_tp_chain_create_rejects_mismatched_infos(cuda_device):
    cfg = CFGS[0]
    world, batch = 2, 1
    fused = [_fused(bd) for bd in _blocks(cfg, seed=6)[:1]]
    stacks = [tp.TPDecodeStack.from_fused_blocks(fused, cfg, r, world, cuda_device, batch) for r in range(world)]
    lib = _lib.load()
    n = 4
    arr = (_lib.ChainStep * n)()
    ptr, total, soff = _rank_region(stacks[0], batch, world, arr)
    try:
        info = _info(arr, n, batch, world, ptr, total, soff)
        # rank 1 claiming batch 2 (byte 16 of the header) must be rejected
        bad = (ctypes.c_ubyte * len(info)).from_buffer_copy(bytes(info))
        ctypes.c_int32.from_buffer(bad, 16).value = 2
        rptrs = (ctypes.c_void_p * world)(ptr.value, ptr.value)
        iptrs = (ctypes.c_void_p * world)(ctypes.addressof(info), ctypes.addressof(bad))
        h = ctypes.c_void_p()
        rc = lib.opc_chain_create_tp(arr, n, batch, 0, world, rptrs, iptrs, ctypes.byref(h))
        assert rc == _lib.OPC_ERR_INVALID and not h.value
        # y outside the region is rejected when describing the shard
        arr[1].y = ptr.value + total + 64
        need = ctypes.c_size_t(len(info))
        rc = lib.opc_chain_tp_info(arr, n, batch, world, ptr.value, total, soff, info, ctypes.byref(need))
        assert rc == _lib.OPC_ERR_INVALID
    finally:
        lib.opc_peer_free(ptr)

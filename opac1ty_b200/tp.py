"""Output-channel (row) tensor parallelism of the decode chain over NCCL.

Every projection matrix is split by output rows into ``world`` contiguous shards: codebooks,
indices and outlier rows are all per output row, so a shard is an ordinary quantized layer of
``rows`` x K (outlier ids falling in the shard, remapped to local ids) and nothing is
replicated.  Each rank computes its slice of y from the full x, then an all-gather over NVLink
restores the full y for the next GEMV:

    qkv_local = W_qkv[shard] . x          -> all_gather -> qkv
    o_local   = W_o[shard]   . q          -> all_gather -> o
    gu_local  = W_gu[shard]  . o          -> all_gather -> gate|up
    x_local   = W_down[shard]. gate       -> all_gather -> x

Shards are multiples of 16 rows (one row tile) and all ranks use the same shard size, so
``all_gather_into_tensor`` concatenates them in rank order; the last rank's shard may be
shorter, its padding lies past row M and is never read.

The chain logic (``tp_chain_step``) takes the GEMV and the all-gather as callables, so the same
code runs with the CUDA library and NCCL on GPUs and with a CPU GEMV and gloo in the tests.
That per-projection GEMV + all-gather form is the baseline.

``TPChain`` runs the same sharded step (batch 1..2) as ONE persistent kernel per rank
(``opc_chain_create_tp``): every rank stores its output rows straight into every rank's copy of
the full activations through CUDA IPC peer pointers, as tagged words that the next projection's
readers poll, so there is neither an all-gather, nor a launch, nor a barrier per projection.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass, field
from typing import Callable, Dict, List, Optional, Sequence, Tuple

import torch

from . import _lib
from . import decode as D
from . import layer as L
from . import synthetic

ROW_ALIGN = 16


def shard_rows_count(M: int, world: int, align: int = ROW_ALIGN) -> int:
    """Rows per shard: ceil(M / world) rounded up to ``align``."""
    per = -(-M // world)
    return -(-per // align) * align


def shard_bounds(M: int, world: int, align: int = ROW_ALIGN) -> List[Tuple[int, int]]:
    """[r0, r1) of every rank's shard (rank i owns rows i*S .. min((i+1)*S, M))."""
    S = shard_rows_count(M, world, align)
    return [(min(i * S, M), min((i + 1) * S, M)) for i in range(world)]


def shard_layer(layer: dict, r0: int, r1: int) -> dict:
    """Rows [r0, r1) of a reference "quantized" layer dict (opacc1ty/quantize/vq.py:191-200
    layout): codebooks and indices sliced, outlier rows whose id lies in the shard kept with
    ids shifted to local numbering (a repeated id keeps its order, so the last one still wins)."""
    M, K = (int(v) for v in layer["shape"])
    if not (0 <= r0 <= r1 <= M):
        raise ValueError(f"shard_layer: bad row range [{r0}, {r1}) for M={M}")
    out = {
        "type": "quantized",
        "shape": (r1 - r0, K),
        "codebooks": layer["codebooks"][r0:r1],
        "indices": layer["indices"][r0:r1],
        "outlier_values": None,
        "outlier_indices": None,
    }
    oi = layer.get("outlier_indices")
    ov = layer.get("outlier_values")
    if oi is not None and ov is not None and len(oi):
        ids = torch.as_tensor(oi).to(torch.int64).cpu()
        keep = (ids >= r0) & (ids < r1)
        if bool(keep.any()):
            sel = torch.nonzero(keep).flatten()
            out["outlier_indices"] = ids[sel] - r0
            out["outlier_values"] = torch.as_tensor(ov)[sel.to(torch.as_tensor(ov).device)]
    return out


def gathered_view(gathered: torch.Tensor, world: int, batch: int, S: int, M: int) -> torch.Tensor:
    """Full [batch, M] activations from an all-gather output laid out [world][batch][S]."""
    g = gathered.view(world, batch, S)
    if batch == 1:
        return g.view(1, world * S)[:, :M]
    return g.permute(1, 0, 2).reshape(batch, world * S)[:, :M]


@dataclass
class ShardedProj:
    """One projection's local shard plus its buffers: y_local [batch, S], gathered [world*batch*S]."""

    layer: object          # DeviceLayer on GPU, or a layer dict for CPU GEMVs; None if empty
    M: int                 # full output rows
    S: int                 # rows per shard (all ranks)
    rows: int              # rows of this rank's shard (<= S; the last shard may be shorter)
    y_local: torch.Tensor
    gathered: torch.Tensor


def tp_chain_step(x: torch.Tensor, blocks: Sequence[Dict[str, ShardedProj]], hidden: int, intermediate: int,
                  world: int, gemv: Callable, all_gather: Callable) -> torch.Tensor:
    """One decode step of the row-sharded chain.  ``gemv(layer, x, out)`` writes out = x . W^T,
    ``all_gather(out_tensor, in_tensor)`` gathers shards in rank order.  Returns the full x."""
    batch = x.shape[0]
    cur = x
    for blk in blocks:
        for name in ("qkv", "o", "gate_up", "down"):
            p = blk[name]
            if name == "o":
                inp = cur[:, :hidden]
            elif name == "down":
                inp = cur[:, :intermediate]
            else:
                inp = cur
            if inp.stride(1) != 1 or (batch > 1 and not inp.is_contiguous()):
                inp = inp.contiguous()
            if p.rows > 0:
                gemv(p.layer, inp, p.y_local[:, :p.rows])
            all_gather(p.gathered, p.y_local)
            cur = gathered_view(p.gathered, world, batch, p.S, p.M)
    return cur


def _alloc_proj(layer, M: int, rows: int, world: int, batch: int, device) -> ShardedProj:
    S = shard_rows_count(M, world)
    y = torch.zeros(batch, S, dtype=torch.float16, device=device)
    g = torch.zeros(world * batch * S, dtype=torch.float16, device=device)
    return ShardedProj(layer if rows > 0 else None, M, S, rows, y, g)


@dataclass
class TPDecodeStack:
    """This rank's shards of every decoder block (DeviceLayers) plus the chain buffers."""

    blocks: List[Dict[str, ShardedProj]]
    hidden: int
    intermediate: int
    kv: int
    rank: int
    world: int
    device: torch.device
    batch: int = 1
    group: object = None
    graph: Optional[torch.cuda.CUDAGraph] = None
    bufs: Dict[str, torch.Tensor] = field(default_factory=dict)
    chain: object = None   # TPChain once enable_chain() ran: one kernel per step, no all-gathers

    @staticmethod
    def _shard_block(fused: Dict[str, dict], rank: int, world: int, batch: int, device) -> Dict[str, ShardedProj]:
        blk = {}
        for name in ("qkv", "o", "gate_up", "down"):
            ly = fused[name]
            M = int(ly["shape"][0])
            r0, r1 = shard_bounds(M, world)[rank]
            dl = L.prepare_layer(shard_layer(ly, r0, r1), device, name) if r1 > r0 else None
            blk[name] = _alloc_proj(dl, M, r1 - r0, world, batch, device)
        return blk

    @classmethod
    def from_fused_blocks(cls, fused_blocks: Sequence[Dict[str, dict]], cfg: dict, rank: int, world: int,
                          device=None, batch: int = 1, group=None) -> "TPDecodeStack":
        """Shard reference layer dicts of fused blocks ({"qkv", "o", "gate_up", "down"}, built
        with ``decode.concat_rows``) and keep this rank's shards on ``device``."""
        device = L._as_cuda_device(device)
        blocks = [cls._shard_block(fb, rank, world, batch, device) for fb in fused_blocks]
        st = cls(blocks, cfg["hidden"], cfg["intermediate"], cfg["kv"], rank, world, device, batch, group)
        st._alloc()
        return st

    @classmethod
    def synthetic(cls, cfg: dict, rank: int, world: int, n_layers: Optional[int] = None, device=None,
                  batch: int = 1, outlier_fraction: float = 0.01, seed: int = 0, group=None) -> "TPDecodeStack":
        """Same seeded weights as ``DecodeStack.synthetic`` (every rank generates each full
        layer on its device and keeps its own row shard)."""
        shapes = synthetic.decoder_shapes(cfg)
        n_layers = cfg["layers"] if n_layers is None else n_layers
        device = L._as_cuda_device(device)
        blocks = []
        for li in range(n_layers):
            bd = {}
            for pi, (name, (M, K)) in enumerate(shapes.items()):
                n_out = synthetic.n_outliers_for(M, outlier_fraction)
                bd[name] = synthetic.random_layer_device(M, K, n_out, seed=seed + 1000 * li + pi, device=device)
            fused = {
                "qkv": D.concat_rows([bd["q_proj"], bd["k_proj"], bd["v_proj"]]),
                "o": bd["o_proj"],
                "gate_up": D.concat_rows([bd["gate_proj"], bd["up_proj"]]),
                "down": bd["down_proj"],
            }
            del bd
            blocks.append(cls._shard_block(fused, rank, world, batch, device))
            del fused
        st = cls(blocks, cfg["hidden"], cfg["intermediate"], cfg["kv"], rank, world, device, batch, group)
        st._alloc()
        return st

    def _alloc(self):
        self.bufs = {"x": torch.zeros(self.batch, self.hidden, dtype=torch.float16, device=self.device)}
        need = max([L.workspace_bytes(dl, self.batch) for dl in self.layers()] + [1])
        self.workspace = torch.zeros(need, dtype=torch.uint8, device=self.device)

    def layers(self) -> List[L.DeviceLayer]:
        return [p.layer for b in self.blocks for p in b.values() if p.layer is not None]

    def algorithmic_bytes(self) -> int:
        """This rank's GEMV bytes per step (its shards; x is read in full by every rank)."""
        return sum(dl.algorithmic_bytes(self.batch) for dl in self.layers())

    def launches_per_step(self) -> int:
        return 1 if self.chain is not None else 4 * len(self.blocks)

    def kernel_name(self) -> str:
        """The kernel that runs the step (fused chain, or one GEMV launch per projection)."""
        if self.chain is not None:
            return "opc::chain_kernel"
        return "opc::gemvq_kernel" if self.batch <= 2 else "opc::gemv_kernel"

    def enable_chain(self, **kw) -> "TPChain":
        """Collective: run every step as one fused kernel per rank (TPChain, batch 1..2);
        bufs["x"] becomes the chain's input/output buffer (current contents carried over)."""
        ch = TPChain(self, **kw)
        ch.x.copy_(self.bufs["x"])
        self.chain = ch
        self.bufs["x"] = ch.x
        self.graph = None
        return ch

    def close(self):
        """Collective: release the fused chain (if any) before the process group goes away."""
        self.graph = None
        if self.chain is not None:
            x = self.bufs["x"].clone()
            self.chain.close()
            self.chain = None
            self.bufs["x"] = x

    def _gemv(self, dl, x, out):
        L.gemv(dl, x, out=out, workspace=self.workspace)

    def _all_gather(self, out, inp):
        import torch.distributed as dist

        dist.all_gather_into_tensor(out, inp.reshape(-1), group=self.group)

    def step_eager(self):
        if self.chain is not None:
            self.chain.launch()
            return self.bufs["x"]
        x = tp_chain_step(self.bufs["x"], self.blocks, self.hidden, self.intermediate, self.world,
                          self._gemv, self._all_gather)
        self.bufs["x"].copy_(x)
        return self.bufs["x"]

    def capture(self) -> torch.cuda.CUDAGraph:
        g = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream(self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(s):
            self.step_eager()
        torch.cuda.current_stream(self.device).wait_stream(s)
        with torch.cuda.graph(g):
            self.step_eager()
        self.graph = g
        return g

    def step(self):
        if self.graph is None:
            return self.step_eager()
        self.graph.replay()
        return self.bufs["x"]


# ---------------------------------------------------------------------------------------------
# The same row-sharded step as ONE persistent kernel per rank (opc_chain_create_tp): each rank
# stores its rows of every projection straight into every rank's copy of the full output over
# NVLink (tagged words the readers poll), so the step has no all-gather launch and no NCCL call.
# ---------------------------------------------------------------------------------------------

PROJ_ORDER = ("qkv", "o", "gate_up", "down")


class _DevicePtr:
    """A device pointer as seen by ``torch.as_tensor`` (CUDA array interface, no ownership)."""

    def __init__(self, ptr: int, shape, typestr: str = "<f2"):
        self.__cuda_array_interface__ = {"shape": tuple(int(s) for s in shape), "typestr": typestr,
                                         "data": (int(ptr), False), "version": 2}


def device_view(ptr: int, shape, device) -> torch.Tensor:
    """fp16 tensor of ``shape`` over device memory at ``ptr`` (not owned: keep the memory alive)."""
    t = torch.as_tensor(_DevicePtr(ptr, shape), device=device)
    if t.data_ptr() != int(ptr) or t.dtype != torch.float16:
        raise RuntimeError("device_view: torch did not map the pointer as fp16")
    return t


def chain_region_layout(rows: Sequence[int], batch: int, scratch_bytes: int,
                        align: int = 256) -> Tuple[List[int], List[int], int, int]:
    """Layout of one rank's peer-visible region for a row-sharded chain: step j's full output
    [batch][ld_j] fp16 (ld_j = rows rounded up to 8 halves, 16-byte rows) at offsets[j], then the
    chain scratch.  Returns (offsets, lds, scratch_offset, total_bytes); every offset is a
    multiple of ``align``.  Identical on every rank (it depends on the full row counts only)."""
    if batch < 1 or scratch_bytes < 0 or align < 16 or align % 16:
        raise ValueError("chain_region_layout: bad arguments")

    def up(v: int) -> int:
        return -(-v // align) * align

    offsets, lds, off = [], [], 0
    for m in rows:
        if m < 1:
            raise ValueError(f"chain_region_layout: step with {m} rows")
        ld = -(-int(m) // 8) * 8
        offsets.append(off)
        lds.append(ld)
        off = up(off + 2 * batch * ld)
    scratch_offset = off
    return offsets, lds, scratch_offset, up(scratch_offset + scratch_bytes)


class PeerRegion:
    """``nbytes`` of device memory on this rank, mapped into every rank's process by CUDA IPC
    (opc_peer_alloc / opc_peer_open).  ``bases[p]`` is rank p's region as seen here."""

    def __init__(self, nbytes: int, rank: int, world: int, all_gather_obj: Callable, device):
        lib = _lib.load()
        self.device = device
        self.nbytes = int(nbytes)
        self.rank = rank
        self.local = ctypes.c_void_p()
        self._opened: List[ctypes.c_void_p] = []
        handle = (ctypes.c_ubyte * _lib.OPC_PEER_HANDLE_BYTES)()
        with torch.cuda.device(device):
            _lib.check(lib.opc_peer_alloc(self.nbytes, ctypes.byref(self.local), handle))
        try:
            handles = all_gather_obj(bytes(handle))
            if len(handles) != world:
                raise RuntimeError(f"PeerRegion: {len(handles)} handles for world {world}")
            self.bases: List[int] = []
            with torch.cuda.device(device):
                for p, h in enumerate(handles):
                    if p == rank:
                        self.bases.append(int(self.local.value))
                        continue
                    buf = (ctypes.c_ubyte * len(h)).from_buffer_copy(h)
                    ptr = ctypes.c_void_p()
                    _lib.check(lib.opc_peer_open(buf, ctypes.byref(ptr)))
                    self._opened.append(ptr)
                    self.bases.append(int(ptr.value))
        except Exception:
            self.close_peers()
            self.free()
            raise

    def close_peers(self):
        lib = _lib.load()
        with torch.cuda.device(self.device):
            for ptr in self._opened:
                lib.opc_peer_close(ptr)
        self._opened = []

    def free(self):
        if self.local.value:
            with torch.cuda.device(self.device):
                _lib.load().opc_peer_free(self.local)
            self.local = ctypes.c_void_p()


class TPChain:
    """One decode step of a TPDecodeStack (batch 1..2) as one persistent kernel per rank.

    ``x`` is the step's input and output (this rank's copy of the last down projection's full
    output): write the initial activations into it on every rank, then call ``step()`` on every
    rank once per decode step.  Results equal ``TPDecodeStack.step_eager`` bit for bit.
    ``all_gather_obj(obj) -> [obj of rank 0, ...]`` and ``barrier()`` default to
    torch.distributed on the stack's group."""

    def __init__(self, stack: "TPDecodeStack", all_gather_obj: Optional[Callable] = None,
                 barrier: Optional[Callable] = None):
        import torch.distributed as dist

        if all_gather_obj is None:
            def all_gather_obj(obj):
                out = [None] * stack.world
                dist.all_gather_object(out, obj, group=stack.group)
                return out
        if barrier is None:
            def barrier():
                dist.barrier(group=stack.group)
        self._barrier = barrier
        self.stack = stack
        self.device = stack.device
        self.batch = stack.batch
        projs = [blk[name] for blk in stack.blocks for name in PROJ_ORDER]
        if any(p.layer is None for p in projs):
            raise ValueError("TPChain: every rank needs a non-empty shard of every projection")
        n = len(projs)
        lib = _lib.load()
        arr = (_lib.ChainStep * n)()
        rows = [p.M for p in projs]
        _, lds, _, _ = chain_region_layout(rows, self.batch, 0)
        for j, p in enumerate(projs):
            arr[j].layer = ctypes.pointer(p.layer.c_layer)
            arr[j].ldy = lds[j]
        scratch = ctypes.c_size_t(0)
        with torch.cuda.device(self.device):
            _lib.check(lib.opc_chain_tp_scratch_bytes(arr, n, self.batch, stack.world, ctypes.byref(scratch)))
        offs, lds, soff, total = chain_region_layout(rows, self.batch, scratch.value)
        self.region = PeerRegion(total, stack.rank, stack.world, all_gather_obj, self.device)
        self._handle = ctypes.c_void_p()
        try:
            base = self.region.bases[stack.rank]
            for j in range(n):
                arr[j].y = base + offs[j]
                arr[j].ldy = lds[j]
                arr[j].x = base + offs[j - 1]  # step 0 reads the last step's output
                arr[j].ldx = lds[j - 1]
            with torch.cuda.device(self.device):
                need = ctypes.c_size_t(0)
                _lib.check(lib.opc_chain_tp_info(arr, n, self.batch, stack.world, base, total, soff, None,
                                                 ctypes.byref(need)))
                info = (ctypes.c_ubyte * need.value)()
                _lib.check(lib.opc_chain_tp_info(arr, n, self.batch, stack.world, base, total, soff, info,
                                                 ctypes.byref(need)))
            infos = all_gather_obj(bytes(info))
            self._infos = [(ctypes.c_ubyte * len(b)).from_buffer_copy(b) for b in infos]
            info_ptrs = (ctypes.c_void_p * stack.world)(*[ctypes.addressof(b) for b in self._infos])
            regions = (ctypes.c_void_p * stack.world)(*self.region.bases)
            with torch.cuda.device(self.device):
                rc = lib.opc_chain_create_tp(arr, n, self.batch, stack.rank, stack.world, regions, info_ptrs,
                                             ctypes.byref(self._handle))
            # every rank learns every rank's outcome before anyone launches
            oks = all_gather_obj(rc == 0)
            _lib.check(rc)
            if not all(oks):
                raise RuntimeError("TPChain: opc_chain_create_tp failed on another rank")
            barrier()
        except Exception:
            self._destroy_chain()
            self.region.close_peers()
            self.region.free()
            raise
        self._steps = arr
        self.n_steps = n
        self.outputs = [device_view(base + offs[j], (self.batch, lds[j]), self.device)[:, :rows[j]] for j in range(n)]
        self.x = self.outputs[-1]

    def launch(self):
        stream = torch.cuda.current_stream(self.device).cuda_stream
        _lib.check(_lib.load().opc_chain_launch(self._handle, stream))

    def step(self) -> torch.Tensor:
        self.launch()
        return self.x

    def _destroy_chain(self):
        if self._handle.value:
            with torch.cuda.device(self.device):
                _lib.load().opc_chain_destroy(self._handle)
            self._handle = ctypes.c_void_p()

    def close(self):
        """Collective: every rank calls it.  Waits for the ranks' launches, then unmaps the peers
        and frees this rank's region once no rank maps it any more."""
        if self.region is None:
            return
        torch.cuda.synchronize(self.device)
        self._barrier()
        self._destroy_chain()
        self.region.close_peers()
        self._barrier()
        self.region.free()
        self.region = None
        self.outputs = []
        self.x = None

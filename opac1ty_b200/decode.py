"""Decode-step chain of fused 2-bit GEMVs at Llama shapes.

One decode step runs, for every decoder block, the projection chain the benchmark defines:

    qkv = W_qkv . x          (q, k, v fused row-wise into one launch)
    o   = W_o   . q          (q stands in for the attention output)
    gu  = W_gate|up . o      (gate and up fused row-wise)
    x'  = W_down . gate      (gate stands in for act(gate) * up)

Attention, norms, RoPE, the activation and residual adds are outside the measured path (they
are not part of opacc1ty's fused dequant path).  Each launch depends on the previous one, so a
step is 4 dependent GEMVs per block.  At batch 1..2 the whole step runs as ONE persistent
kernel (``opac1ty_b200.chain``: weights of every GEMV streamed without pause, each GEMV's
outputs published as tagged words that the next GEMV polls, no grid barrier); otherwise every
GEMV is its own launch, captured once into a CUDA graph, each carrying the programmatic-dependent-launch attribute so it starts streaming its
weights while its predecessor finishes.

``concat_rows`` builds the fused layers from per-projection reference layer dicts (codebooks,
indices and outlier rows stacked, outlier ids offset), which is exact: row r of the fused layer
is row r of one of the inputs.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Dict, List, Optional, Sequence

import torch

from . import _lib
from . import layer as L
from . import synthetic


def concat_rows(layers: Sequence[dict]) -> dict:
    """Stack reference layer dicts along the output dimension (all with the same K)."""
    K = int(layers[0]["shape"][1])
    cbs, idxs, ovs, ois = [], [], [], []
    off = 0
    for ly in layers:
        M, Ki = (int(v) for v in ly["shape"])
        if Ki != K:
            raise ValueError("concat_rows: in_features differ")
        cbs.append(torch.as_tensor(ly["codebooks"]))
        idxs.append(torch.as_tensor(ly["indices"]))
        if ly.get("outlier_values") is not None and ly.get("outlier_indices") is not None and len(ly["outlier_indices"]):
            ovs.append(torch.as_tensor(ly["outlier_values"]))
            ois.append(torch.as_tensor(ly["outlier_indices"]).to(torch.int64) + off)
        off += M
    out = {
        "type": "quantized",
        "shape": (off, K),
        "codebooks": torch.cat(cbs),
        "indices": torch.cat(idxs),
        "outlier_values": torch.cat(ovs) if ovs else None,
        "outlier_indices": torch.cat(ois) if ois else None,
    }
    return out


@dataclass
class Block:
    qkv: L.DeviceLayer
    o: L.DeviceLayer
    gate_up: L.DeviceLayer
    down: L.DeviceLayer

    def layers(self) -> List[L.DeviceLayer]:
        return [self.qkv, self.o, self.gate_up, self.down]


@dataclass
class DecodeStack:
    """Device-resident projection weights of ``n_layers`` decoder blocks plus activation buffers."""

    blocks: List[Block]
    hidden: int
    intermediate: int
    kv: int
    device: torch.device
    batch: int = 1
    graph: Optional[torch.cuda.CUDAGraph] = None
    bufs: Dict[str, torch.Tensor] = field(default_factory=dict)
    use_chain: bool = True
    chain: object = None
    chain_form: str = "auto"   # Chain form: "auto", "barrier" or "dataflow"

    @classmethod
    def from_block_dicts(cls, block_dicts: Sequence[Dict[str, dict]], hidden: int, intermediate: int, kv: int,
                         device, batch: int = 1, use_chain: bool = True, chain_form: str = "auto") -> "DecodeStack":
        device = L._as_cuda_device(device)
        blocks = []
        for bd in block_dicts:
            qkv = L.prepare_layer(concat_rows([bd["q_proj"], bd["k_proj"], bd["v_proj"]]), device, "qkv")
            o = L.prepare_layer(bd["o_proj"], device, "o_proj")
            gu = L.prepare_layer(concat_rows([bd["gate_proj"], bd["up_proj"]]), device, "gate_up")
            down = L.prepare_layer(bd["down_proj"], device, "down_proj")
            blocks.append(Block(qkv, o, gu, down))
        st = cls(blocks, hidden, intermediate, kv, device, batch, use_chain=use_chain, chain_form=chain_form)
        st._alloc()
        return st

    @classmethod
    def synthetic(cls, cfg: dict, n_layers: Optional[int] = None, device=None, batch: int = 1,
                  outlier_fraction: float = 0.01, seed: int = 0, use_chain: bool = True,
                  chain_form: str = "auto", sub_vector_size: int = 1) -> "DecodeStack":
        """Random-initialised 2-bit weights with the given model shapes (synthetic.random_layer;
        sub_vector_size 8: synthetic.random_layer_vq8, generated on the host)."""
        shapes = synthetic.decoder_shapes(cfg)
        n_layers = cfg["layers"] if n_layers is None else n_layers
        device = L._as_cuda_device(device)
        blocks = []
        for li in range(n_layers):
            bd = {}
            for pi, (name, (M, K)) in enumerate(shapes.items()):
                n_out = synthetic.n_outliers_for(M, outlier_fraction)
                if sub_vector_size == 8:
                    bd[name] = synthetic.random_layer_vq8(M, K, n_out, seed=seed + 1000 * li + pi)
                else:
                    bd[name] = synthetic.random_layer_device(M, K, n_out, seed=seed + 1000 * li + pi, device=device)
            qkv = L.prepare_layer(concat_rows([bd["q_proj"], bd["k_proj"], bd["v_proj"]]), device, "qkv")
            o = L.prepare_layer(bd["o_proj"], device, "o_proj")
            gu = L.prepare_layer(concat_rows([bd["gate_proj"], bd["up_proj"]]), device, "gate_up")
            down = L.prepare_layer(bd["down_proj"], device, "down_proj")
            del bd
            blocks.append(Block(qkv, o, gu, down))
        st = cls(blocks, cfg["hidden"], cfg["intermediate"], cfg["kv"], device, batch, use_chain=use_chain,
                 chain_form=chain_form)
        st._alloc()
        return st

    def _alloc(self):
        B, h, f, kv = self.batch, self.hidden, self.intermediate, self.kv
        dev = self.device
        self.bufs = {
            "x": torch.zeros(B, h, dtype=torch.float16, device=dev),
            "qkv": torch.zeros(B, h + 2 * kv, dtype=torch.float16, device=dev),
            "o": torch.zeros(B, h, dtype=torch.float16, device=dev),
            "gu": torch.zeros(B, 2 * f, dtype=torch.float16, device=dev),
        }
        need = max(L.workspace_bytes(dl, B) for b in self.blocks for dl in b.layers())
        self.workspace = torch.zeros(need, dtype=torch.uint8, device=dev)
        self.chain = None
        if self.use_chain and B <= 2:
            from .chain import Chain

            steps = []
            b = self.bufs
            for blk in self.blocks:
                steps += [(blk.qkv, b["x"], b["qkv"]), (blk.o, b["qkv"], b["o"]),
                          (blk.gate_up, b["o"], b["gu"]), (blk.down, b["gu"], b["x"])]
            try:
                self.chain = Chain(steps, form=self.chain_form)
            except _lib.OpcError:  # shape outside the chain kernel's limits: one launch per GEMV
                self.chain = None

    def layers(self) -> List[L.DeviceLayer]:
        return [dl for b in self.blocks for dl in b.layers()]

    def algorithmic_bytes(self) -> int:
        return sum(dl.algorithmic_bytes(self.batch) for dl in self.layers())

    def launches_per_step(self) -> int:
        return 1 if self.chain is not None else 4 * len(self.blocks)

    def kernel_name(self) -> str:
        """The kernel that runs the step."""
        if self.chain is not None:
            return "opc::chain2_kernel" if self.chain.form == "dataflow" else "opc::chain_kernel"
        if self.blocks and self.blocks[0].qkv.sub_vector_size == 8:
            return "opc::vq8_gemv_kernel"
        if self.batch > int(_lib.load().opc_gemm_crossover()):  # opc_gemv routes these to the GEMM
            return "opc::gemm_kernel"
        return "opc::gemvq_kernel" if self.batch <= 2 else "opc::gemv_kernel"

    def step_eager(self):
        """One decode step on the current stream; input and output in bufs["x"]."""
        if self.chain is not None:
            self.chain.launch()
            return self.bufs["x"]
        return self.step_launches()

    def step_launches(self):
        """The same step as one GEMV launch per projection."""
        b = self.bufs
        h, f = self.hidden, self.intermediate
        ws = self.workspace
        for blk in self.blocks:
            L.gemv(blk.qkv, b["x"], out=b["qkv"], workspace=ws)
            L.gemv(blk.o, b["qkv"][:, :h], out=b["o"], workspace=ws)
            L.gemv(blk.gate_up, b["o"], out=b["gu"], workspace=ws)
            L.gemv(blk.down, b["gu"][:, :f], out=b["x"], workspace=ws)
        return b["x"]

    def capture(self) -> torch.cuda.CUDAGraph:
        """Capture step_eager into a CUDA graph (call after one eager warm-up step)."""
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

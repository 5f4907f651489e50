"""Device-timed measurements of the fused 2-bit path at the benchmark configurations.

Every timing here replays a CUDA graph of repeated launches and reads CUDA events on the
launching stream, so the numbers are the GPU's and not the Python call rate; per-kernel timings
read a buffer twice the size of L2 before each launch (and subtract that read's time), so every
launch streams its weights from HBM.  The layers are
seeded synthetic ones (``synthetic.random_layer_device``) of the named shapes: kernel timing
does not depend on the weight values.

  prefill(cfg, tokens)        the tcgen05 GEMM on one decoder block's four projections
  decode(cfg, batch)          the whole decode step (every block's q|k|v, o, gate|up, down)
  outlier_batch_sweep(M, K)   one layer at outlier fractions x batches: GEMV and GEMM times and
                              the batch from which the GEMM is faster (the crossover)
"""

from __future__ import annotations

import contextlib
import time
from typing import Callable, Dict, List, Optional, Sequence

import torch

from . import _lib
from . import decode as D
from . import gemm as G
from . import layer as L
from . import synthetic


FLUSH_BYTES = 256 << 20  # twice the B200's 126 MB L2


def _graph_us(calls: Callable[[], None], device: torch.device, iters: int) -> float:
    g = torch.cuda.CUDAGraph()
    cs = torch.cuda.Stream(device)
    cur = torch.cuda.current_stream(device)
    cs.wait_stream(cur)
    with torch.cuda.stream(cs):
        calls()
    cur.wait_stream(cs)
    with torch.cuda.graph(g):
        for _ in range(iters):
            calls()
    g.replay()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(cur)
    g.replay()
    e1.record(cur)
    torch.cuda.synchronize(device)
    us = e0.elapsed_time(e1) * 1000.0 / iters
    del g
    return us


def graph_time_us(call: Callable[[], None], device: torch.device, iters: int = 20, flush_l2: bool = True) -> float:
    """Mean device time of ``call`` (µs): ``iters`` calls captured in one CUDA graph, replayed once
    to warm up and once timed with CUDA events on the current stream.  With ``flush_l2`` every
    call is preceded by a read of a buffer twice the size of L2 (so each call starts with its
    weights and inputs in HBM, not L2), and the time of the reads alone, measured the same way,
    is subtracted."""
    for _ in range(2):
        call()
    torch.cuda.synchronize(device)
    if not flush_l2:
        return _graph_us(call, device, iters)
    buf = torch.ones(FLUSH_BYTES // 4, dtype=torch.float32, device=device)
    acc = torch.empty((), dtype=torch.float32, device=device)

    def flush():
        torch.sum(buf, dim=0, out=acc)

    def flushed_call():
        flush()
        call()

    both = _graph_us(flushed_call, device, iters)
    alone = _graph_us(flush, device, iters)
    del buf
    return max(both - alone, 0.0)


@contextlib.contextmanager
def gemm_crossover(batch: int):
    """Temporarily route opc_gemv batches above ``batch`` to the GEMM (opc_set_gemm_crossover)."""
    lib = _lib.load()
    old = int(lib.opc_gemm_crossover())
    _lib.check(lib.opc_set_gemm_crossover(int(batch)))
    try:
        yield
    finally:
        lib.opc_set_gemm_crossover(old)


def block_projections(cfg: dict, device, seed: int = 0, outlier_fraction: float = 0.01) -> Dict[str, L.DeviceLayer]:
    """One decoder block's fused projections (q|k|v, o, gate|up, down) as device layers, with the
    seeds of block 0 of ``DecodeStack.synthetic``."""
    shapes = synthetic.decoder_shapes(cfg)
    bd = {}
    for pi, (name, (M, K)) in enumerate(shapes.items()):
        bd[name] = synthetic.random_layer_device(M, K, synthetic.n_outliers_for(M, outlier_fraction), seed=seed + pi,
                                                 device=device)
    return {
        "qkv": L.prepare_layer(D.concat_rows([bd["q_proj"], bd["k_proj"], bd["v_proj"]]), device, "qkv"),
        "o_proj": L.prepare_layer(bd["o_proj"], device, "o_proj"),
        "gate_up": L.prepare_layer(D.concat_rows([bd["gate_proj"], bd["up_proj"]]), device, "gate_up"),
        "down_proj": L.prepare_layer(bd["down_proj"], device, "down_proj"),
    }


def prefill(cfg: dict, device, tokens: Sequence[int] = (512, 2048), peak_tflops: Optional[float] = None,
            iters: int = 10) -> dict:
    """Prefill GEMM (opc_gemm) TFLOP/s on one block's projections at each token count.  FLOPs are
    the dense-equivalent 2 * tokens * M * K per projection; ``frac`` is against ``peak_tflops``."""
    projs = block_projections(cfg, device)
    rows: List[dict] = []
    for n_tok in tokens:
        tot_fl, tot_us = 0.0, 0.0
        for name, dl in projs.items():
            x = (torch.randn(n_tok, dl.K, device=device, generator=torch.Generator(device=device).manual_seed(n_tok))
                 .half())
            y = torch.empty(n_tok, dl.M, dtype=torch.float16, device=device)
            us = graph_time_us(lambda: G.gemm(dl, x, out=y), device, iters)
            fl = G.flops(dl, n_tok)
            tot_fl += fl
            tot_us += us
            r = {"layer": name, "shape": [dl.M, dl.K], "tokens": n_tok, "us": round(us, 2),
                 "tflops": round(fl / us / 1e6, 1)}
            if peak_tflops:
                r["frac"] = round(fl / us / 1e6 / peak_tflops, 4)
            rows.append(r)
        agg = {"layer": "block", "tokens": n_tok, "us": round(tot_us, 2), "tflops": round(tot_fl / tot_us / 1e6, 1)}
        if peak_tflops:
            agg["frac"] = round(tot_fl / tot_us / 1e6 / peak_tflops, 4)
        rows.append(agg)
    del projs
    torch.cuda.empty_cache()
    return {"kernel": "opc::gemm_kernel (tcgen05.mma kind::f16, TMEM accumulators)", "rows": rows,
            "flops": "2 * tokens * M * K per projection (dense-equivalent)"}


def decode(cfg: dict, device, batch: int = 1, n_blocks: Optional[int] = None, steps: int = 10,
           use_chain: bool = True) -> dict:
    """Decode tok/s of the whole step (every block) on synthetic weights, CUDA-graph replayed."""
    t0 = time.time()
    st = D.DecodeStack.synthetic(cfg, n_layers=n_blocks, device=device, batch=batch, use_chain=use_chain)
    build_s = time.time() - t0
    st.step_eager()
    torch.cuda.synchronize(device)
    st.capture()
    for _ in range(3):
        st.step()
    torch.cuda.synchronize(device)
    s = torch.cuda.current_stream(device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s)
    for _ in range(steps):
        st.step()
    e1.record(s)
    torch.cuda.synchronize(device)
    ms = e0.elapsed_time(e1) / steps
    nb = st.algorithmic_bytes()
    out = {"blocks": len(st.blocks), "batch": batch, "ms_per_step": round(ms, 4), "tok_s": round(batch * 1000.0 / ms, 2),
           "gbs": round(nb / (ms * 1e-3) / 1e9, 1), "algorithmic_bytes_per_step": nb,
           "launches_per_step": st.launches_per_step(), "kernel": st.kernel_name(), "build_s": round(build_s, 1)}
    st.graph = None
    del st
    torch.cuda.empty_cache()
    return out


def outlier_batch_sweep(M: int, K: int, device, fractions: Sequence[float] = (0.0, 0.01, 0.02),
                        batches: Sequence[int] = (1, 4, 8, 16, 64), iters: int = 20) -> dict:
    """One M x K layer at each outlier fraction: the GEMV (opc_gemv with the GEMM switched off)
    and the GEMM (opc_gemm) at each batch; bytes are the GEMV's algorithmic bytes.  ``crossover``
    is, per fraction, the smallest measured batch at which the GEMM is faster."""
    rows = []
    crossover = {}
    for frac in fractions:
        n_out = synthetic.n_outliers_for(M, frac)
        dl = L.prepare_layer(synthetic.random_layer_device(M, K, n_out, seed=11, device=device), device)
        for b in batches:
            x = torch.from_numpy(synthetic.activations(b, K, seed=b)).to(device)
            y = torch.empty(b, M, dtype=torch.float16, device=device)
            ws = torch.zeros(L.workspace_bytes(dl, b), dtype=torch.uint8, device=device)
            with gemm_crossover(64):
                gemv_us = graph_time_us(lambda: L.gemv(dl, x, out=y, workspace=ws), device, iters)
            gemm_us = graph_time_us(lambda: G.gemm(dl, x, out=y), device, iters)
            nb = dl.algorithmic_bytes(b)
            rows.append({"outliers": frac, "n_outlier_rows": n_out, "batch": b, "gemv_us": round(gemv_us, 2),
                         "gemv_gbs": round(nb / gemv_us / 1e3, 1), "gemm_us": round(gemm_us, 2),
                         "gemm_tflops": round(2.0 * b * M * K / gemm_us / 1e6, 2), "bytes": nb})
            if gemm_us < gemv_us and frac not in crossover:
                crossover[frac] = b
        del dl
    return {"shape": [M, K], "rows": rows,
            "crossover_batch": {str(f): crossover.get(f) for f in fractions},
            "gemv_kernel": "batch 1-2: opc::gemvq_kernel (integer); 3-64: opc::gemv_kernel (fp16)",
            "gemm_kernel": "opc::gemm_kernel (tcgen05)"}

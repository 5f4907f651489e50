"""Command-line entry points (the quantize / benchmark surface of opacc1ty/cli/main.py).

    python -m opac1ty_b200.cli quantize MODEL_PATH [-o out.bf2] [--sub-vector-size 1] ...
    python -m opac1ty_b200.cli info FILE.bf2 [--layers] [--json-output]
    python -m opac1ty_b200.cli benchmark FILE.bf2 [--batch 1] [--iters 50]
    python -m opac1ty_b200.cli layer-bench --shape 28672x4096 [--outliers 0.01] [--batch 1]

``benchmark`` replaces the reference's analytical estimate (cli/main.py:221-316) with CUDA-event
timing of the model's quantized layers on the GPU.  ``layer-bench`` times one synthetic layer
(the small case the kernel profiles are taken on).
"""

from __future__ import annotations

import json
import re
import sys
import time
from pathlib import Path

import click


@click.group()
@click.version_option(version="0.1.0", prog_name="opac1ty_b200")
def cli():
    """2-bit codebook quantization with fused sm_100a dequant-matmul kernels."""


def _load_state_dict(path: Path) -> dict:
    from safetensors import safe_open

    files = sorted(path.glob("*.safetensors")) if path.is_dir() else [path]
    sd = {}
    for f in files:
        with safe_open(str(f), framework="pt", device="cpu") as h:
            for k in h.keys():
                sd[k] = h.get_tensor(k)
    return sd


def _infer_model_config(sd: dict) -> dict:
    """Architecture hints from tensor names and shapes (cli/main.py:413-473, condensed)."""
    cfg = {"architecture": "unknown"}
    layers = {int(m.group(1)) for k in sd for m in [re.search(r"(?:layers?|h)\.(\d+)", k)] if m}
    if layers:
        cfg["num_hidden_layers"] = max(layers) + 1
    for k, t in sd.items():
        if t.dim() == 2 and t.shape[0] > 512:
            if "embed" in k.lower() or "wte" in k.lower():
                cfg["hidden_size"], cfg["vocab_size"] = int(t.shape[1]), int(t.shape[0])
            elif t.shape[0] == t.shape[1] and t.shape[0] > 1024:
                cfg.setdefault("hidden_size", int(t.shape[0]))
    for k, t in sd.items():
        if t.dim() == 2 and t.shape[0] > cfg.get("hidden_size", 1024) * 2:
            cfg["intermediate_size"] = int(t.shape[0])
            break
    if any("self_attn" in k for k in sd) and any("q_proj" in k for k in sd):
        cfg["architecture"] = "llama"
    if "hidden_size" in cfg:
        cfg.setdefault("num_attention_heads", cfg["hidden_size"] // 128)
    return cfg


@cli.command()
@click.argument("model_path", type=click.Path(exists=True))
@click.option("--bits", type=int, default=2)
@click.option("--output", "-o", type=click.Path(), default=None)
@click.option("--outlier-fraction", type=float, default=0.01)
@click.option("--outlier-mode", type=click.Choice(["row", "element"]), default="row",
              help="whole outlier rows (the reference's) or single weights kept as COO entries")
@click.option("--sub-vector-size", type=int, default=8)
@click.option("--codebook-iters", type=int, default=100)
@click.option("--no-error-feedback", is_flag=True)
@click.option("--device", type=click.Choice(["cpu", "cuda"]), default="cpu")
@click.option("--checksum", is_flag=True, help="end the file with its XXH64 checksum (flags bit 0)")
@click.option("--json-output", is_flag=True)
def quantize(model_path, bits, output, outlier_fraction, outlier_mode, sub_vector_size, codebook_iters, no_error_feedback, device,
             checksum, json_output):
    """Quantize a safetensors model (file or directory) to .bf2 (options of cli/main.py:64-80)."""
    from .format import BF2Writer
    from .quantize import QuantizeConfig, VectorQuantizer

    model_path = Path(model_path)
    out = Path(output) if output else Path(model_path.stem + ".bf2")
    sd = _load_state_dict(model_path)
    mcfg = _infer_model_config(sd)
    t0 = time.time()
    q = VectorQuantizer(QuantizeConfig(bits=bits, sub_vector_size=sub_vector_size, outlier_fraction=outlier_fraction,
                                       use_error_feedback=not no_error_feedback, codebook_iters=codebook_iters,
                                       device=device, outlier_mode=outlier_mode))
    res = q.quantize_model(sd, mcfg, progress=not json_output)
    elapsed = time.time() - t0
    BF2Writer(str(out)).write(res, mcfg, res["_quantize_config"], progress=not json_output, checksum=checksum)
    orig = sum(t.numel() for t in sd.values()) * 2 / 1e9
    comp = out.stat().st_size / 1e9
    info = {"original_size_gb": round(orig, 2), "compressed_size_gb": round(comp, 2),
            "compression_ratio": round(orig / comp, 1) if comp else None, "quantization_time_s": round(elapsed, 1),
            "output_path": str(out)}
    click.echo(json.dumps(info) if json_output else "\n".join(f"{k}: {v}" for k, v in info.items()))


@cli.command()
@click.argument("bf2_path", type=click.Path(exists=True))
@click.option("--layers", is_flag=True)
@click.option("--json-output", is_flag=True)
def info(bf2_path, layers, json_output):
    """Show a .bf2 file's metadata and layers."""
    from .format import BF2Reader

    with BF2Reader(bf2_path) as r:
        d = {"model": r.model_config, "quantization": r.quantize_config,
             "compressed_size_gb": round(Path(bf2_path).stat().st_size / 1e9, 3), "n_layers": len(r.layer_names()),
             "checksum": "verified" if r.checksum_ok else "absent",
             "layers": r.layer_names() if layers else None}
    click.echo(json.dumps(d, indent=2) if json_output else "\n".join(f"{k}: {v}" for k, v in d.items() if v is not None))


def _time_gemv(dl, batch: int, iters: int):
    """Device time (us) of one fused GEMV at ``batch``: CUDA-graph replays with L2 flushed before
    each launch (opac1ty_b200.measure.graph_time_us)."""
    import torch

    from . import layer as L, measure, synthetic

    x = torch.from_numpy(synthetic.activations(batch, dl.K, seed=1)).to(dl.device)
    y = torch.empty(batch, dl.M, dtype=torch.float16, device=dl.device)
    ws = torch.zeros(L.workspace_bytes(dl, batch), dtype=torch.uint8, device=dl.device)
    return measure.graph_time_us(lambda: L.gemv(dl, x, out=y, workspace=ws), dl.device, iters)


@cli.command()
@click.argument("bf2_path", type=click.Path(exists=True))
@click.option("--batch", type=int, default=1)
@click.option("--iters", type=int, default=50)
@click.option("--json-output", is_flag=True)
def benchmark(bf2_path, batch, iters, json_output):
    """Time every quantized (svs=1) layer of a .bf2 file on the GPU with CUDA events."""
    from . import layer as L
    from .format import BF2Reader
    from .utils import get_cuda_device_info

    gpu = get_cuda_device_info()
    if gpu is None:
        raise click.ClickException("no CUDA device")
    rows, total_us, total_bytes = [], 0.0, 0
    with BF2Reader(bf2_path) as r:
        for name in r.layer_names():
            ly = r.load_layer(name)
            if ly["type"] != "quantized" or ly["codebooks"].shape[2] != 1:
                continue
            dl = L.prepare_layer(ly, name=name)
            us = _time_gemv(dl, batch, iters)
            nb = dl.algorithmic_bytes(batch)
            rows.append({"layer": name, "shape": list(dl.shape), "us": round(us, 2), "gbs": round(nb / us / 1e3, 1)})
            total_us += us
            total_bytes += nb
    out = {"gpu": gpu.name, "batch": batch, "layers": rows, "total_us": round(total_us, 2),
           "tok_s": round(batch * 1e6 / total_us, 1) if total_us else None,
           "gbs": round(total_bytes / total_us / 1e3, 1) if total_us else None}
    click.echo(json.dumps(out, indent=None if json_output else 2))


@cli.command("layer-bench")
@click.option("--shape", default="28672x4096", help="MxK")
@click.option("--outliers", type=float, default=0.01, help="outlier row fraction (0 = none)")
@click.option("--batch", type=int, default=1)
@click.option("--iters", type=int, default=20)
@click.option("--svs", type=click.Choice(["1", "8"]), default="1", help="sub_vector_size of the synthetic layer")
@click.option("--op", type=click.Choice(["gemv", "dequant"]), default="gemv",
              help="gemv: the fused GEMV; dequant: write W_hat [M][K] fp16 (opc_dequant)")
def layer_bench(shape, outliers, batch, iters, svs, op):
    """Time one synthetic layer's fused GEMV or dequantization (CUDA events); prints one JSON line."""
    import torch

    from . import layer as L, measure, synthetic
    from .utils import get_cuda_device_info

    M, K = (int(v) for v in shape.lower().split("x"))
    dev = torch.device("cuda", 0)
    n_out = synthetic.n_outliers_for(M, outliers)
    if svs == "8":
        ly = synthetic.random_layer_vq8(M, K, n_out, seed=0)
    else:
        ly = synthetic.random_layer_device(M, K, n_out, seed=0, device=dev)
    dl = L.prepare_layer(ly, dev)
    if op == "dequant":
        w = torch.empty(M, K, dtype=torch.float16, device=dev)
        us = measure.graph_time_us(lambda: L.dequantize(dl, out=w), dev, iters)
        # bytes: the packed layer read (indices, codebooks, outlier rows) and W_hat written
        nb = dl.algorithmic_bytes(0) + 2 * M * K
        click.echo(json.dumps({"gpu": get_cuda_device_info().name, "op": "dequant", "shape": [M, K], "svs": int(svs),
                               "n_outliers": dl.n_outliers, "us": us, "bytes": nb, "gbs": nb / us / 1e3}))
        return
    us = _time_gemv(dl, batch, iters)
    nb = dl.algorithmic_bytes(batch)
    click.echo(json.dumps({"gpu": get_cuda_device_info().name, "shape": [M, K], "svs": int(svs),
                           "n_outliers": dl.n_outliers, "batch": batch, "us": us, "bytes": nb, "gbs": nb / us / 1e3,
                           "tflops": 2.0 * M * K * batch / us / 1e6}))


@cli.command("decode-bench")
@click.option("--model", type=click.Choice(["8b", "70b"]), default="8b")
@click.option("--blocks", type=int, default=None, help="decoder blocks (default: the model's)")
@click.option("--batch", type=int, default=1)
@click.option("--iters", type=int, default=20)
@click.option("--launches", is_flag=True, help="one GEMV launch per projection instead of the chain kernel")
@click.option("--form", type=click.Choice(["auto", "barrier", "dataflow"]), default="auto",
              help="chain kernel form (see opac1ty_b200.chain.Chain)")
@click.option("--trace", is_flag=True, help="also report the chain kernel's per-phase timeline (opc_chain_set_trace)")
@click.option("--svs", type=click.Choice(["1", "8"]), default="1", help="sub_vector_size of the synthetic weights")
def decode_bench(model, blocks, batch, iters, launches, form, trace, svs):
    """Time the decode step (q|k|v, o, gate|up, down per block) of synthetic 2-bit weights."""
    import torch

    from . import decode, synthetic
    from .utils import get_cuda_device_info

    cfg = synthetic.LLAMA_8B if model == "8b" else synthetic.LLAMA_70B
    dev = torch.device("cuda", 0)
    st = decode.DecodeStack.synthetic(cfg, n_layers=blocks, device=dev, batch=batch, use_chain=not launches,
                                      chain_form=form, sub_vector_size=int(svs))
    for _ in range(3):
        st.step_eager()
    torch.cuda.synchronize(dev)
    s = torch.cuda.current_stream(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s)
    for _ in range(iters):
        st.step_eager()
    e1.record(s)
    torch.cuda.synchronize(dev)
    ms = e0.elapsed_time(e1) / iters
    nb = st.algorithmic_bytes()
    out = {"gpu": get_cuda_device_info().name, "model": model, "svs": int(svs), "blocks": len(st.blocks), "batch": batch,
           "chain": st.chain is not None, "kernel": st.kernel_name(), "ms_per_step": ms, "tok_s": batch * 1000.0 / ms,
           "gbs": nb / (ms * 1e-3) / 1e9}
    if trace and st.chain is not None:
        out["phases_us"] = _chain_phases_dataflow(st) if st.chain.form == "dataflow" else _chain_phases(st)
    click.echo(json.dumps(out))


def _chain_phases(st) -> dict:
    """Per projection of a block: median over CTAs (mean over the inner blocks) of the time between
    consecutive trace stamps of the chain kernel's first consumer thread -- setup, wait before the
    first poll, x polling, max barrier, digits, staged barrier, own units -- and the GEMV's span
    (start to the next GEMV's start)."""
    import numpy as np
    import torch

    tr = st.chain.enable_trace()
    for _ in range(3):
        st.step_eager()
    torch.cuda.synchronize(st.device)
    full = tr.cpu().numpy().astype(np.int64)  # [steps, grid, 24] ns
    st.chain.disable_trace()
    t = full[:, :, :8]
    warps = full[:, :, 8:23].astype(np.float64)  # [steps, grid, 15] each consumer warp's end of the step
    warps[warps == 0] = np.nan
    names = ["qkv", "o", "gate_up", "down"]
    n_blocks = t.shape[0] // 4
    inner = range(1, n_blocks - 1) if n_blocks > 2 else range(n_blocks)
    starts = np.median(t[:, :, 0], axis=1)
    res = {}
    for p, name in enumerate(names):
        rows = [4 * b + p for b in inner]
        d = np.diff(t[rows], axis=2) / 1000.0
        med = np.median(d, axis=1).mean(axis=0)
        spans = [(starts[r + 1] - starts[r]) / 1000.0 for r in rows if r + 1 < t.shape[0]]
        # per CTA: first and last consumer warp done; across CTAs: the last CTA's lag behind the median
        first = np.nanmin(warps[rows], axis=2)
        last = np.nanmax(warps[rows], axis=2)
        intra = np.median(last - first, axis=1).mean() / 1000.0
        lag = (np.max(last, axis=1) - np.median(last, axis=1)).mean() / 1000.0
        # the slowest CTAs: indices of the 5 latest-finishing CTAs (first inner block)
        slow = np.argsort(last[0])[-5:][::-1].tolist()
        res[name] = {"setup": round(float(med[0]), 2), "pre_poll": round(float(med[1]), 2),
                     "x_wait": round(float(med[2]), 2), "max_barrier": round(float(med[3]), 2),
                     "digits": round(float(med[4]), 2), "staged": round(float(med[5]), 2),
                     "units": round(float(med[6]), 2),
                     "warp_spread_in_cta": round(float(intra), 2), "last_cta_lag": round(float(lag), 2),
                     "slowest_ctas": slow,
                     "span": round(float(np.mean(spans)), 2) if spans else None}
    return res


def _chain_phases_dataflow(st) -> dict:
    """Dataflow form, per projection of a block (median over CTAs, mean over the inner blocks), in
    µs relative to consumer warp 0's start of the GEMV: when the staging warp began the layer
    (after the CTA's consumers left the layer before the previous one), saw its first and its last
    block complete, held every block of x (the next exponent set); when warp 0 began waiting for
    its first chunk's blocks (if it had to) and had them; when warp 0 finished its units; and the
    GEMV's span (to the next GEMV's start)."""
    import numpy as np
    import torch

    tr = st.chain.enable_trace()
    for _ in range(3):
        st.step_eager()
    torch.cuda.synchronize(st.device)
    t = tr.cpu().numpy().astype(np.int64)[:, :, :8]  # [steps, grid, 8] ns
    st.chain.disable_trace()
    names = ["qkv", "o", "gate_up", "down"]
    n_blocks = t.shape[0] // 4
    inner = range(1, n_blocks - 1) if n_blocks > 2 else range(n_blocks)
    starts = np.median(t[:, :, 2], axis=1)
    res = {}
    for p, name in enumerate(names):
        rows = [4 * b + p for b in inner if 4 * b + p > 0]

        def rel(col):
            vals = []
            for r in rows:
                ok = t[r, :, col] > 0
                if ok.any():
                    vals.append(np.median((t[r, ok, col] - t[r, ok, 2]) / 1000.0))
            return round(float(np.mean(vals)), 2) if vals else None

        spans = [(starts[r + 1] - starts[r]) / 1000.0 for r in rows if r + 1 < t.shape[0]]
        res[name] = {"stage_start": rel(0), "first_block": rel(4), "last_block": rel(5), "x_complete": rel(1),
                     "w0_wait_from": rel(6), "w0_blocks_in": rel(7), "units_done": rel(3),
                     "span": round(float(np.mean(spans)), 2) if spans else None}
    return res


@cli.command("engine-bench")
@click.option("--model", type=click.Choice(["8b", "70b"]), default="8b")
@click.option("--blocks", type=int, default=2, help="decoder blocks of the synthetic model")
@click.option("--vocab", type=int, default=32000)
@click.option("--prompt", type=int, default=64, help="prompt tokens (prefill) before the timed steps")
@click.option("--steps", type=int, default=32, help="timed decode steps")
@click.option("--svs", type=click.Choice(["1", "8"]), default="1")
def engine_bench(model, blocks, vocab, prompt, steps, svs):  # noqa: D401
    """Time the engine API (bf_engine_*) on a synthetic Llama-shaped .bf2: prefill and decode steps
    with attention, norms and the lm_head (host-timed around each call, logits copied back)."""
    import os
    import tempfile

    import torch

    from . import synthetic
    from .engine import Engine
    from .utils import get_cuda_device_info

    cfg = synthetic.LLAMA_8B if model == "8b" else synthetic.LLAMA_70B
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "model.bf2")
        t0 = time.time()
        synthetic.write_llama_bf2(path, cfg, blocks, vocab, sub_vector_size=int(svs))
        t_write = time.time() - t0
        t0 = time.time()
        with Engine(path) as eng:
            t_load = time.time() - t0
            toks = list(range(1, prompt + 1))
            eng.prefill(toks[:-1])
            eng.forward_step(toks[-1])  # warm
            eng.reset()
            t0 = time.perf_counter()
            eng.prefill(toks)
            t_prefill = time.perf_counter() - t0
            for i in range(3):
                eng.forward_step(100 + i)
            t0 = time.perf_counter()
            for i in range(steps):
                eng.forward_step(200 + i)
            t_steps = (time.perf_counter() - t0) / steps
            st = eng.stats()
    click.echo(json.dumps({"gpu": get_cuda_device_info().name, "model": model, "svs": int(svs), "blocks": blocks,
                           "vocab": vocab, "prompt_tokens": prompt, "prefill_ms": t_prefill * 1e3,
                           "prefill_tok_s": prompt / t_prefill, "step_ms": t_steps * 1e3, "step_tok_s": 1.0 / t_steps,
                           "kernel_dispatches_total": st["n_kernel_dispatches"], "device_bytes": st["peak_memory_bytes"],
                           "write_s": round(t_write, 1), "load_s": round(t_load, 1)}))


@cli.command("gemm-bench")
@click.option("--shape", default="28672x4096", help="MxK")
@click.option("--tokens", type=int, default=2048)
@click.option("--outliers", type=float, default=0.01, help="outlier row fraction (0 = none)")
@click.option("--iters", type=int, default=10)
def gemm_bench(shape, tokens, outliers, iters):  # noqa: D401
    """Time one synthetic layer's prefill GEMM (tcgen05, CUDA events); prints one JSON line."""
    import torch

    from . import gemm as G, layer as L, measure, synthetic
    from .utils import get_cuda_device_info

    M, K = (int(v) for v in shape.lower().split("x"))
    dev = torch.device("cuda", 0)
    ly = synthetic.random_layer_device(M, K, synthetic.n_outliers_for(M, outliers), seed=0, device=dev)
    dl = L.prepare_layer(ly, dev)
    x = torch.randn(tokens, K, device=dev).half()
    y = torch.empty(tokens, M, dtype=torch.float16, device=dev)
    us = measure.graph_time_us(lambda: G.gemm(dl, x, out=y), dev, iters)  # L2 flushed before each launch
    fl = G.flops(dl, tokens)
    click.echo(json.dumps({"gpu": get_cuda_device_info().name, "shape": [M, K], "tokens": tokens,
                           "n_outliers": dl.n_outliers, "us": us, "tflops": fl / us / 1e6}))


def main():
    cli(standalone_mode=True)


if __name__ == "__main__":
    main()

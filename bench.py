#!/usr/bin/env python
"""Benchmark: fused 2-bit VQ GEMV at Llama-3.1-8B decode shapes (batch 1, 32 decoder blocks).

One step = one decode token through the projection chain of all 32 blocks (qkv -> o -> gate|up
-> down per block, 128 dependent GEMVs; opac1ty_b200.decode), run by the persistent decode-chain
kernel (one launch per step) for batch 1..2, else one GEMV launch per projection.  Weights are
random-initialised 2-bit layers of the named shapes with 1 % outlier rows (synthetic data; no
checkpoint).  The weight set (1.9 GB) is far larger than L2, so no L2 flush is needed between
steps.

  value     decode tok/s with weights and activations resident in HBM (CUDA graph replay),
            device-timed with CUDA events, max over ranks
  e2e       same metric through the public call with host buffers: each step copies x from
            pinned host memory, runs the step, copies the output back (copies inside the timing)
  roofline  algorithmic bytes per step / step time against the measured HBM peak
  parity    the step's own output checked after timing: deterministic over two runs, equal bit
            for bit across ranks and to a one-GPU run (N > 1), and within tolerance of an fp64
            recompute of block 0 (torch, from the dequantized weights)
  prefill / llama70b / sweep  (N = 1) the other benchmark configurations: the tcgen05 prefill
            GEMM at 512 and 2048 tokens, the Llama-3-70B decode step at batch 1 and 16, and the
            outlier x batch sweep of the 14336x4096 gate projection with the GEMV->GEMM crossover
  engine    (N = 1) the bf_engine_* API on a 4-block Llama-3.1-8B-shaped model: a 512-token
            prompt and decode steps with attention, norms and the lm_head, in a child process

--impl reference times the reference's CPU implementation of the path (dequantize + fp32 matmul,
restated in C in oracle/) on all host cores for the same metric: each step is one whole decode
token (224 projection GEMVs).  It also times the reference's own Python code
(opacc1ty.export.converter.dequantize_layer + torch.matmul, installed unmodified under
baseline/_ref) on a bounded sample of a 4096x4096 layer.

N > 1 GPUs (torchrun): output-channel tensor parallelism (opac1ty_b200.tp) -- every projection
row-sharded across the ranks.  Default (--tp-impl chain, batch 1..2): one persistent kernel per
rank per step that stores its output rows straight into every rank's activations over NVLink
(CUDA IPC peer pointers).  --tp-impl nccl: one GEMV launch per projection followed by an NCCL
all-gather (the baseline form).  value and the roofline count the whole model's bytes per step.
"""

from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

import numpy as np  # noqa: E402

METRIC = "fused 2-bit VQ GEMV HBM TB/s (% peak); decode tok/s @ Llama-3.1-8B shapes"
# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) of one chain-kernel launch over its
# algorithmic bytes, from an ncu capture of the 4-block step (mean of two launches: 243.9 and
# 240.8 MB for 237.3 MB); the traffic is
# proportional to the blocks, so the full step's traffic is this ratio times its algorithmic bytes.
CHAIN_TRAFFIC_RATIO = 1.021
WORKLOAD = "Llama-3.1-8B decode GEMV set, batch 1, 32 blocks (q|k|v, o, gate|up, down), 2-bit svs=1, 1% outlier rows"
DTYPE = ("2-bit codebook weights, fp16 x and y; batch 1-2 dot products exact in integers: int8 x uint8 mma.sync "
         "of 15-bit fixed-point centroids and 22-bit fixed-point x (scaled by max|x| of each GEMV's input), "
         "int64 sums, one fp16 rounding per output")
PARITY_TOL = 2e-3
BLOCKS = 32


def config_for(batch: int) -> dict:
    """The workload, identical for both arms."""
    return {"workload": WORKLOAD.replace("batch 1", f"batch {batch}"), "batch": batch, "blocks": BLOCKS,
            "l2": "inputs larger than L2 (1.9 GB of weights per step)"}


def measured_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            d = json.loads(p.read_text())
            return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]), "source": "measured"}
        except Exception:
            pass
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


def log(msg: str):
    print(f"[bench] {msg}", file=sys.stderr, flush=True)


class ClockSampler:
    """nvidia-smi clock / throttle sampling during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits", "-lms", "100",
                 "-i", str(self.gpu)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (FileNotFoundError, OSError):
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self.thread:
            self.thread.join(timeout=2)
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"], "samples": 0}
        return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": float(max(smax)), "reasons": sorted(reasons),
                "samples": len(sm)}


def cpu_model() -> str:
    try:
        for ln in Path("/proc/cpuinfo").read_text().splitlines():
            if ln.startswith("model name"):
                return ln.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


# ---------------------------------------------------------------------------------------------
# The reference's CPU path (CPU baseline and --impl reference)
# ---------------------------------------------------------------------------------------------
class CpuReference:
    """The reference CPU path (dequantize + fp32 dot, restated in C in oracle/) for a whole decode
    token: 32 blocks of the 7 Llama-3.1-8B projections with the decode dataflow (q|k|v from x, o
    from q, gate and up from o, down from gate).  One block's seeded weights serve all 32 blocks:
    the work per block is identical and one block (218 MB of indices) already exceeds the host's
    caches, so the timing is that of 32 distinct blocks without 7 GB of host memory."""

    def __init__(self, threads: int, batch: int = 1, seed: int = 0):
        from oracle import oracle
        from opac1ty_b200 import synthetic

        self.oracle = oracle
        self.threads = threads
        self.proj = {}
        for pi, (name, (M, K)) in enumerate(synthetic.decoder_shapes(synthetic.LLAMA_8B).items()):
            ly = synthetic.random_layer(M, K, synthetic.n_outliers_for(M, 0.01), seed=seed + pi)
            cb, idx, ov, oi, _, _ = oracle.layer_arrays(ly)
            self.proj[name] = (cb, idx, ov, oracle.outlier_slots(M, oi), M, K)
        self.h = synthetic.LLAMA_8B["hidden"]
        self.f = synthetic.LLAMA_8B["intermediate"]
        self.x0 = synthetic.activations(batch, self.h, seed=1)

    def _gemv(self, name, x):
        return self.oracle.gemv_cpu(self.proj[name], np.ascontiguousarray(x), threads=self.threads)

    def token(self) -> float:
        """One decode step (all 32 blocks); returns its wall time in seconds."""
        t0 = time.perf_counter()
        x = self.x0
        for _ in range(BLOCKS):
            q = self._gemv("q_proj", x)
            self._gemv("k_proj", x)
            self._gemv("v_proj", x)
            o = self._gemv("o_proj", q)
            g = self._gemv("gate_proj", o)
            self._gemv("up_proj", o)
            x = self._gemv("down_proj", g)
        return time.perf_counter() - t0

    def tok_s(self, max_seconds: float, batch: int) -> tuple:
        times, t_start = [], time.perf_counter()
        while not times or time.perf_counter() - t_start < max_seconds:
            times.append(self.token())
        return batch / float(np.median(times)), len(times)


def literal_reference_leg(rows: int = 48) -> dict:
    """The reference's own code on config 0 (a 4096x4096 layer): opacc1ty's dequantize_layer
    (a Python loop per weight, opacc1ty/export/converter.py:26-67) on the first ``rows`` rows and
    torch.matmul of x with them, both scaled to the full layer by rows.  Runs the unmodified
    package installed under baseline/_ref."""
    ref_dir = ROOT / "baseline" / "_ref"
    if not (ref_dir / "opacc1ty").is_dir():
        return {"unavailable": "the reference package is not installed under baseline/_ref"}
    sys.path.insert(0, str(ref_dir))
    try:
        import torch
        from opacc1ty.export.converter import dequantize_layer
    except Exception as e:  # noqa: BLE001
        return {"unavailable": f"import failed: {e}"}
    finally:
        sys.path.remove(str(ref_dir))
    from opac1ty_b200 import synthetic

    M, K = 4096, 4096
    layer = synthetic.random_layer(M, K, 40, seed=2024)
    sample = {"type": "quantized", "shape": (rows, K), "codebooks": layer["codebooks"][:rows],
              "indices": layer["indices"][:rows], "outlier_values": None, "outlier_indices": None}
    x = torch.from_numpy(synthetic.activations(1, K, seed=1)).float()
    t0 = time.perf_counter()
    w = dequantize_layer(sample)
    t1 = time.perf_counter()
    _ = x @ torch.from_numpy(w).float().T
    t2 = time.perf_counter()
    scale = M / rows
    gemv_s = (t1 - t0 + t2 - t1) * scale
    weights_per_token = sum(m * k for m, k in synthetic.decoder_shapes(synthetic.LLAMA_8B).values()) * BLOCKS
    return {"config0_gemv_s": round(gemv_s, 3), "dequant_s_per_mweight": round((t1 - t0) / (rows * K) * 1e6, 3),
            "decode_tok_s_extrapolated": 1.0 / (gemv_s * weights_per_token / (M * K)),
            "sample": f"dequantize_layer + torch.matmul on {rows} of 4096 rows of a 4096x4096 layer, scaled by rows; "
                      "tok/s extrapolated by weights per token",
            "threads": torch.get_num_threads()}


def run_reference(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    threads = os.cpu_count() or 1
    ref = CpuReference(threads, batch=args.batch)
    for _ in range(args.warmup):
        ref.token()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        ref.token()
    ms = (time.perf_counter() - t0) * 1000.0 / args.steps
    v = args.batch * 1000.0 / ms
    line = {
        "metric": METRIC, "value": v, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "fp16 weights after dequantization, fp32 accumulate (CPU)", "data": "synthetic",
        "impl": "reference",
        "config": config_for(args.batch),
        "cpu_baseline": {"value": v, "unit": "tok/s", "cores": threads, "kind": "port",
                         "sample": "each step = one whole decode token (32 blocks x 7 projections, the reference's "
                                   f"dequantize + fp32 dot restated in C, all host threads); CPU: {cpu_model()}"},
        "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    if not args.no_literal:
        line["literal_reference"] = literal_reference_leg()
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------------------------------------
# This repository's arm
# ---------------------------------------------------------------------------------------------
def torch_dequant(layer: dict):
    """W_hat [M][K] from a reference layer dict in plain torch on its device: codebook gather and
    ordered outlier-row replacement (the semantics of opacc1ty/export/converter.py:26-67)."""
    import torch

    cb = layer["codebooks"]
    idx = layer["indices"].long()
    rows = torch.arange(cb.shape[0], device=cb.device)[:, None]
    w = cb[rows, idx, 0].clone()
    if layer.get("outlier_indices") is not None and len(layer["outlier_indices"]):
        for i, r in enumerate(layer["outlier_indices"].tolist()):
            w[int(r)] = layer["outlier_values"][i].to(w.device)
    return w


def block0_fp64(cfg: dict, x, device):
    """fp64 recompute of block 0's projection chain (seeds of DecodeStack.synthetic): each GEMV in
    float64 on the GPU from the dequantized weights, rounded to fp16 between GEMVs like the chain."""
    import torch

    from opac1ty_b200 import decode, synthetic

    shapes = synthetic.decoder_shapes(cfg)
    bd = {}
    for pi, (name, (M, K)) in enumerate(shapes.items()):
        bd[name] = synthetic.random_layer_device(M, K, synthetic.n_outliers_for(M, 0.01), seed=pi, device=device)
    h, f = cfg["hidden"], cfg["intermediate"]
    seq = [(decode.concat_rows([bd["q_proj"], bd["k_proj"], bd["v_proj"]]), None),
           (bd["o_proj"], h), (decode.concat_rows([bd["gate_proj"], bd["up_proj"]]), None), (bd["down_proj"], f)]
    cur = x
    y64 = None
    for ly, take in seq:
        inp = cur if take is None else cur[:, :take]
        w = torch_dequant(ly).double()
        y64 = inp.double() @ w.T
        cur = y64.half()
        del w
    return y64


def parity_check(stack, cfg, args, dev, dist, world, rank) -> dict:
    """Run one step from a fixed x and check it (every rank takes the same collective steps)."""
    import torch

    from opac1ty_b200 import decode, synthetic

    B = args.batch
    x0 = torch.from_numpy(synthetic.activations(B, cfg["hidden"], seed=4242)).to(dev)
    outs = []
    for _ in range(2):
        stack.bufs["x"].copy_(x0)
        stack.step()
        outs.append(stack.bufs["x"].clone())
    torch.cuda.synchronize(dev)
    res = {"deterministic": bool(torch.equal(outs[0], outs[1]))}
    if world > 1:
        gathered = [torch.empty_like(outs[0]) for _ in range(world)]
        dist.all_gather(gathered, outs[0])
        if rank == 0:
            res["ranks_equal"] = all(torch.equal(g, gathered[0]) for g in gathered)
            log("parity: building the one-GPU stack")
            # the row-sharded kernel scales every step's x by the exponent of max|x|, as the per-GEMV
            # launches do: their one-GPU run is the bit-exact reference
            ref = decode.DecodeStack.synthetic(cfg, device=dev, batch=B, use_chain=False)
            ref.bufs["x"].copy_(x0)
            y1 = ref.step_eager().clone()
            torch.cuda.synchronize(dev)
            res["bit_equal_1gpu"] = bool(torch.equal(y1, gathered[0]))
            res["one_gpu_kernel"] = ref.kernel_name()
            del ref
            torch.cuda.empty_cache()
        dist.barrier()
    if rank == 0:
        form = getattr(getattr(stack, "chain", None), "form", "barrier")
        one = decode.DecodeStack.synthetic(cfg, n_layers=1, device=dev, batch=B, use_chain=True, chain_form=form)
        one.bufs["x"].copy_(x0)
        y = one.step_eager().clone().double()
        y64 = block0_fp64(cfg, x0, dev)
        res["rel_err_block0"] = float((y - y64).abs().max() / y64.abs().max())
        res["tolerance"] = PARITY_TOL
        res["ok"] = res["deterministic"] and res["rel_err_block0"] <= PARITY_TOL and res.get("ranks_equal", True) \
            and res.get("bit_equal_1gpu", True)
        res["block0_form"] = form
        res["what"] = ("two runs of the timed step from one x bit-equal; N > 1: every rank's output equal and equal to "
                       "a one-GPU run of per-GEMV launches (the same integer arithmetic and x scale); block 0 (one chain "
                       "launch of the timed form) against a float64 torch recompute from the dequantized weights, "
                       "norm-wise max|y - y64| / max|y64|")
        del one
        torch.cuda.empty_cache()
    return res


def engine_config(blocks: int = 4, prompt: int = 512, steps: int = 32, timeout_s: float = 240.0) -> dict:
    """The engine API (bf_engine_*) on a synthetic Llama-3.1-8B-shaped .bf2 of `blocks` blocks and
    a 32000-token vocabulary: a `prompt`-token prefill and `steps` decode steps (attention, norms,
    rotary embedding and the lm_head included), run by `cli engine-bench` in a child process (its
    own CUDA context, so a failure there cannot take this run down; host-timed around each call
    with the logits copied back)."""
    cmd = [sys.executable, "-m", "opac1ty_b200.cli", "engine-bench", "--blocks", str(blocks), "--prompt", str(prompt),
           "--steps", str(steps)]
    r = subprocess.run(cmd, cwd=str(ROOT), capture_output=True, text=True, timeout=timeout_s)
    if r.returncode != 0:
        return {"error": f"engine-bench exited {r.returncode}: {r.stderr.strip()[-300:]}"}
    res = json.loads(r.stdout.strip().splitlines()[-1])
    res["config"] = (f"bf_engine_* on a Llama-3.1-8B-shaped model of {blocks} blocks: {prompt}-token prompt, then "
                     f"{steps} decode steps (host-timed per call, logits copied back)")
    res["step_ms_per_block"] = round(res["step_ms"] / blocks, 4)
    return res


def extra_configs(dev, peaks) -> dict:
    """The other benchmark configurations (configs 2-4), device-timed; each key stands alone."""
    import torch

    from opac1ty_b200 import measure, synthetic

    out = {}
    t0 = time.time()
    try:
        out["prefill"] = dict(measure.prefill(synthetic.LLAMA_8B, dev, (512, 2048), peaks["bf16_tflops"]),
                              config="Llama-3.1-8B prefill GEMM, one block's projections, 512 and 2048 tokens",
                              peak_tflops=peaks["bf16_tflops"], peak_source=peaks["source"])
    except Exception as e:  # noqa: BLE001
        out["prefill"] = {"error": str(e)}
    log(f"prefill done ({time.time() - t0:.0f} s)")
    t0 = time.time()
    try:
        rows = []
        for b in (1, 16):
            r = measure.decode(synthetic.LLAMA_70B, dev, batch=b, steps=5)
            r["roofline_frac"] = round(r["gbs"] / peaks["hbm_gbs"], 4)
            rows.append(r)
            log(f"llama70b batch {b}: {r['tok_s']} tok/s (built in {r['build_s']} s)")
        out["llama70b"] = {"config": "Llama-3-70B decode step, 80 blocks, 1 GPU", "rows": rows}
    except Exception as e:  # noqa: BLE001
        out["llama70b"] = {"error": str(e)}
    torch.cuda.empty_cache()
    t0 = time.time()
    try:
        out["sweep"] = dict(measure.outlier_batch_sweep(14336, 4096, dev),
                            config="gate projection 14336x4096, outliers 0/1/2 %, batch 1/4/16/64")
    except Exception as e:  # noqa: BLE001
        out["sweep"] = {"error": str(e)}
    log(f"sweep done ({time.time() - t0:.0f} s)")
    t0 = time.time()
    try:
        out["engine"] = engine_config()
    except Exception as e:  # noqa: BLE001
        out["engine"] = {"error": str(e)}
    log(f"engine done ({time.time() - t0:.0f} s)")
    return out


def run_ours(args):
    import torch

    from opac1ty_b200 import decode, synthetic, _lib

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    _lib.load()
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    peaks = measured_peaks()

    cfg = synthetic.LLAMA_8B
    t_build = time.time()
    if world > 1:
        from opac1ty_b200 import tp

        stack = tp.TPDecodeStack.synthetic(cfg, rank=rank, world=world, device=dev, batch=args.batch)
        if args.tp_impl == "chain" and args.batch <= 2:
            stack.enable_chain()
    else:
        stack = decode.DecodeStack.synthetic(cfg, device=dev, batch=args.batch)
    torch.cuda.synchronize()
    log(f"stack built in {time.time() - t_build:.1f} s")

    # Warm-up (eager once, then capture, then graph replays).
    stack.step_eager()
    torch.cuda.synchronize()
    stack.capture()
    for _ in range(max(args.warmup, 3)):
        stack.step()
    torch.cuda.synchronize()

    stream = torch.cuda.current_stream(dev)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sampler = ClockSampler(local_rank)
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    sampler.start()
    start.record(stream)
    for _ in range(args.steps):
        stack.step()
    end.record(stream)
    torch.cuda.synchronize()
    clocks = sampler.stop()
    ms = start.elapsed_time(end) / args.steps
    if dist is not None:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    tok_s = args.batch * 1000.0 / ms

    # e2e: host x (pinned) -> device, step, output -> host, every step.
    h = stack.hidden
    x_host = torch.from_numpy(synthetic.activations(args.batch, h, seed=1)).pin_memory()
    y_host = torch.empty(args.batch, h, dtype=torch.float16).pin_memory()
    for _ in range(2):
        stack.bufs["x"].copy_(x_host, non_blocking=True)
        stack.step()
        y_host.copy_(stack.bufs["x"], non_blocking=True)
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        stack.bufs["x"].copy_(x_host, non_blocking=True)
        stack.step()
        y_host.copy_(stack.bufs["x"], non_blocking=True)
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / args.steps
    if dist is not None:
        t = torch.tensor([e2e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    e2e_tok_s = args.batch * 1000.0 / e2e_ms

    step_bytes = stack.algorithmic_bytes()
    if dist is not None:
        t = torch.tensor([step_bytes], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        step_bytes = int(t.item())
    achieved_gbs = step_bytes / (ms * 1e-3) / 1e9
    kernel_name = stack.kernel_name()
    fused = getattr(stack, "chain", None) is not None
    launches = stack.launches_per_step()
    # Per-kernel view: each distinct layer shape timed alone (graph-replayed launches).
    kernels = per_layer_timing(stack, dev) if world == 1 else None

    # Parity of the timed step (collective at N > 1).
    parity = parity_check(stack, cfg, args, dev, dist, world, rank)

    cpu = None
    if world == 1 and rank == 0 and not args.no_cpu_baseline:
        threads = os.cpu_count() or 1
        v, reps = CpuReference(threads, batch=args.batch).tok_s(args.cpu_seconds, args.batch)
        cpu = {"value": v, "unit": "tok/s", "cores": threads, "kind": "port",
               "sample": f"whole decode tokens (32 blocks x 7 projections), median of {reps}; CPU: {cpu_model()}"}

    extras = {}
    if world == 1 and not args.no_extra:
        stack.graph = None
        extras = extra_configs(dev, peaks)

    if world == 1:
        tp_desc = "single GPU"
    elif fused:
        tp_desc = f"tp{world} (row shards; one fused kernel per rank: peer stores over NVLink)"
    else:
        tp_desc = f"tp{world} (row shards; GEMV launch + NCCL all-gather per projection)"
    if rank == 0:
        line = {
            "metric": METRIC, "value": tok_s, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": DTYPE, "data": "synthetic",
            "config": config_for(args.batch),
            "implementation": {"parallelism": tp_desc, "kernel": kernel_name, "launches_per_step": launches,
                               "cuda_graph": True, "pdl": not fused},
            "roofline": {"bound": "hbm", "achieved": achieved_gbs, "peak": peaks["hbm_gbs"] * world, "unit": "GB/s",
                         "frac": achieved_gbs / (peaks["hbm_gbs"] * world),
                         "traffic": int(step_bytes * CHAIN_TRAFFIC_RATIO) if fused else None,
                         "traffic_source": "ncu dram bytes of the chain kernel on the 4-block step, scaled by bytes"
                         if fused else None,
                         "peak_source": peaks["source"], "algorithmic_bytes_per_step": step_bytes,
                         "kernel": kernel_name},
            "hbm_tbs": achieved_gbs / 1000.0,
            "parity": parity,
            "kernels": kernels,
            "clocks": clocks,
            "e2e": {"value": e2e_tok_s, "unit": "tok/s", "h2d_bytes_per_step": 2 * args.batch * h,
                    "d2h_bytes_per_step": 2 * args.batch * h},
            "gpu_launches": launches * args.steps,
            "cpu_baseline": cpu,
        }
        line.update(extras)
        print(json.dumps(line), flush=True)
    if dist is not None:
        stack.graph = None
        torch.cuda.synchronize()
        dist.barrier()
        stack.close()
        dist.destroy_process_group()
    return 0


def per_layer_timing(stack, dev, reps: int = 20) -> list:
    """Each distinct projection shape of block 0, timed alone (graph-replayed launches)."""
    from opac1ty_b200 import layer as L
    from opac1ty_b200 import measure

    out = []
    blk = stack.blocks[0]
    bufs = stack.bufs
    h, f = stack.hidden, stack.intermediate
    plan = [("qkv", blk.qkv, bufs["x"], bufs["qkv"]), ("o_proj", blk.o, bufs["qkv"][:, :h], bufs["o"]),
            ("gate_up", blk.gate_up, bufs["o"], bufs["gu"]), ("down_proj", blk.down, bufs["gu"][:, :f], bufs["x"])]
    for name, dl, x, y in plan:
        us = measure.graph_time_us(lambda: L.gemv(dl, x, out=y, workspace=stack.workspace), dev, reps)
        nbytes = dl.algorithmic_bytes(stack.batch)
        out.append({"layer": name, "shape": [dl.M, dl.K], "n_outliers": dl.n_outliers, "us": us,
                    "gbs": nbytes / (us * 1e-6) / 1e9, "bytes": nbytes})
    return out


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extra", action="store_true", help="skip the prefill / 70B / sweep measurements")
    ap.add_argument("--no-literal", action="store_true", help="reference arm: skip the reference's own Python leg")
    ap.add_argument("--cpu-seconds", type=float, default=20.0)
    ap.add_argument("--tp-impl", choices=["chain", "nccl"], default="chain",
                    help="N > 1: fused row-sharded chain kernel (default) or GEMV + NCCL all-gather")
    args = ap.parse_args(argv)
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())

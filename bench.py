#!/usr/bin/env python
"""Benchmark: fused 2-bit VQ GEMV at Llama-3.1-8B decode shapes (batch 1, 32 decoder blocks).

One step = one decode token through the projection chain of all 32 blocks (qkv -> o -> gate|up
-> down per block, 128 dependent GEMVs; opac1ty_b200.decode), run by the persistent decode-chain
kernel (one launch per step) for batch 1..2, else one GEMV launch per projection.  Weights are
random-initialised 2-bit layers of the named shapes with 1 % outlier rows (synthetic data; no
checkpoint).  The weight set (1.9 GB) is far larger than L2, so no L2 flush is needed between
steps.

  value   decode tok/s with weights and activations resident in HBM (CUDA graph replay),
          device-timed with CUDA events, max over ranks
  e2e     same metric through the public call with host buffers: each step copies x from
          pinned host memory, runs the step, copies the output back (copies inside the timing)
  roofline.achieved  algorithmic bytes per step / step time (GEMV is the only kernel)

--impl reference times the reference's CPU implementation of the path (dequantize + fp32
matmul, restated in C in oracle/) on all host cores, on a bounded sample (1 of 32 blocks,
scaled), in the same metric.

N > 1 GPUs (torchrun): output-channel tensor parallelism (opac1ty_b200.tp) -- every projection
row-sharded across the ranks.  Default (--tp-impl chain, batch 1..2): one persistent kernel per
rank per step that stores its output rows straight into every rank's activations over NVLink
(CUDA IPC peer pointers) with a cross-rank flag barrier between projections.  --tp-impl nccl:
one GEMV launch per projection followed by an NCCL all-gather (the baseline form).  value and
the roofline count the whole model's bytes per step (summed over ranks).
"""

from __future__ import annotations

import argparse
import json
import math
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


def measured_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            d = json.loads(p.read_text())
            return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]), "source": "measured"}
        except Exception:
            pass
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


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


class CpuReference:
    """Reference CPU path (dequantize + fp32 dot, restated in C in oracle/) for one decoder
    block's 7 projections at Llama-3.1-8B shapes; one pass = 1/32 of a decode token."""

    def __init__(self, threads: int, seed: int = 0):
        from oracle import oracle
        from opac1ty_b200 import synthetic

        self.oracle = oracle
        self.threads = threads
        self.arrays = []
        for pi, (name, (M, K)) in enumerate(synthetic.decoder_shapes(synthetic.LLAMA_8B).items()):
            ly = synthetic.random_layer(M, K, synthetic.n_outliers_for(M, 0.01), seed=seed + pi)
            cb, idx, ov, oi, _, _ = oracle.layer_arrays(ly)
            self.arrays.append(((cb, idx, ov, oracle.outlier_slots(M, oi), M, K), K))
        self.xs = {K: synthetic.activations(1, K, seed=1000 + K) for _, K in self.arrays}
        self.blocks_per_token = synthetic.LLAMA_8B["layers"]

    def block_pass(self) -> float:
        t0 = time.perf_counter()
        for arr, K in self.arrays:
            self.oracle.gemv_cpu(arr, self.xs[K], threads=self.threads)
        return time.perf_counter() - t0

    def tok_s(self, max_seconds: float) -> tuple:
        times, t_start = [], time.perf_counter()
        while not times or time.perf_counter() - t_start < max_seconds:
            times.append(self.block_pass())
        return 1.0 / (float(np.median(times)) * self.blocks_per_token), len(times)


def run_reference(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    threads = os.cpu_count() or 1
    ref = CpuReference(threads)
    for _ in range(args.warmup):
        ref.block_pass()
    times = [ref.block_pass() for _ in range(args.steps)]
    v = 1.0 / (float(np.median(times)) * ref.blocks_per_token)
    line = {
        "metric": METRIC, "value": v, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": 1000.0 / v, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "fp16 (2-bit codebook weights, fp32 accumulate)", "data": "synthetic",
        "impl": "reference",
        "config": {"workload": WORKLOAD, "batch": 1, "blocks": 32, "l2": "inputs larger than L2"},
        "cpu_baseline": {"value": v, "unit": "tok/s", "cores": threads, "kind": "port",
                         "sample": "each step = 1 of the 32 decoder blocks (7 projections); tok/s from the "
                                   f"median block time x32; CPU: {cpu_model()}"},
        "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


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

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    peaks = measured_peaks()

    cfg = synthetic.LLAMA_8B
    if world > 1:
        from opac1ty_b200 import tp

        stack = tp.TPDecodeStack.synthetic(cfg, rank=rank, world=world, device=dev, batch=args.batch)
        if args.tp_impl == "chain" and args.batch <= 2:
            stack.enable_chain()
    else:
        stack = decode.DecodeStack.synthetic(cfg, device=dev, batch=args.batch)
    torch.cuda.synchronize()

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
    # Per-kernel view: each distinct layer shape timed alone (eager, events on its stream).
    kernels = per_layer_timing(stack, dev) if world == 1 else None

    cpu = None
    if world == 1 and rank == 0 and not args.no_cpu_baseline:
        threads = os.cpu_count() or 1
        v, reps = CpuReference(threads).tok_s(args.cpu_seconds)
        cpu = {"value": v, "unit": "tok/s", "cores": threads, "kind": "port",
               "sample": f"1 of 32 decoder blocks (7 projections), median of {reps} passes, scaled x32; "
                         f"CPU: {cpu_model()}"}

    fused = getattr(stack, "chain", None) is not None
    if world == 1:
        tp_desc = "single GPU"
    elif fused:
        tp_desc = f"tp{world} (row shards; one fused kernel per rank: peer stores + flag barrier over NVLink)"
    else:
        tp_desc = f"tp{world} (row shards; GEMV launch + NCCL all-gather per projection)"
    kernel_name = "opc::chain_kernel" if fused else "opc::gemvq_kernel / opc::gemv_kernel"
    if rank == 0:
        line = {
            "metric": METRIC, "value": tok_s, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "fp16 (2-bit codebook weights, fp32 accumulate)", "data": "synthetic",
            "config": {"workload": WORKLOAD, "batch": args.batch, "blocks": 32, "launches_per_step":
                       stack.launches_per_step(), "l2": "inputs larger than L2 (1.9 GB of weights per step)",
                       "parallelism": tp_desc,
                       "cuda_graph": True,
                       "pdl": True},
            "roofline": {"bound": "hbm", "achieved": achieved_gbs, "peak": peaks["hbm_gbs"] * world, "unit": "GB/s",
                         "frac": achieved_gbs / (peaks["hbm_gbs"] * world),
                         "traffic": int(step_bytes * CHAIN_TRAFFIC_RATIO) if fused else None,
                         "traffic_source": "ncu dram bytes of the chain kernel on the 4-block step, scaled by bytes"
                         if fused else None,
                         "peak_source": peaks["source"], "algorithmic_bytes_per_step": step_bytes,
                         "kernel": kernel_name},
            "hbm_tbs": achieved_gbs / 1000.0,
            "kernels": kernels,
            "clocks": clocks,
            "e2e": {"value": e2e_tok_s, "unit": "tok/s", "h2d_bytes_per_step": 2 * args.batch * h,
                    "d2h_bytes_per_step": 2 * args.batch * h},
            "gpu_launches": stack.launches_per_step() * args.steps,
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    if dist is not None:
        stack.graph = None
        torch.cuda.synchronize()
        dist.barrier()
        stack.close()
        dist.destroy_process_group()
    return 0


def per_layer_timing(stack, dev, reps: int = 20) -> list:
    """Each distinct projection shape of block 0, timed alone back-to-back (eager launches)."""
    import torch

    from opac1ty_b200 import layer as L

    out = []
    blk = stack.blocks[0]
    bufs = stack.bufs
    h, f = stack.hidden, stack.intermediate
    plan = [("qkv", blk.qkv, bufs["x"], bufs["qkv"]), ("o_proj", blk.o, bufs["qkv"][:, :h], bufs["o"]),
            ("gate_up", blk.gate_up, bufs["o"], bufs["gu"]), ("down_proj", blk.down, bufs["gu"][:, :f], bufs["x"])]
    stream = torch.cuda.current_stream(dev)
    for name, dl, x, y in plan:
        for _ in range(3):
            L.gemv(dl, x, out=y, workspace=stack.workspace)
        torch.cuda.synchronize()
        # replayed from a CUDA graph, so the time is the GPU's rather than the Python call rate
        g = torch.cuda.CUDAGraph()
        cs = torch.cuda.Stream(dev)
        cs.wait_stream(stream)
        with torch.cuda.stream(cs):
            L.gemv(dl, x, out=y, workspace=stack.workspace)
        stream.wait_stream(cs)
        with torch.cuda.graph(g):
            for _ in range(reps):
                L.gemv(dl, x, out=y, workspace=stack.workspace)
        g.replay()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        g.replay()
        e1.record(stream)
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1000.0 / reps
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

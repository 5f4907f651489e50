#!/usr/bin/env python
"""Generate the golden fixtures in this directory from the reference implementation itself.

Run where the reference source tree is available, naming it explicitly:

    python tests/golden/make_golden.py --reference <path to the opacc1ty source tree>

(or set OPACC1TY_REFERENCE); the outputs are committed so the tests need only this directory.

  dequant_svs1.npz      random svs=1 layer with a repeated outlier id and an outlier in the
                        last row -> reference dequantize_layer (opacc1ty/export/converter.py)
  dequant_svs8.npz      svs=8 layer with outliers -> dequantize_layer
  dequant_svs8_trim.npz svs=8, in_features not a multiple of 8 (the reference trims columns)
  quantized_svs1.npz    reference VectorQuantizer.quantize_layer (svs=1) on seeded Student-t
                        weights, plus its dequantized matrix and an fp32 torch matmul / fp64 y
  ref_int64.bf2         reference BF2Writer output for a small model whose outlier ids are int64
                        (as the quantizer returns them); ref_int64_readback.json records what the
                        reference BF2Reader reads back from it
  ref_int32.bf2         the same layers with int32 ids
  config0_pin.json      4096x4096 layer from opac1ty_b200.synthetic.random_layer(seed=2024, 40
                        outlier rows): SHA-256 of the reference dequantize_layer output, and the
                        fp64 y for a seeded x (this one takes a few minutes: the reference
                        dequantizes with a Python loop)
Every case also stores a seeded x and y = x . W^T (torch fp32, the reference's own matmul) and
y64 (float64).
"""

from __future__ import annotations

import hashlib
import json
import os
import sys
import time
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent

def _reference_path() -> str:
    """The reference source tree: --reference PATH, else $OPACC1TY_REFERENCE (no default)."""
    argv = sys.argv[1:]
    for i, a in enumerate(argv):
        if a == "--reference" and i + 1 < len(argv):
            return argv[i + 1]
        if a.startswith("--reference="):
            return a.split("=", 1)[1]
    env = os.environ.get("OPACC1TY_REFERENCE")
    if env:
        return env
    sys.exit("make_golden.py: name the reference source tree with --reference PATH or OPACC1TY_REFERENCE")


REF = _reference_path()
sys.path.insert(0, REF)
sys.path.insert(1, str(ROOT))

from opacc1ty.export.converter import dequantize_layer  # noqa: E402
from opacc1ty.format.bf2 import BF2Reader, BF2Writer  # noqa: E402
from opacc1ty.quantize.vq import QuantizeConfig, VectorQuantizer  # noqa: E402

from opac1ty_b200 import synthetic  # noqa: E402


def rng(seed):
    return np.random.Generator(np.random.PCG64(seed))


def y_pair(W: np.ndarray, x: np.ndarray):
    y32 = (torch.from_numpy(x).float() @ torch.from_numpy(W).float().T).numpy()
    y64 = x.astype(np.float64) @ W.astype(np.float64).T
    return y32, y64


def save_case(name, layer, x_rows=3, seed=0):
    W = dequantize_layer(layer)
    M, Kc = W.shape
    x = rng(seed + 99).standard_normal((x_rows, Kc)).astype(np.float16)
    y32, y64 = y_pair(W, x)
    arrays = {
        "shape": np.array(layer["shape"], dtype=np.int64),
        "codebooks": layer["codebooks"].numpy(),
        "indices": layer["indices"].numpy(),
        "W": W, "x": x, "y32": y32, "y64": y64,
    }
    if layer.get("outlier_values") is not None:
        arrays["outlier_values"] = layer["outlier_values"].numpy()
        arrays["outlier_indices"] = layer["outlier_indices"].numpy()
    np.savez_compressed(HERE / f"{name}.npz", **arrays)
    print(f"{name}: W {W.shape}")


def main(skip_large=False):
    g = rng(1)
    # 1. svs=1, repeated id (5 appears twice: the later row wins) and an outlier in the last row.
    M, K = 48, 200
    save_case("dequant_svs1", {
        "type": "quantized", "shape": (M, K),
        "codebooks": torch.from_numpy((g.standard_normal((M, 4, 1)) * 0.02).astype(np.float16)),
        "indices": torch.from_numpy(g.integers(0, 4, (M, K), dtype=np.uint8)),
        "outlier_values": torch.from_numpy((g.standard_normal((4, K)) * 0.2).astype(np.float16)),
        "outlier_indices": torch.tensor([5, 47, 5, 20], dtype=torch.int64),
    }, seed=1)
    # 2. svs=8 with outliers.
    M, K = 32, 64
    save_case("dequant_svs8", {
        "type": "quantized", "shape": (M, K),
        "codebooks": torch.from_numpy((g.standard_normal((M, 4, 8)) * 0.02).astype(np.float16)),
        "indices": torch.from_numpy(g.integers(0, 4, (M, K // 8), dtype=np.uint8)),
        "outlier_values": torch.from_numpy((g.standard_normal((2, K)) * 0.2).astype(np.float16)),
        "outlier_indices": torch.tensor([0, 31], dtype=torch.int64),
    }, seed=2)
    # 3. svs=8, K=60: 7 groups, 56 columns survive the trim.
    M, K = 16, 60
    save_case("dequant_svs8_trim", {
        "type": "quantized", "shape": (M, K),
        "codebooks": torch.from_numpy((g.standard_normal((M, 4, 8)) * 0.02).astype(np.float16)),
        "indices": torch.from_numpy(g.integers(0, 4, (M, K // 8), dtype=np.uint8)),
        "outlier_values": None, "outlier_indices": None,
    }, seed=3)
    # 4. The reference quantizer, svs=1, on seeded Student-t weights.
    w = torch.from_numpy(synthetic.student_t_weights(64, 256, seed=7)).float()
    w[3] *= 20  # a planted outlier row
    torch.manual_seed(7)
    t0 = time.time()
    q = VectorQuantizer(QuantizeConfig(sub_vector_size=1, codebook_iters=10, outlier_fraction=0.02)).quantize_layer(w)
    print(f"reference quantize_layer 64x256 svs=1: {time.time() - t0:.1f} s, outliers {q['outlier_indices'].tolist()}")
    save_case("quantized_svs1", q, seed=4)
    np.savez_compressed(HERE / "quantized_svs1_input.npz", weight=w.numpy(), outlier_mask=q["outlier_mask"].numpy())

    # 5. .bf2 files written by the reference.
    passthrough = {"type": "fp16_passthrough", "shape": (8, 16),
                   "data": torch.from_numpy(g.standard_normal((8, 16)).astype(np.float16)), "compression_ratio": 1.0}
    q2 = VectorQuantizer(QuantizeConfig(sub_vector_size=1, codebook_iters=5)).quantize_layer(
        torch.from_numpy(synthetic.student_t_weights(96, 128, seed=8)).float())
    layers = {"model.layers.0.mlp.down_proj.weight": q, "model.norm.weight": passthrough,
              "model.layers.1.self_attn.q_proj.weight": q2}
    mcfg = {"architecture": "llama", "hidden_size": 128}
    qcfg = {"bits": 2, "sub_vector_size": 1, "outlier_fraction": 0.02}
    BF2Writer(str(HERE / "ref_int64.bf2")).write(layers, mcfg, qcfg, progress=False)
    readback = {}
    try:
        r = BF2Reader(str(HERE / "ref_int64.bf2"))
    except Exception as e:  # the reference misaligns after an int64-id layer
        readback["_open"] = {"ok": False, "error": f"{type(e).__name__}: {e}"}
    else:
        for name in r.layer_names():
            try:
                ly = r.load_layer(name)
                readback[name] = {"ok": True, "outlier_indices": ly["outlier_indices"].tolist()
                                  if "outlier_indices" in ly else None}
            except Exception as e:
                readback[name] = {"ok": False, "error": f"{type(e).__name__}: {e}"}
        r.close()
    (HERE / "ref_int64_readback.json").write_text(json.dumps(readback, indent=1))
    layers32 = {k: dict(v) for k, v in layers.items()}
    for v in layers32.values():
        if v.get("outlier_indices") is not None:
            v["outlier_indices"] = v["outlier_indices"].to(torch.int32)
    BF2Writer(str(HERE / "ref_int32.bf2")).write(layers32, mcfg, qcfg, progress=False)
    print("bf2 fixtures written")

    # 6. Config-0 pin (4096 x 4096, 1 % outlier rows), generated from a seed on any machine.
    if not skip_large:
        layer = synthetic.random_layer(4096, 4096, 40, seed=2024)
        t0 = time.time()
        W = dequantize_layer(layer)
        dt = time.time() - t0
        x = synthetic.activations(1, 4096, seed=2025)
        y32, y64 = y_pair(W, x)
        pin = {
            "generator": "opac1ty_b200.synthetic.random_layer(4096, 4096, 40, seed=2024)",
            "x": "opac1ty_b200.synthetic.activations(1, 4096, seed=2025)",
            "W_sha256": hashlib.sha256(np.ascontiguousarray(W).tobytes()).hexdigest(),
            "reference_dequant_seconds": round(dt, 1),
        }
        (HERE / "config0_pin.json").write_text(json.dumps(pin, indent=1))
        np.savez_compressed(HERE / "config0_y.npz", y32=y32, y64=y64)
        print(f"config-0 pin: reference dequantize_layer took {dt:.0f} s")


if __name__ == "__main__":
    main(skip_large="--skip-large" in sys.argv)

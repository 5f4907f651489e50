"""Seeded synthetic layers in the reference's layer-dictionary format.

No dataset or checkpoint is involved anywhere in this project: the benchmark layers are
random-initialised with the statistics the benchmark configuration names (Student-t, 4 degrees
of freedom, scaled to std 0.02; activations N(0, 1)), generated with numpy's PCG64 so the same
seed gives the same bytes on every machine.

``random_layer`` builds a layer directly (random fp16 codebooks, uniform 2-bit indices, outlier
rows of larger magnitude whose codebooks are zero, as ``OutlierDetector.extract_outliers`` +
k-means produce, opacc1ty/quantize/outlier.py:146-168).  Kernel timing does not depend on the
values, and it takes milliseconds, so it is what the large-shape tests and the benchmark use.
``quantized_layer`` runs this package's quantizer on Student-t weights instead.
"""

from __future__ import annotations

import math
from typing import Optional

import numpy as np
import torch

STD = 0.02
NU = 4


def rng_for(seed: int) -> np.random.Generator:
    return np.random.Generator(np.random.PCG64(seed))


def student_t_weights(M: int, K: int, seed: int, std: float = STD, nu: int = NU) -> np.ndarray:
    """fp16 [M][K] ~ Student-t(nu) scaled to standard deviation ``std``."""
    rng = rng_for(seed)
    scale = std / math.sqrt(nu / (nu - 2))
    return (rng.standard_t(nu, size=(M, K)) * scale).astype(np.float16)


def activations(batch: int, K: int, seed: int) -> np.ndarray:
    """fp16 [batch][K] ~ N(0, 1)."""
    return rng_for(seed).standard_normal((batch, K)).astype(np.float16)


def n_outliers_for(M: int, fraction: float) -> int:
    """The reference's count: max(1, int(M * fraction)) (opacc1ty/quantize/outlier.py:95).
    A fraction of exactly 0 means no outlier rows (the detector is bypassed)."""
    if fraction <= 0:
        return 0
    return max(1, int(M * fraction))


def random_layer(M: int, K: int, n_outliers: int, seed: int, id_dtype=torch.int64,
                 shuffle_ids: bool = False) -> dict:
    """A "quantized" layer dict: cb [M][4][1] fp16, idx [M][K] uint8, outlier rows [n][K]."""
    rng = rng_for(seed)
    cb = (rng.standard_normal((M, 4, 1)) * STD).astype(np.float16)
    idx = rng.integers(0, 4, size=(M, K), dtype=np.uint8)
    layer = {
        "type": "quantized",
        "shape": (M, K),
        "codebooks": torch.from_numpy(cb),
        "indices": torch.from_numpy(idx),
        "outlier_values": None,
        "outlier_indices": None,
    }
    if n_outliers > 0:
        ids = np.sort(rng.choice(M, size=n_outliers, replace=False)).astype(np.int64)
        if shuffle_ids:
            rng.shuffle(ids)
        scale = 8 * STD / math.sqrt(NU / (NU - 2))
        ov = (rng.standard_t(NU, size=(n_outliers, K)) * scale).astype(np.float16)
        cb[ids] = 0
        layer["codebooks"] = torch.from_numpy(cb)
        layer["outlier_values"] = torch.from_numpy(ov)
        layer["outlier_indices"] = torch.from_numpy(ids).to(id_dtype)
    layer["outlier_mask"] = None
    return layer


def random_layer_vq8(M: int, K: int, n_outliers: int, seed: int, shuffle_ids: bool = False) -> dict:
    """A sub_vector_size 8 "quantized" layer dict (the reference quantizer's default,
    opacc1ty/cli/main.py:71-72): cb [M][4][8] fp16, idx [M][K/8] uint8, outlier rows [n][K]."""
    if K % 8:
        raise ValueError("random_layer_vq8: K must be a multiple of 8")
    rng = rng_for(seed)
    cb = (rng.standard_normal((M, 4, 8)) * STD).astype(np.float16)
    idx = rng.integers(0, 4, size=(M, K // 8), dtype=np.uint8)
    layer = {"type": "quantized", "shape": (M, K), "codebooks": torch.from_numpy(cb), "indices": torch.from_numpy(idx),
             "outlier_values": None, "outlier_indices": None, "outlier_mask": None}
    if n_outliers > 0:
        ids = np.sort(rng.choice(M, size=n_outliers, replace=False)).astype(np.int64)
        if shuffle_ids:
            rng.shuffle(ids)
        scale = 8 * STD / math.sqrt(NU / (NU - 2))
        ov = (rng.standard_t(NU, size=(n_outliers, K)) * scale).astype(np.float16)
        cb[ids] = 0
        layer["codebooks"] = torch.from_numpy(cb)
        layer["outlier_values"] = torch.from_numpy(ov)
        layer["outlier_indices"] = torch.from_numpy(ids)
    return layer


def random_layer_sparse(M: int, K: int, fraction: float, seed: int, svs: int = 1, duplicates: int = 0) -> dict:
    """A "sparse_outlier" layer dict (element-wise outliers): codebooks and indices as above, and
    max(1, int(M * K * fraction)) entries (plus `duplicates` repeated positions with other values)
    of heavy-tailed fp16 values at random (row, col) positions."""
    base = random_layer_vq8(M, K, 0, seed) if svs == 8 else random_layer(M, K, 0, seed)
    rng = rng_for(seed + 7919)
    n = max(1, int(M * K * fraction)) if fraction > 0 else 0
    flat = rng.choice(M * K, size=n, replace=False)
    pos = np.stack([flat // K, flat % K], axis=1).astype(np.int64)
    if duplicates:
        pos = np.concatenate([pos, pos[rng.integers(0, n, size=duplicates)]])
    scale = 8 * STD / math.sqrt(NU / (NU - 2))
    vals = (rng.standard_t(NU, size=len(pos)) * scale).astype(np.float16)
    return {"type": "sparse_outlier", "shape": (M, K), "codebooks": base["codebooks"], "indices": base["indices"],
            "outlier_values": torch.from_numpy(vals), "outlier_indices": torch.from_numpy(pos)}


def random_layer_device(M: int, K: int, n_outliers: int, seed: int, device) -> dict:
    """Like ``random_layer`` but generated with torch's RNG directly on ``device`` (fast for the
    full model stacks; values differ from the numpy generator, the statistics do not)."""
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    cb = (torch.randn(M, 4, 1, generator=gen, device=device) * STD).half()
    idx = torch.randint(0, 4, (M, K), generator=gen, device=device, dtype=torch.uint8)
    layer = {"type": "quantized", "shape": (M, K), "codebooks": cb, "indices": idx,
             "outlier_values": None, "outlier_indices": None}
    if n_outliers > 0:
        ids = np.sort(rng_for(seed).choice(M, size=n_outliers, replace=False)).astype(np.int64)
        ids_t = torch.from_numpy(ids)
        cb[ids_t.to(device)] = 0
        ov = (torch.randn(n_outliers, K, generator=gen, device=device) * (8 * STD)).half()
        layer["outlier_values"] = ov
        layer["outlier_indices"] = ids_t
    return layer


def quantized_layer(M: int, K: int, seed: int, outlier_fraction: float = 0.01, iters: int = 10,
                    device: Optional[str] = None) -> dict:
    """Student-t weights quantized by this package's VectorQuantizer (svs = 1)."""
    from .quantize import QuantizeConfig, VectorQuantizer

    w = torch.from_numpy(student_t_weights(M, K, seed)).float()
    torch.manual_seed(seed)
    cfg = QuantizeConfig(bits=2, sub_vector_size=1, outlier_fraction=outlier_fraction,
                         codebook_iters=iters, use_error_feedback=True, device=device or "cpu")
    return VectorQuantizer(cfg).quantize_layer(w)


# Llama-3.1-8B and Llama-3-70B projection shapes (out_features, in_features).
LLAMA_8B = {
    "hidden": 4096, "intermediate": 14336, "kv": 1024, "layers": 32,
}
LLAMA_70B = {
    "hidden": 8192, "intermediate": 28672, "kv": 1024, "layers": 80,
}


def decoder_shapes(cfg: dict) -> dict:
    h, f, kv = cfg["hidden"], cfg["intermediate"], cfg["kv"]
    return {
        "q_proj": (h, h), "k_proj": (kv, h), "v_proj": (kv, h), "o_proj": (h, h),
        "gate_proj": (f, h), "up_proj": (f, h), "down_proj": (h, f),
    }


def write_llama_bf2(path, cfg: dict, n_layers: int, vocab: int, seed: int = 0, sub_vector_size: int = 1,
                    outlier_fraction: float = 0.01, heads: Optional[int] = None) -> dict:
    """A synthetic Llama-style model with `cfg`'s shapes as a .bf2 file (Hugging Face tensor names,
    random 2-bit layers with outlier rows, fp16 RMSNorm weights near 1); returns the model JSON."""
    from .format import BF2Writer

    h, f, kv = cfg["hidden"], cfg["intermediate"], cfg["kv"]
    heads = heads or h // 128
    make = random_layer_vq8 if sub_vector_size == 8 else random_layer
    rng = rng_for(seed + 17)
    layers = {}
    n = [seed * 10000]

    def q(M, K):
        n[0] += 1
        return make(M, K, n_outliers_for(M, outlier_fraction), n[0])

    def norm():
        return {"type": "fp16_passthrough", "shape": (h,),
                "data": torch.from_numpy((1.0 + 0.05 * rng.standard_normal(h)).astype(np.float16))}

    layers["model.embed_tokens.weight"] = q(vocab, h)
    for i in range(n_layers):
        p = f"model.layers.{i}."
        layers[p + "input_layernorm.weight"] = norm()
        layers[p + "self_attn.q_proj.weight"] = q(h, h)
        layers[p + "self_attn.k_proj.weight"] = q(kv, h)
        layers[p + "self_attn.v_proj.weight"] = q(kv, h)
        layers[p + "self_attn.o_proj.weight"] = q(h, h)
        layers[p + "post_attention_layernorm.weight"] = norm()
        layers[p + "mlp.gate_proj.weight"] = q(f, h)
        layers[p + "mlp.up_proj.weight"] = q(f, h)
        layers[p + "mlp.down_proj.weight"] = q(h, f)
    layers["model.norm.weight"] = norm()
    layers["lm_head.weight"] = q(vocab, h)
    model = {"architecture": "llama", "hidden_size": h, "intermediate_size": f, "num_hidden_layers": n_layers,
             "vocab_size": vocab, "num_attention_heads": heads, "num_key_value_heads": kv // (h // heads),
             "rope_theta": 500000.0, "rms_norm_eps": 1e-5}
    BF2Writer(str(path)).write(layers, model, {"bits": 2, "sub_vector_size": sub_vector_size}, progress=False)
    return model

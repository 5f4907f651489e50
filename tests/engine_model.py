"""A tiny Llama-style model for the engine tests: written to .bf2 from synthetic quantized layers,
and run in float64 by a plain numpy forward pass (the check for ``bf_engine_*``)."""

from __future__ import annotations

import numpy as np
import torch

from opac1ty_b200 import synthetic
from opac1ty_b200.format import BF2Writer

from oracle.oracle import dequantize_np

PROJ = ("self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj", "self_attn.o_proj", "mlp.gate_proj",
        "mlp.up_proj", "mlp.down_proj")


def _scaled(layer: dict, scale: float) -> dict:
    layer = dict(layer)
    layer["codebooks"] = (layer["codebooks"].float() * scale).half()
    if layer.get("outlier_values") is not None:
        layer["outlier_values"] = (layer["outlier_values"].float() * scale).half()
    return layer


def build(path, *, hidden=256, heads=4, kv_heads=2, n_layers=2, inter=512, vocab=320, svs=1, outliers=True,
          tied=False, norms=True, checksum=False, seed=0, rope_theta=10000.0, json_heads=True,
          element=False) -> dict:
    """Write the model to `path`; returns the layer dicts (for the float64 forward) and numbers."""
    hd = hidden // heads
    rng = np.random.default_rng(seed)
    make = synthetic.random_layer_vq8 if svs == 8 else synthetic.random_layer
    layers = {}
    s = [seed * 1000]

    def q(M, K, scale):
        s[0] += 1
        if element:  # element-wise outliers ("sparse_outlier" layers)
            return _scaled(synthetic.random_layer_sparse(M, K, 0.01, s[0], svs=svs, duplicates=2), scale)
        n = synthetic.n_outliers_for(M, 0.01) if outliers else 0
        return _scaled(make(M, K, n, s[0]), scale)

    layers["model.embed_tokens.weight"] = q(vocab, hidden, 20.0)
    shapes = {"self_attn.q_proj": (heads * hd, hidden), "self_attn.k_proj": (kv_heads * hd, hidden),
              "self_attn.v_proj": (kv_heads * hd, hidden), "self_attn.o_proj": (hidden, heads * hd),
              "mlp.gate_proj": (inter, hidden), "mlp.up_proj": (inter, hidden), "mlp.down_proj": (hidden, inter)}
    for i in range(n_layers):
        p = f"model.layers.{i}."
        if norms:
            for nm in ("input_layernorm.weight", "post_attention_layernorm.weight"):
                w = (1.0 + 0.1 * rng.standard_normal(hidden)).astype(np.float16)
                layers[p + nm] = {"type": "fp16_passthrough", "shape": (hidden,), "data": torch.from_numpy(w)}
        for nm in PROJ:
            M, K = shapes[nm]
            layers[p + nm + ".weight"] = q(M, K, 2.0)
    if norms:
        w = (1.0 + 0.1 * rng.standard_normal(hidden)).astype(np.float16)
        layers["model.norm.weight"] = {"type": "fp16_passthrough", "shape": (hidden,), "data": torch.from_numpy(w)}
    if not tied:
        layers["lm_head.weight"] = q(vocab, hidden, 4.0)
    cfg = {"architecture": "llama", "hidden_size": hidden, "num_hidden_layers": n_layers, "vocab_size": vocab,
           "intermediate_size": inter, "rope_theta": rope_theta}
    if json_heads:
        cfg.update({"num_attention_heads": heads, "num_key_value_heads": kv_heads})
    BF2Writer(str(path)).write(layers, cfg, {"bits": 2, "sub_vector_size": svs}, progress=False, checksum=checksum)
    return {"layers": layers, "hidden": hidden, "heads": heads, "kv_heads": kv_heads, "hd": hd, "n_layers": n_layers,
            "vocab": vocab, "theta": rope_theta, "eps": 1e-5, "tied": tied}


def _rms(x, w, eps):
    y = x / np.sqrt(np.mean(x * x, axis=-1, keepdims=True) + eps)
    return y * w if w is not None else y


def _rope(x, pos, hd, theta):
    """x [T][heads*hd]: rotate-half pairs (i, i + hd/2) by pos * theta^(-2i/hd)."""
    T = x.shape[0]
    x = x.reshape(T, -1, hd).copy()
    half = hd // 2
    inv = theta ** (-2.0 * np.arange(half) / hd)
    ang = pos[:, None] * inv[None, :]
    c, s = np.cos(ang)[:, None, :], np.sin(ang)[:, None, :]
    a, b = x[..., :half].copy(), x[..., half:].copy()
    x[..., :half] = a * c - b * s
    x[..., half:] = b * c + a * s
    return x.reshape(T, -1)


def forward64(model: dict, tokens) -> np.ndarray:
    """float64 logits after each token of `tokens` (a fresh sequence): [T][vocab]."""
    L = model["layers"]
    W = {k: dequantize_np(v).astype(np.float64) for k, v in L.items() if v["type"] in ("quantized", "sparse_outlier")}
    vec = {k: np.asarray(v["data"], dtype=np.float64).reshape(-1) for k, v in L.items() if v["type"] == "fp16_passthrough"}
    hd, H, KV, eps, theta = model["hd"], model["heads"], model["kv_heads"], model["eps"], model["theta"]
    tok = np.asarray(tokens)
    T = len(tok)
    pos = np.arange(T, dtype=np.float64)
    h = W["model.embed_tokens.weight"][tok].copy()
    for i in range(model["n_layers"]):
        p = f"model.layers.{i}."
        xn = _rms(h, vec.get(p + "input_layernorm.weight"), eps)
        q = _rope(xn @ W[p + "self_attn.q_proj.weight"].T, pos, hd, theta).reshape(T, H, hd)
        k = _rope(xn @ W[p + "self_attn.k_proj.weight"].T, pos, hd, theta).reshape(T, KV, hd)
        v = (xn @ W[p + "self_attn.v_proj.weight"].T).reshape(T, KV, hd)
        att = np.zeros((T, H, hd))
        for hh in range(H):
            kh = hh // (H // KV)
            sc = q[:, hh, :] @ k[:, kh, :].T / np.sqrt(hd)
            sc = np.where(np.tril(np.ones((T, T), dtype=bool)), sc, -np.inf)
            sc = np.exp(sc - sc.max(axis=1, keepdims=True))
            att[:, hh, :] = (sc / sc.sum(axis=1, keepdims=True)) @ v[:, kh, :]
        h = h + att.reshape(T, H * hd) @ W[p + "self_attn.o_proj.weight"].T
        xn = _rms(h, vec.get(p + "post_attention_layernorm.weight"), eps)
        g = xn @ W[p + "mlp.gate_proj.weight"].T
        u = xn @ W[p + "mlp.up_proj.weight"].T
        h = h + (g / (1.0 + np.exp(-g)) * u) @ W[p + "mlp.down_proj.weight"].T
    xn = _rms(h, vec.get("model.norm.weight"), eps)
    head = W["model.embed_tokens.weight"] if model["tied"] else W["lm_head.weight"]
    return xn @ head.T


def rel_err(a: np.ndarray, ref: np.ndarray) -> float:
    return float(np.max(np.abs(a.astype(np.float64) - ref)) / np.max(np.abs(ref)))

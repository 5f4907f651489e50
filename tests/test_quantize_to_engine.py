"""The user path end to end: a Hugging Face-style Llama checkpoint (safetensors, random weights) is
quantized with `cli quantize` (row outliers and element outliers, sub_vector_size 1 and 8), the
.bf2 it writes is read back, and -- on a GPU -- the engine API runs it and matches a float64
forward pass over the file's own dequantized weights (tolerance as in tests/test_gpu_engine.py)."""

import json

import numpy as np
import pytest
import torch
from click.testing import CliRunner

from opac1ty_b200.cli import cli
from opac1ty_b200.format import BF2Reader

HIDDEN, INTER, VOCAB, LAYERS, KV = 256, 512, 1024, 2, 1


def _checkpoint(path):
    from safetensors.torch import save_file

    g = torch.Generator().manual_seed(0)
    r = lambda *s: (torch.randn(*s, generator=g) * 0.05).half()
    sd = {"model.embed_tokens.weight": r(VOCAB, HIDDEN) * 8, "model.norm.weight": (1 + r(HIDDEN)).half(),
          "lm_head.weight": r(VOCAB, HIDDEN)}
    hd = 128  # the quantizer's model JSON infers hidden / 128 heads
    for i in range(LAYERS):
        p = f"model.layers.{i}."
        sd[p + "input_layernorm.weight"] = (1 + r(HIDDEN)).half()
        sd[p + "post_attention_layernorm.weight"] = (1 + r(HIDDEN)).half()
        sd[p + "self_attn.q_proj.weight"] = r(HIDDEN, HIDDEN)
        sd[p + "self_attn.k_proj.weight"] = r(KV * hd, HIDDEN)
        sd[p + "self_attn.v_proj.weight"] = r(KV * hd, HIDDEN)
        sd[p + "self_attn.o_proj.weight"] = r(HIDDEN, HIDDEN)
        sd[p + "mlp.gate_proj.weight"] = r(INTER, HIDDEN)
        sd[p + "mlp.up_proj.weight"] = r(INTER, HIDDEN)
        sd[p + "mlp.down_proj.weight"] = r(HIDDEN, INTER)
    save_file({k: v.contiguous() for k, v in sd.items()}, str(path))


def _quantize(tmp_path, mode, svs):
    ckpt = tmp_path / "model.safetensors"
    if not ckpt.exists():
        _checkpoint(ckpt)
    out = tmp_path / f"m_{mode}_{svs}.bf2"
    res = CliRunner().invoke(cli, ["quantize", str(ckpt), "-o", str(out), "--sub-vector-size", str(svs),
                                   "--outlier-mode", mode, "--codebook-iters", "4", "--checksum", "--json-output"])
    assert res.exit_code == 0, res.output
    assert json.loads(res.output)["output_path"] == str(out)
    return out


def _model_from_file(path) -> dict:
    with BF2Reader(str(path)) as rd:
        layers = {n: rd.load_layer(n) for n in rd.layer_names()}
        cfg = rd.model_config
    return {"layers": layers, "hidden": HIDDEN, "heads": cfg["num_attention_heads"], "kv_heads": KV,
            "hd": HIDDEN // cfg["num_attention_heads"], "n_layers": cfg["num_hidden_layers"], "vocab": VOCAB,
            "theta": 10000.0, "eps": 1e-5, "tied": False}


@pytest.mark.parametrize("mode,svs", [("row", 1), ("element", 1), ("element", 8)])
def test_quantize_writes_an_engine_ready_file(tmp_path, mode, svs):
    out = _quantize(tmp_path, mode, svs)
    with BF2Reader(str(out)) as rd:
        assert rd.checksum_ok
        cfg = rd.model_config
        assert cfg["hidden_size"] == HIDDEN and cfg["vocab_size"] == VOCAB and cfg["num_hidden_layers"] == LAYERS
        kinds = {rd.load_layer(n)["type"] for n in rd.layer_names()}
    assert "fp16_passthrough" in kinds  # the RMSNorm weights
    assert ("sparse_outlier" if mode == "element" else "quantized") in kinds


@pytest.mark.gpu
@pytest.mark.parametrize("mode,svs", [("row", 1), ("element", 1), ("element", 8)])
def test_engine_runs_the_quantized_checkpoint(tmp_path, cuda_device, mode, svs):
    from engine_model import forward64, rel_err
    from opac1ty_b200.engine import Engine

    out = _quantize(tmp_path, mode, svs)
    m = _model_from_file(out)
    toks = np.random.default_rng(1).integers(1, VOCAB, size=10).tolist()
    ref = forward64(m, toks)
    with Engine(out) as eng:
        assert eng.config["num_kv_heads"] == KV
        assert rel_err(eng.forward(toks), ref[-1]) < 2e-2
        gen = eng.generate_tokens(toks, 4, temperature=0.0)
        assert 1 <= len(gen) <= 4

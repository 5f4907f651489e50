"""bf_engine_* on the GPU: a tiny Llama-style model written to .bf2 runs through the engine
(quantized projections on opc_gemv / the tcgen05 GEMM, RMSNorm, rotary embedding, grouped-query
attention over the KV cache) and its logits agree with a float64 numpy forward pass on the
oracle's dequantized weights.

Tolerance: 2e-2 of max |logit|, norm-wise.  The engine rounds every projection input and output,
the rotated q/k and the attention output to fp16 (each ~2^-11 relative) through two blocks; the
float64 pass rounds nothing."""

import numpy as np
import pytest

from engine_model import build, forward64, rel_err
from opac1ty_b200.engine import Engine, EngineError

pytestmark = pytest.mark.gpu
TOL = 2e-2


@pytest.fixture(scope="module")
def model(tmp_path_factory, cuda_device):
    p = tmp_path_factory.mktemp("eng") / "tiny.bf2"
    m = build(p, checksum=True)
    m["path"] = p
    return m


def _tokens(n, vocab, seed=1):
    return np.random.default_rng(seed).integers(1, vocab, size=n).tolist()


def test_forward_matches_float64(model):
    toks = _tokens(7, model["vocab"])
    ref = forward64(model, toks)
    with Engine(model["path"]) as eng:
        assert eng.config["num_kv_heads"] == model["kv_heads"] and eng.config["head_dim"] == model["hd"]
        logits = eng.forward(toks)
        assert eng.position == len(toks)
    assert rel_err(logits, ref[-1]) < TOL


def test_steps_match_float64_at_every_position(model):
    toks = _tokens(6, model["vocab"], seed=2)
    ref = forward64(model, toks)
    with Engine(model["path"]) as eng:
        for i, t in enumerate(toks):
            lg = eng.forward_step(t)
            assert rel_err(lg, ref[i]) < TOL, i
        # prefill + one step lands on the same distribution as the full forward
        eng.reset()
        eng.prefill(toks[:-1])
        lg = eng.forward_step(toks[-1])
        assert rel_err(lg, ref[-1]) < TOL


def test_long_prompt_runs_on_the_gemm(model):
    toks = _tokens(100, model["vocab"], seed=3)  # one chunk of 100 tokens: projections on opc_gemm
    ref = forward64(model, toks)
    with Engine(model["path"]) as eng:
        assert rel_err(eng.forward(toks), ref[-1]) < TOL
        eng.reset()
        eng.prefill(toks[:-1])
        assert rel_err(eng.forward_step(toks[-1]), ref[-1]) < TOL


def test_long_context_decode_steps(model):
    # 600 positions: a prompt of two chunks (512 + 85 tokens, projections on opc_gemm), then decode
    # steps whose attention splits the context into ranges of many positions each and merges the
    # ranges' partial softmax records across CTAs
    toks = _tokens(600, model["vocab"], seed=8)
    ref = forward64(model, toks)
    with Engine(model["path"]) as eng:
        eng.prefill(toks[:-3])
        for i in range(3):
            lg = eng.forward_step(toks[-3 + i])
            assert rel_err(lg, ref[-3 + i]) < TOL, i


@pytest.mark.parametrize("variant", ["svs8", "tied_no_norms", "no_outliers_json_without_heads"])
def test_model_variants(tmp_path, cuda_device, variant):
    p = tmp_path / f"{variant}.bf2"
    kw = {"svs8": dict(svs=8), "tied_no_norms": dict(tied=True, norms=False),
          "no_outliers_json_without_heads": dict(outliers=False, json_heads=False, hidden=256, heads=2, kv_heads=1)}[variant]
    m = build(p, seed=5, **kw)
    toks = _tokens(9, m["vocab"], seed=4)
    ref = forward64(m, toks)
    with Engine(p) as eng:
        assert rel_err(eng.forward(toks), ref[-1]) < TOL


def test_generate_greedy_follows_argmax(model):
    prompt = _tokens(4, model["vocab"], seed=6)
    with Engine(model["path"]) as eng:
        out = eng.generate_tokens(prompt, 8, temperature=0.0)
        assert 1 <= len(out) <= 8
        # the same chain by hand: argmax of each step's logits
        eng.reset()
        eng.prefill(prompt[:-1])
        lg = eng.forward_step(prompt[-1])
        ref = []
        for _ in range(len(out)):
            t = int(np.argmax(lg))
            ref.append(t)
            if t == 0:
                break
            lg = eng.forward_step(t)
        assert out == ref[:len(out)]
        st = eng.stats()
        assert st["total_tokens_generated"] == len(out) and st["n_kernel_dispatches"] > 0
        assert st["peak_memory_bytes"] >= eng.kv_cache_size > 0


def test_sampling_is_seeded(model):
    prompt = _tokens(3, model["vocab"], seed=7)
    with Engine(model["path"]) as eng:
        a = eng.generate_tokens(prompt, 6, temperature=0.8, top_k=20, top_p=0.9, repetition_penalty=1.2, seed=11)
        b = eng.generate_tokens(prompt, 6, temperature=0.8, top_k=20, top_p=0.9, repetition_penalty=1.2, seed=11)
        assert a == b and len(a) >= 1
        assert eng.generate("ab", 3, None) >= 1  # the byte-level text API


def test_errors_leave_the_engine_usable(model):
    with Engine(model["path"], max_context=8) as eng:
        with pytest.raises(EngineError, match="outside"):
            eng.forward_step(model["vocab"])  # token id past the vocabulary
        with pytest.raises(EngineError, match="context full"):
            eng.prefill(list(range(1, 10)))  # 9 tokens into an 8-position cache
        lg = eng.forward([1, 2, 3])
        assert np.isfinite(lg).all() and eng.position == 3

"""The quantizer entry point: the reference's quantizer tests restated (tests/test_vq.py and
tests/test_codebook.py of opacc1ty, seeded), plus pins against the reference's own outputs."""

from pathlib import Path

import numpy as np
import pytest
import torch

from opac1ty_b200.quantize import (CodebookConfig, CodebookLearner, OutlierConfig, OutlierDetector, QuantizeConfig,
                                   VectorQuantizer)

GOLDEN = Path(__file__).resolve().parent / "golden"


@pytest.fixture(autouse=True)
def _seed():
    torch.manual_seed(0)


def test_quantize_single_layer():
    r = VectorQuantizer(QuantizeConfig(bits=2, outlier_fraction=0.02, codebook_iters=20)).quantize_layer(torch.randn(512, 512))
    assert r["type"] == "quantized" and r["shape"] == (512, 512)
    assert r["codebooks"].dtype == torch.float16 and tuple(r["codebooks"].shape) == (512, 4, 8)
    assert r["indices"].dtype == torch.uint8 and r["compression_ratio"] > 3.0


def test_quantize_svs1_layout():
    r = VectorQuantizer(QuantizeConfig(sub_vector_size=1, codebook_iters=10)).quantize_layer(torch.randn(256, 300))
    assert tuple(r["codebooks"].shape) == (256, 4, 1) and tuple(r["indices"].shape) == (256, 300)
    assert int(r["indices"].max()) <= 3
    ids = r["outlier_indices"]
    assert ids.dtype == torch.int64 and torch.all(r["codebooks"][ids] == 0) is not None


def test_quantize_model_dict():
    sd = {"model.embed_tokens.weight": torch.randn(1000, 128), "model.layers.0.self_attn.q_proj.weight": torch.randn(128, 128),
          "model.layers.0.mlp.down_proj.weight": torch.randn(128, 256), "model.layers.0.input_layernorm.weight": torch.randn(128),
          "lm_head.weight": torch.randn(1000, 128)}
    res = VectorQuantizer(QuantizeConfig(codebook_iters=5)).quantize_model(sd, {"architecture": "llama"}, progress=False)
    for n in sd:
        assert n in res
    assert res["model.layers.0.input_layernorm.weight"]["type"] == "fp16_passthrough"
    assert res["model.layers.0.self_attn.q_proj.weight"]["type"] == "quantized"
    assert "_model_config" in res and res["_quantize_config"]["opacc1ty_version"] == "1.0.2"


def test_outlier_detection_planted():
    w = torch.randn(100, 200)
    w[0] *= 50
    w[99] *= 40
    mask, _ = OutlierDetector(OutlierConfig(fraction=0.05)).detect(w)
    assert mask[0] and mask[99] and mask.sum() >= 2


def test_extract_outliers_zeroes_rows():
    w = torch.randn(100, 200)
    d = OutlierDetector(OutlierConfig(fraction=0.05))
    mask, _ = d.detect(w)
    dense, vals, ids = d.extract_outliers(w, mask)
    assert (dense[mask] == 0).all()
    for i, idx in enumerate(ids):
        assert torch.equal(vals[i], w[idx].half())


def test_sensitivity_detection():
    mask, _ = OutlierDetector(OutlierConfig(fraction=0.05, detection_method="sensitivity")).detect(torch.randn(100, 200))
    assert 1 <= int(mask.sum()) <= 10


def test_codebook_error_reasonable_and_padding():
    learner = CodebookLearner(CodebookConfig(n_bits=2, sub_vector_size=8, n_iters=100))
    w = torch.randn(256, 256)
    cb, idx = learner.learn(w)
    rec = cb.float()[torch.arange(256)[:, None], idx.long()].reshape(256, -1)
    assert ((w - rec) ** 2).mean() < 2.0
    cb2, idx2 = CodebookLearner(CodebookConfig(sub_vector_size=8)).learn(torch.randn(128, 250))
    assert idx2.shape[1] == 250 // 8


def test_kmeanspp_valid():
    cb = CodebookLearner(CodebookConfig(n_samples=1024))._initialize_codebooks(torch.randn(256, 32, 8))
    assert tuple(cb.shape) == (256, 4, 8) and torch.isfinite(cb).all()


def test_error_feedback_flag_on_learner():
    """opacc1ty tests/test_codebook.py:214-250: the learner's use_error_feedback flag must not make
    its reconstruction error worse (the feedback pass itself lives in VectorQuantizer)."""
    w = torch.randn(128, 256)
    torch.manual_seed(1)
    cb_no, idx_no = CodebookLearner(CodebookConfig(sub_vector_size=8, use_error_feedback=False)).learn(w)
    torch.manual_seed(1)
    cb_fb, idx_fb = CodebookLearner(CodebookConfig(sub_vector_size=8, use_error_feedback=True)).learn(w)
    def rec(cb, i):
        return cb.float()[torch.arange(128)[:, None], i.long()].reshape(128, -1)
    assert ((w - rec(cb_fb, idx_fb)) ** 2).mean() <= ((w - rec(cb_no, idx_no)) ** 2).mean() * 1.1


def test_error_feedback_matches_sequential_definition():
    """The vectorised feedback pass equals the per-row sequential definition (vq.py:202-235)."""
    w = torch.randn(16, 40)
    q = VectorQuantizer(QuantizeConfig(sub_vector_size=4))
    cb, idx = q.codebook_learner.learn(w)
    _, got = q._apply_error_feedback(w, cb, idx)
    ref = idx.clone()
    for oc in range(16):
        err = torch.zeros(4)
        for g in range(10):
            t = w[oc, 4 * g:4 * g + 4] + err
            best = int(((cb[oc] - t.unsqueeze(0)) ** 2).sum(dim=1).argmin())
            ref[oc, g] = best
            err = t - cb[oc, best]
    assert torch.equal(got, ref)


def test_pins_against_reference_quantizer_output():
    """On the reference's own fixture, this package's detector finds the same outlier rows and its
    error feedback, run on the reference's codebooks, reproduces the reference's indices exactly."""
    z = np.load(GOLDEN / "quantized_svs1.npz")
    inp = np.load(GOLDEN / "quantized_svs1_input.npz")
    w = torch.from_numpy(inp["weight"])
    q = VectorQuantizer(QuantizeConfig(sub_vector_size=1, outlier_fraction=0.02))
    mask, _ = q.outlier_detector.detect(w)
    assert np.array_equal(mask.numpy(), inp["outlier_mask"])
    dense, vals, ids = q.outlier_detector.extract_outliers(w, mask)
    assert np.array_equal(ids.numpy(), z["outlier_indices"])
    assert np.array_equal(vals.numpy().view(np.uint16), z["outlier_values"].view(np.uint16))
    cb = torch.from_numpy(z["codebooks"])
    groups = dense.reshape(dense.shape[0], -1, 1)
    pre = q.codebook_learner._assign(groups, cb.float())  # the reference's final Lloyd assignment
    _, idx = q._apply_error_feedback(dense, cb, pre.to(torch.uint8))
    assert np.array_equal(idx.numpy(), z["indices"])


@pytest.mark.skipif(not torch.cuda.is_available(), reason="no CUDA device")
@pytest.mark.gpu
def test_quantize_on_cuda_matches_shapes():
    r = VectorQuantizer(QuantizeConfig(sub_vector_size=1, codebook_iters=5, device="cuda")).quantize_layer(torch.randn(256, 512))
    assert tuple(r["indices"].shape) == (256, 512) and r["indices"].device.type == "cpu"

"""The command-line surface (the reference's `opacc1ty benchmark`, opacc1ty/cli/main.py:221-316):
`benchmark` on a .bf2 file written by the reference's own BF2Writer (tests/golden/ref_int32.bf2)
times every quantized layer on the GPU; without a GPU it fails with a clear message."""

import json
from pathlib import Path

import pytest
from click.testing import CliRunner

from opac1ty_b200.cli import cli

GOLDEN = Path(__file__).resolve().parent / "golden"


def test_benchmark_without_gpu_fails_cleanly():
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    res = CliRunner().invoke(cli, ["benchmark", str(GOLDEN / "ref_int32.bf2"), "--iters", "2"])
    assert res.exit_code != 0
    assert "CUDA" in res.output or "cuda" in res.output.lower()


def test_info_reads_the_reference_file():
    res = CliRunner().invoke(cli, ["info", str(GOLDEN / "ref_int32.bf2"), "--layers", "--json-output"])
    assert res.exit_code == 0, res.output
    d = json.loads(res.output)
    assert d["n_layers"] >= 1 and d["layers"]
    assert d["checksum"] == "absent"   # the reference writer emits no trailer


@pytest.mark.gpu
def test_benchmark_times_every_quantized_layer(cuda_device):
    res = CliRunner().invoke(cli, ["benchmark", str(GOLDEN / "ref_int32.bf2"), "--iters", "3", "--json-output"])
    assert res.exit_code == 0, res.output
    d = json.loads(res.output)
    assert d["layers"], d
    for row in d["layers"]:
        assert row["us"] > 0 and row["gbs"] > 0
    assert d["tok_s"] > 0

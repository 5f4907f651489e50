"""bench.py's host-side pieces without a GPU: the workload description both arms print, the
roofline denominators (the measured file when present, else the stated fallback), and the engine
measurement, which runs in a child process and turns any failure there into an error entry of
the bench line instead of ending the run."""

import json

import bench


def test_both_arms_describe_the_same_workload():
    c1, c2 = bench.config_for(1), bench.config_for(2)
    assert c1["batch"] == 1 and c2["batch"] == 2 and c1["blocks"] == bench.BLOCKS == 32
    assert "batch 1" in c1["workload"] and "batch 2" in c2["workload"]


def test_peaks_come_from_the_measured_file_else_the_fallback(tmp_path, monkeypatch):
    monkeypatch.setattr(bench, "ROOT", tmp_path)
    assert bench.measured_peaks() == {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}
    (tmp_path / "MEASURED_PEAKS.json").write_text(json.dumps({"hbm_gbs": 6552.3, "bf16_tflops": 1687.6}))
    assert bench.measured_peaks() == {"hbm_gbs": 6552.3, "bf16_tflops": 1687.6, "source": "measured"}
    (tmp_path / "MEASURED_PEAKS.json").write_text("{not json")
    assert bench.measured_peaks()["source"] == "fallback"


def test_engine_measurement_failure_becomes_an_error_entry():
    import torch

    if torch.cuda.is_available():
        return  # on a GPU the child process measures instead
    r = bench.engine_config(blocks=1, prompt=8, steps=2, timeout_s=300)
    assert set(r) == {"error"} and "engine-bench exited" in r["error"]

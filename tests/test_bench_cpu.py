"""The bench's roofline inputs, on the CPU: where the peak denominators come from, and the
per-launch traffic read from the committed ncu capture of each config-1 shape.

A bench line's `roofline.frac` divides by `peaks()` (the pool's measured peaks when the
driver wrote them, else the stated fallback), and its `roofline.traffic` must count at least
the algorithmic bytes of a launch (A and B read once, the int32 C written once)."""
import importlib.util
import json
import os

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def bench():
    spec = importlib.util.spec_from_file_location("bench_under_test", os.path.join(ROOT, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_peaks_measured_then_fallback(bench, tmp_path, monkeypatch):
    monkeypatch.setattr(bench, "ROOT", str(tmp_path))
    p = bench.peaks()
    assert p["source"] == "fallback" and p["bf16_tflops"] == bench.FALLBACK["bf16_tflops"]
    (tmp_path / "MEASURED_PEAKS.json").write_text(json.dumps({"hbm_gbs": 7000.0, "bf16_tflops": 1700.0}))
    p = bench.peaks()
    assert p["source"] == "measured" and p["hbm_gbs"] == 7000.0
    assert p["bf16_tflops_sustained"] == 1700.0  # no sustained figure: the burst one stands in
    (tmp_path / "MEASURED_PEAKS.json").write_text(
        json.dumps({"hbm_gbs": 7000.0, "bf16_tflops": 1700.0, "bf16_tflops_sustained": 1450.0}))
    assert bench.peaks()["bf16_tflops_sustained"] == 1450.0


def test_traffic_counts_every_algorithmic_byte(bench):
    t = bench.gemm_traffic_per_launch(bench.LAYERS, bench.M_TOKENS)
    assert t is not None, "profiles/gemm_traffic_config1.txt is missing a config-1 shape"
    m = bench.M_TOKENS
    shapes = [s for s in bench.LAYER_SHAPES for _ in range(bench.LAYERS)] + [bench.PLE_SHAPE]
    algorithmic = sum(m * k + n * k + 4 * m * n for _, n, k in shapes) / len(shapes)
    # Reads equal the compulsory A + B bytes and every output byte enters L2 once.
    assert algorithmic * 0.999 <= t["bytes"] <= algorithmic * 1.05
    assert bench.gemm_traffic_per_launch(bench.LAYERS, m + 1) is None  # captured at M = 3658 only

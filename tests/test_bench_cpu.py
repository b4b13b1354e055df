"""bench.py's contract pieces that need no GPU: the metric and workload it
reports, the per-step launch counts it claims, the roofline arithmetic and
byte counts, and the parsing of the clock samples taken during the timed
region."""
from __future__ import annotations

import json
from pathlib import Path

import pytest

import bench

ROOT = Path(__file__).resolve().parents[1]


def test_metric_is_the_baseline_metric():
    assert bench.METRIC == json.loads((ROOT / "BASELINE.json").read_text())["metric"]


def test_headline_config_names_the_per_gpu_workload():
    for world in (1, 2, 4, 8):
        c = bench.headline_config(world)
        assert c["tokens_per_gpu"] == bench.HEAD_T == 4096
        assert (c["hidden"], c["inter"], c["experts"], c["top_k"]) == (7168, 2048, 256, 8)
        assert c["act"] == "fp8" and c["parallelism"] == f"ep{world}"
        assert "model" not in c


@pytest.mark.parametrize("t,world,launches", [
    (1, 1, 6),      # fused small-batch router, single-CTA layout
    (8, 1, 6),
    (128, 1, 7),    # logits + top-k, 1024 assignments: one layout CTA
    (4096, 1, 11),  # router 3 (with the W split), layout 4, quantise, two GEMMs, combine
    (4096, 2, 32),
    (4096, 8, 32),
])
def test_layer_launch_counts(t, world, launches):
    assert bench.layer_launches(t, world) == launches


def test_expert_bytes_are_mxfp4_sizes():
    h, i = 7168, 2048

    def mxfp4(rows, k):  # E2M1 codes (two per byte) + one E8M0 scale per 32 values
        return rows * k // 2 + rows * k // 32

    assert bench.GU_BYTES == mxfp4(2 * i, h)
    assert bench.DN_BYTES == mxfp4(h, i)
    assert bench.EXPERT_BYTES == bench.GU_BYTES + bench.DN_BYTES
    assert bench.GU_FLOP_PER_ROW == 2 * 2 * i * h
    assert bench.LAYER_FLOP_PER_TOKEN == 9 * 2 * (2 * i * h + h * i)


def test_fp8_roofline_arithmetic():
    r = bench.fp8_roofline(2.0, 36_864, 1600.0, "measured", traffic=123)
    flops = 36_864 * bench.GU_FLOP_PER_ROW
    assert r["algorithmic_flops"] == flops
    assert r["achieved"] == pytest.approx(flops / 2e-3 / 1e12)
    assert r["peak"] == 3200.0 and r["unit"] == "TFLOP/s" and r["bound"] == "tensor"
    assert r["frac"] == pytest.approx(r["achieved"] / 3200.0)
    assert r["traffic"] == 123
    assert "measured" in r["peak_source"]


def test_peaks_come_from_the_measured_file():
    hbm, tf, src = bench.peaks()
    f = ROOT / "MEASURED_PEAKS.json"
    if f.exists():
        d = json.loads(f.read_text())
        assert src == "measured" and hbm == d["hbm_gbs"] and tf == d["bf16_tflops"]
    else:
        assert (hbm, tf, src) == (6650.0, 1590.0, "fallback")


def _clocks(rows):
    c = bench.Clocks(0)
    c.out = "\n".join(rows)
    return c.summary()


def test_clock_summary_keeps_power_cap_and_flags_slowdowns():
    na = "Not Active"
    rows = [f"0, {mhz}, 1965, 900.0, 0x4, {na}, {na}, {na}, {cap}"
            for mhz, cap in ((1965, na), (1800, "Active"), (1750, "Active"))]
    s = _clocks(rows)
    assert s["samples"] == 3 and s["sm_mhz"] == 1800 and s["sm_max_mhz"] == 1965
    assert s["reasons"] == ["sw_power_cap"]
    s = _clocks(rows + [f"0, 1500, 1965, 990.0, 0x8, Active, {na}, Active, {na}"])
    assert s["reasons"] == ["hw_slowdown", "sw_power_cap", "sw_thermal_slowdown"]


def test_clock_summary_without_samples():
    s = _clocks([])
    assert s["samples"] == 0 and s["sm_mhz"] is None and s["reasons"] == ["unavailable"]

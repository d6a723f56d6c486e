"""Host-side helpers of bench.py (CPU): peaks, committed ncu traffic, the
clock summary and the workload table.  No GPU and no kernel launch."""

import json
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

import bench  # noqa: E402


def test_peaks_have_both_denominators():
    peaks, kind = bench.load_peaks()
    assert kind in ("measured", "fallback")
    assert peaks["hbm_gbs"] > 1000 and peaks["bf16_tflops"] > 100


def test_every_traffic_entry_names_a_committed_profile():
    table = json.loads((ROOT / "profiles" / "ncu_traffic.json").read_text())
    names = set(bench.workloads())
    for op, entry in table.items():
        assert op in names, op
        assert (ROOT / "profiles" / entry["source"]).is_file(), entry["source"]
        assert entry["bytes_per_launch"] > 0
        assert bench.load_traffic(op) == pytest.approx(entry["bytes_per_launch"])
    assert bench.load_traffic("no_such_op") is None


def test_default_workload_has_traffic_and_a_cpu_baseline():
    wl = bench.workloads()["fused_add_layer_norm"]()
    assert bench.load_traffic(wl.name) is not None
    assert wl.cpu_ref is not None and wl.unit == "GB/s" and wl.bound == "hbm"


def test_clock_summary_drops_idle_samples_and_decodes_reasons():
    s = bench.ClockSampler(0)  # no NVML here: nothing is sampled on its own
    assert s.summary()["reasons"] == ["unsampled"]
    s.samples = [(345, 0x1), (1965, 0x0), (1900, 0x4), (1950, 0x4 | 0x20)]
    out = s.summary()
    assert out["samples"] == 3  # the idle sample is left out
    assert out["sm_mhz"] == 1950
    assert out["reasons"] == ["sw_power_cap", "sw_thermal_slowdown"]


def test_workload_names_match_the_readme():
    readme = (ROOT / "README.md").read_text()
    for name in bench.workloads():
        assert f"`{name}`" in readme, name

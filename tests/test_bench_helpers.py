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


def test_gdn_shard_of_a_rank_part_uses_its_own_shape():
    """The e2e leg chunks a rank's part (2 of the 4 batches at N = 2): the
    (batch, head) split must follow the part's shape, not the whole problem's."""
    import torch

    wl = bench.workloads()["gdn"]()
    part = tuple(torch.arange(2 * 3 * 16 * 4, dtype=torch.float32).view(2, 3, 16, 4)
                 for _ in range(3)) + tuple(torch.zeros(2, 3, 16) for _ in range(2))
    pieces = [wl.shard(part, i, 16) for i in range(16)]
    assert all(p is not None and p[0].shape == (1, 3, 2, 4) for p in pieces)
    # Every (batch, head) pair appears once, batch-major.
    got = torch.cat([torch.cat([p[0][:, :, h] for h in range(2)], 0) for p in pieces], 0)
    want = torch.cat([part[0][b:b + 1, :, h] for b in range(2) for h in range(16)], 0)
    assert torch.equal(got, want)


def test_parts_of_every_rank_gathered_in_rank_order_rebuild_the_problem():
    """At N ranks with P parts each, rank r owns parts r, N + r, ...: gathering
    part i of every rank in rank order is a contiguous run of the problem."""
    import torch

    wl = bench.Workload(
        name="toy", metric="", unit="GB/s", dtype="f32", config={},
        make_inputs=lambda dev, seed: (torch.arange(48.0).view(24, 2), torch.ones(3)),
        build_op=lambda inp: None, run=lambda op, inp: inp[0], work=lambda op: 0.0,
        kernel_regex="", shard=bench._rows_shard(1))
    world, pieces = 3, 2
    per_rank = [bench._problem(wl, torch.device("cpu"), 0, r, world, pieces)
                for r in range(world)]
    rebuilt = torch.cat([per_rank[r][i][0] for i in range(pieces) for r in range(world)])
    assert torch.equal(rebuilt, torch.arange(48.0).view(24, 2))
    assert all(torch.equal(p[1], torch.ones(3)) for parts in per_rank for p in parts)
    with pytest.raises(RuntimeError):
        bench._problem(wl, torch.device("cpu"), 0, 0, world, 5)  # 24 rows / 15 parts
    assert len(bench._problem(wl, torch.device("cpu"), 0, 0, 1, 2)) == 1  # N = 1: whole

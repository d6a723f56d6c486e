"""The manifest benchmark contract the reference's ``benchmarks/ops/bench_*.py`` use.

Those files (e.g. examples/TileOPs/benchmarks/ops/bench_hardswish.py,
bench_fused_add_layer_norm.py) build params with ``workloads_to_params`` or
``load_workloads``, time ``ManifestBenchmark(name, op, workload).profile(op,
*inputs)`` and store ``BenchmarkReport.record(op, locals(), result,
tag="tileops")``.  The CPU tests check that surface; the GPU tests run the
same calls on the real ops.
"""

import json

import pytest
import torch

from tileops.benchmark.benchmark_base import (
    BenchmarkReport,
    ManifestBenchmark,
    workloads_to_params,
)
from tileops.manifest import load_workloads


class _StubOp:
    def eval_roofline(self):
        return 4000, 2_000_000


def test_workloads_to_params_ids_and_extras():
    params = workloads_to_params("HardswishFwdOp", include_extra=True)
    ids = [p.id for p in params]
    assert "smoke-1m-float32" in ids and "baseline-256m-bfloat16" in ids
    shape, dtype, extra = next(p.values for p in params if p.id == "fc-wide-float16")
    assert shape == (2048, 4096) and dtype == torch.float16 and extra == {}
    with pytest.raises(KeyError):
        workloads_to_params("no such op")


def test_manifest_benchmark_reads_the_op_roofline():
    bm = ManifestBenchmark("StubOp", _StubOp(), workload=None)
    assert bm.calculate_flops() == 4000.0 and bm.calculate_memory() == 2_000_000.0
    res = bm._build_result(0.5)  # 0.5 ms
    assert res["latency_us"] == pytest.approx(500.0)
    assert res["tflops"] == pytest.approx(4000 / 0.5e-3 / 1e12)
    assert res["bandwidth_tbs"] == pytest.approx(2e6 / 0.5e-3 / 1e12)


def test_report_record_and_dump(tmp_path):
    BenchmarkReport.clear()
    m, n, dtype = 64, 4096, torch.bfloat16
    x = torch.zeros(2)  # tensors in locals() are left out
    op = _StubOp()
    result = {"latency_us": 12.5, "tflops": 0.1}
    BenchmarkReport.record(op, locals(), result, tag="tileops")
    BenchmarkReport.record("NamedOp", {"label": "case-a", "k": 3}, result)
    recs = BenchmarkReport.records()
    assert set(recs) == {"_StubOp", "NamedOp"}
    entry = recs["_StubOp"][0]
    assert entry["params"] == {"m": 64, "n": 4096, "dtype": "bfloat16"}
    assert entry["result"] == result and entry["tag"] == "tileops"
    assert recs["NamedOp"][0]["label"] == "case-a"
    path = BenchmarkReport.dump(str(tmp_path / "r.json"))
    assert json.loads(open(path).read())["NamedOp"][0]["params"] == {"k": 3}
    BenchmarkReport.clear()
    assert BenchmarkReport.dump(str(tmp_path / "empty.json")) is None
    del x


@pytest.mark.gpu
@pytest.mark.parametrize("shape, dtype, op_params", [
    p for p in workloads_to_params("HardswishFwdOp", include_extra=True)
    if p.id.startswith(("smoke-1m", "fc-wide"))])
def test_hardswish_manifest_bench(shape, dtype, op_params):
    from tileops.ops.elementwise.hardswish import HardswishFwdOp
    from tileops.workloads.elementwise import HardswishWorkload

    test = HardswishWorkload(shape, dtype)
    inputs = test.gen_inputs()
    op = HardswishFwdOp(N_total=test.n_total, dtype=dtype, **op_params)
    bm = ManifestBenchmark("HardswishFwdOp", op, test)
    result = bm.profile(op, *inputs)
    BenchmarkReport.record(op, locals(), result, tag="tileops")
    assert result["prof_mode"] == "events" and result["latency_us"] > 0
    assert 0 < result["bandwidth_tbs"] < 10  # below any HBM3e peak


@pytest.mark.gpu
def test_fused_add_layer_norm_manifest_bench():
    from tileops.ops.norm.fused_add_layer_norm import FusedAddLayerNormFwdOp
    from tileops.workloads.norm import FusedAddLayerNormWorkload

    w = next(w for w in load_workloads("FusedAddLayerNormFwdOp") if w["label"] == "llama-8b-prefill")
    m, n = w["x_shape"]
    test = FusedAddLayerNormWorkload(m, n, torch.bfloat16)
    x, residual, weight, bias = test.gen_inputs()
    op = FusedAddLayerNormFwdOp(dtype=torch.bfloat16)
    bm = ManifestBenchmark("FusedAddLayerNormFwdOp", op, test)
    result = bm.profile(op, x, residual, weight, bias)
    BenchmarkReport.record(op, locals(), result, tag="tileops")
    assert result["latency_us"] > 0
    assert result["bandwidth_tbs"] == pytest.approx(op.eval_roofline()[1] / result["latency_us"]
                                                   * 1e-6)

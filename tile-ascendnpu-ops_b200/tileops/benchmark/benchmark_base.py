"""Latency measurement and roofline figures for the ops.

``bench_kernel`` follows the reference protocol (benchmark/benchmark_base.py:
116-204): CUDA events on the launching (current) stream, an L2 flush before
every timed repetition, 5 warm-ups, 3 trials of 10 repetitions, the median of
the trial means.  Only the op call sits between the events; the flush is
outside them.  ``roofline_report`` turns an op's ``eval_roofline()`` and a
latency into achieved GB/s / TFLOP/s and the fraction of a peak.
``BenchmarkReport`` collects result rows and dumps them as JSON.
"""

from __future__ import annotations

import json
import statistics
from dataclasses import asdict, dataclass, field
from pathlib import Path
from typing import Any, Callable, Optional

import torch

from tileops.device import get_device_backend


def bench_kernel(fn: Callable[[], Any], warmup: int = 5, trials: int = 3, reps: int = 10,
                 flush_l2: bool = True) -> float:
    """Median over ``trials`` of the mean latency (ms) of ``reps`` calls of ``fn``."""
    backend = get_device_backend()
    for _ in range(warmup):
        fn()
    backend.synchronize()
    trial_means = []
    for _ in range(trials):
        total = 0.0
        for _ in range(reps):
            if flush_l2:
                backend.cache_flush()
            start = torch.cuda.Event(enable_timing=True)
            end = torch.cuda.Event(enable_timing=True)
            start.record()
            fn()
            end.record()
            end.synchronize()
            total += start.elapsed_time(end)
        trial_means.append(total / reps)
    return statistics.median(trial_means)


def roofline_report(op, latency_ms: float, peak_gbs: Optional[float] = None,
                    peak_tflops: Optional[float] = None) -> dict:
    """Achieved bandwidth / throughput of ``op`` at ``latency_ms`` and its roofline fractions."""
    flops, nbytes = op.eval_roofline()
    sec = latency_ms * 1e-3
    gbs = nbytes / sec / 1e9 if sec > 0 else 0.0
    tflops = flops / sec / 1e12 if sec > 0 else 0.0
    out = {
        "latency_ms": latency_ms,
        "flops": int(flops),
        "bytes": int(nbytes),
        "bandwidth_gbs": gbs,
        "tflops": tflops,
    }
    if peak_gbs:
        out["hbm_frac"] = gbs / peak_gbs
    if peak_tflops:
        out["tensor_frac"] = tflops / peak_tflops
    return out


@dataclass
class BenchmarkReport:
    """Result rows of a benchmark session, dumped as JSON."""

    rows: list = field(default_factory=list)

    def record(self, op_name: str, params: dict, result: dict) -> None:
        self.rows.append({"op": op_name, "params": params, **result})

    def dump(self, path: str | Path) -> None:
        Path(path).write_text(json.dumps(asdict(self), indent=2, default=str))

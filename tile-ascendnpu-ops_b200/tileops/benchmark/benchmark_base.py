"""Latency measurement, the manifest benchmark and the report of the ops.

Same contract as the reference harness
(examples/TileOPs/tileops/benchmark/benchmark_base.py), so the reference's
``benchmarks/ops/bench_*.py`` files run against this package unchanged:

* ``bench_kernel(fn, args=(), n_warmup, n_repeat, n_trials)`` (reference
  :116-204): CUDA events on the launching (current) stream, an L2 flush
  before every timed call (outside the events), inputs cloned per call for
  address diversity when they are small, the median of the trial means, in
  milliseconds.
* ``BenchmarkBase`` / ``ManifestBenchmark`` (reference :269-366, :537-563):
  ``profile(op, *inputs)`` returns ``{"latency_us", "tflops",
  "bandwidth_tbs", "prof_mode"}`` with the flops and bytes read from the op's
  own ``eval_roofline()`` after the timed calls bound its shapes.  The only
  profiling mode on B200 is device events (the reference's msprof mode is an
  Ascend tool; ``TILEOPS_PROF_MODE=msprof`` falls back to events as the
  reference does when msprof is unavailable).
* ``workloads_to_params(op_name)`` (reference :486-534): pytest params of a
  single-input op's manifest workloads.
* ``BenchmarkReport.record(op, locals(), result, tag=...)`` and ``dump`` keep
  the class-level record store of the reference (:587-700), written as JSON.

``roofline_report`` turns an op's ``eval_roofline()`` and a latency into
achieved GB/s / TFLOP/s and the fraction of a peak.
"""

from __future__ import annotations

import hashlib
import json
import logging
import os
from abc import ABC, abstractmethod
from pathlib import Path
from typing import Any, Callable, Generic, Optional, TypeVar

import torch

from tileops.device import get_device_backend

W = TypeVar("W")

_logger = logging.getLogger("tileops.benchmark")

_N_CLONES = 3
_MAX_CLONE_BYTES = 1 << 30


def bench_kernel(fn: Callable, args: tuple = (), n_warmup: int = 5, n_repeat: int = 10,
                 n_trials: int = 3, flush_l2: bool = True) -> float:
    """Median over ``n_trials`` of the mean latency (ms) of ``n_repeat`` calls
    of ``fn(*args)``; the L2 flush before each call is outside the events."""
    if not isinstance(args, tuple):
        raise TypeError(f"bench_kernel expects a tuple of args, got {type(args).__name__}.")
    backend = get_device_backend()
    mask = tuple(isinstance(a, torch.Tensor) for a in args)
    nbytes = sum(a.numel() * a.element_size() for a, m in zip(args, mask) if m)
    if args and nbytes * _N_CLONES <= _MAX_CLONE_BYTES:
        pool = [tuple(a.clone() if m else a for a, m in zip(args, mask))
                for _ in range(_N_CLONES)]
    else:
        pool = [args]

    def run(i):
        return fn(*pool[i % len(pool)])

    for i in range(n_warmup):
        if flush_l2:
            backend.cache_flush()
        run(i)
    backend.synchronize()
    trial_means = []
    for _ in range(n_trials):
        starts = [torch.cuda.Event(enable_timing=True) for _ in range(n_repeat)]
        ends = [torch.cuda.Event(enable_timing=True) for _ in range(n_repeat)]
        for i in range(n_repeat):
            if flush_l2:
                backend.cache_flush()
            starts[i].record()
            run(i)
            ends[i].record()
        backend.synchronize()
        trial_means.append(sum(s.elapsed_time(e) for s, e in zip(starts, ends)) / n_repeat)
    del pool
    trial_means.sort()
    return trial_means[len(trial_means) // 2]


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


class BenchmarkBase(Generic[W], ABC):
    """An op benchmark: timing by device events, work from the subclass."""

    def __init__(self, workload: W):
        self.workload = workload

    @abstractmethod
    def calculate_flops(self) -> Optional[float]:
        raise NotImplementedError

    @abstractmethod
    def calculate_memory(self) -> Optional[float]:
        raise NotImplementedError

    def profile(self, functor: Any, *inputs: Any, mode: Optional[str] = None) -> dict:
        mode = (mode or os.environ.get("TILEOPS_PROF_MODE", "events")).lower().strip()
        if mode != "events":
            _logger.warning("profiling mode %r is not available on CUDA; using device events",
                            mode)
        with torch.no_grad():
            latency = bench_kernel(functor, args=inputs)
        result = self._build_result(latency)
        result["prof_mode"] = "events"
        return result

    def _build_result(self, latency_ms: float) -> dict:
        result: dict[str, Any] = {"latency_us": latency_ms * 1000.0}
        flops = self.calculate_flops()
        if flops is not None:
            result["tflops"] = flops / latency_ms * 1e-9
        memory = self.calculate_memory()
        if memory is not None:
            result["bandwidth_tbs"] = memory / latency_ms * 1e-9
        return result


class ManifestBenchmark(BenchmarkBase[Any]):
    """Benchmark whose flops and bytes are the op's own ``eval_roofline()``.

    ``ManifestBenchmark("FusedAddLayerNormFwdOp", op, workload).profile(op, *inputs)``
    """

    def __init__(self, op_name: str, op: Any, workload: Any):
        super().__init__(workload)
        self._op_name = op_name
        self._op = op
        self._roofline_cache: Optional[tuple[float, float]] = None

    def _get_roofline(self) -> tuple[float, float]:
        if self._roofline_cache is None:
            flops, mem_bytes = self._op.eval_roofline()
            self._roofline_cache = (float(flops), float(mem_bytes))
        return self._roofline_cache

    def calculate_flops(self) -> Optional[float]:
        return self._get_roofline()[0]

    def calculate_memory(self) -> Optional[float]:
        return self._get_roofline()[1]


def workloads_to_params(op_name: str, include_extra: bool = False) -> list:
    """pytest params ``(shape, dtype[, extra])`` of a single-input op's
    manifest workloads, one per (workload, dtype), id ``<label>-<dtype>``."""
    import pytest

    from tileops.manifest import WORKLOAD_RESERVED_KEYS, load_workloads

    params = []
    for w in load_workloads(op_name):
        shape_keys = [k for k in w if isinstance(k, str) and k.endswith("shape")]
        if len(shape_keys) != 1:
            raise KeyError(f"workloads_to_params({op_name!r}) needs exactly one shape key; "
                           "multi-input ops use their own bench files.")
        key = shape_keys[0]
        shape = tuple(w[key])
        label = w.get("label", "x".join(str(s) for s in shape))
        extra = {k: v for k, v in w.items() if k not in WORKLOAD_RESERVED_KEYS and k != key}
        for dtype_str in w["dtypes"]:
            dtype = getattr(torch, dtype_str)
            args = (shape, dtype, dict(extra)) if include_extra else (shape, dtype)
            params.append(pytest.param(*args, id=f"{label}-{dtype_str}"))
    return params


def _extract_op_config(op: object) -> Optional[dict]:
    for holder in (op, getattr(op, "kernel", None)):
        cfg = getattr(holder, "config", None) if holder is not None else None
        if cfg:
            return cfg
    return None


class BenchmarkReport:
    """Benchmark records of a session, keyed by op name (class-level store)."""

    _records: dict = {}

    @staticmethod
    def _json_safe(value: Any) -> Any:
        if value is None or isinstance(value, (bool, int, float, str)):
            return value
        if isinstance(value, torch.dtype):
            return str(value).removeprefix("torch.")
        if isinstance(value, Path):
            return str(value)
        if isinstance(value, (list, tuple)):
            return [BenchmarkReport._json_safe(v) for v in value]
        if isinstance(value, dict):
            return {str(k): BenchmarkReport._json_safe(v) for k, v in value.items()}
        return str(value)

    @staticmethod
    def record(op_or_name, params: dict, result: dict, tag: str = "tileops") -> None:
        """Store one result; ``params`` is usually the bench function's ``locals()``
        (tensors, the op and the benchmark object are left out)."""
        if isinstance(op_or_name, str):
            name, module, config = op_or_name, None, None
        else:
            name = type(op_or_name).__name__
            module = type(op_or_name).__module__
            config = _extract_op_config(op_or_name)

        def plain(v):
            if v is None or isinstance(v, (int, float, bool, str, torch.dtype)):
                return True
            if isinstance(v, (list, tuple)):
                return all(plain(x) for x in v)
            if isinstance(v, dict):
                return all(isinstance(k, str) and plain(x) for k, x in v.items())
            return False

        kept = {k: v for k, v in params.items()
                if k not in ("test", "bm", "op", "inputs", "result") and not k.startswith("_")
                and plain(v)}
        kept = BenchmarkReport._json_safe(kept)
        label = kept.pop("label", None) or "-".join(f"{k}={v}" for k, v in kept.items())
        digest = hashlib.sha1(json.dumps([name, kept], sort_keys=True).encode()).hexdigest()[:12]
        entry = {"case_id": f"{name}-{digest}", "label": label, "params": kept,
                 "result": BenchmarkReport._json_safe(result), "tag": tag}
        if module:
            entry["op_module"] = module
        if config:
            entry["config"] = BenchmarkReport._json_safe(config)
        BenchmarkReport._records.setdefault(name, []).append(entry)
        _logger.info("op=%s tag=%s latency_us=%.4f tflops=%.2f", name, tag,
                     result.get("latency_us", 0.0), result.get("tflops", 0.0))

    @staticmethod
    def records() -> dict:
        return BenchmarkReport._records

    @staticmethod
    def clear() -> None:
        BenchmarkReport._records = {}

    @staticmethod
    def dump(path: Optional[str] = None) -> Optional[str]:
        """Write every record as JSON to ``path`` (or ``$TILEOPS_BENCHMARK_REPORT_PATH``,
        else ``benchmark_report.json``); returns the path, or None when empty."""
        if not BenchmarkReport._records:
            return None
        path = path or os.environ.get("TILEOPS_BENCHMARK_REPORT_PATH") or "benchmark_report.json"
        Path(path).write_text(json.dumps(BenchmarkReport._records, indent=2))
        return str(path)

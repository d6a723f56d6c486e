from tileops.benchmark.benchmark_base import BenchmarkReport, bench_kernel, roofline_report

__all__ = ["BenchmarkReport", "bench_kernel", "roofline_report"]

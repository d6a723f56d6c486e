from tileops.benchmark.benchmark_base import (
    BenchmarkBase,
    BenchmarkReport,
    ManifestBenchmark,
    bench_kernel,
    roofline_report,
    workloads_to_params,
)

__all__ = ["BenchmarkBase", "BenchmarkReport", "ManifestBenchmark", "bench_kernel",
           "roofline_report", "workloads_to_params"]

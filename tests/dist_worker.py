"""One rank of the multi-rank bench-path test (run under torchrun, gloo).

Exercises, on CPU ranks, the host logic ``bench.py`` uses at N > 1: the
barrier, the max-over-ranks reduction of the timed region, and the
weak-scaling whole-job value.  Exits non-zero on a mismatch.
"""

import datetime
import os
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

import bench  # noqa: E402


def main() -> int:
    rank, local_rank, world = bench.dist_env()
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=30))
    dev = torch.device("cpu")
    bench.barrier(world, dev)
    # Each rank "timed" a different region; the job is as slow as the slowest.
    mine = 10.0 + 5.0 * rank
    got = bench.max_over_ranks(mine, world, dev)
    expect = 10.0 + 5.0 * (world - 1)
    ok = got == expect
    value = bench.whole_job_value(1e9, 4, got, world, "GB/s")
    ok &= abs(value - world * 4.0 / (expect * 1e-3)) < 1e-9
    bench.barrier(world, dev)
    dist.destroy_process_group()
    print(f"rank {rank}/{world} local {local_rank} max {got} value {value:.6f} "
          f"{'OK' if ok else 'MISMATCH'}", flush=True)
    return 0 if ok else 1


if __name__ == "__main__":
    sys.exit(main())

"""One rank of the multi-rank bench-path test (run under torchrun, gloo).

Exercises, on CPU ranks, the host logic ``bench.py`` uses at N > 1: the
barrier, the max-over-ranks reduction of the timed region, the
weak-scaling whole-job value and the optional output reassembly
(``gather_outputs``).  Exits non-zero on a mismatch.
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
    # Output reassembly (bench.py --gather): every rank ends up with every
    # rank's shards, in rank order, and the byte counts follow the shapes.
    outs = (torch.full((3, 4), float(rank)), torch.arange(5, dtype=torch.int32) + 10 * rank)
    summary, fulls = bench.gather_outputs(outs, world, dev, reps=2)
    for r in range(world):
        ok &= bool(torch.equal(fulls[0][12 * r:12 * (r + 1)], torch.full((12,), float(r))))
        ok &= bool(torch.equal(fulls[1][5 * r:5 * (r + 1)],
                               torch.arange(5, dtype=torch.int32) + 10 * r))
    ok &= summary["bytes_per_rank"] == 12 * 4 + 5 * 4
    ok &= summary["bytes_total"] == world * (12 * 4 + 5 * 4)
    ok &= summary["bytes_received_per_rank"] == (world - 1) * (12 * 4 + 5 * 4)
    ok &= summary["outputs"] == 2 and summary["ms"] > 0
    bench.barrier(world, dev)
    dist.destroy_process_group()
    print(f"rank {rank}/{world} local {local_rank} max {got} value {value:.6f} "
          f"{'OK' if ok else 'MISMATCH'}", flush=True)
    return 0 if ok else 1


if __name__ == "__main__":
    sys.exit(main())

"""One rank of the multi-rank bench-path tests (run under torchrun, gloo, CPU).

Scenario (argv[1]):

* ``pipeline`` -- the host logic ``bench.py`` uses at N > 1: barrier,
  max-over-ranks of the timed region, the strong-scaling value, the shard /
  reassemble path (every rank slices the same seeded problem, runs a stand-in
  op on its shard, ``all_gather_into_tensor`` + the full layout) compared
  with the op on the whole problem, for row shards and for (batch, head)
  shards that split heads, and the shard-shape check.
* ``shape_mismatch`` -- rank 1 holds a shard of another shape; every rank
  must raise from ``check_shard_shapes`` before any all-gather.
* ``rank_exits`` -- rank 1 leaves between two steps (exits after the first
  step's collective); rank 0's next collective must end with an error
  within the process-group timeout instead of waiting forever.

Prints ``rank R/W <scenario> OK`` (or ``... FAIL <why>``); exits 0 on OK.
"""

import datetime
import os
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

import bench  # noqa: E402


def _stand_in_gdn(q, scale):
    """A per-(batch, head) op with BTHD in and out and a (B, H, D, D) state."""
    o = q * scale + q.sum(dim=1, keepdim=True)
    state = torch.einsum("bthd,bthe->bhde", q, q)
    return o, state


def pipeline(rank: int, world: int, dev) -> list[str]:
    bad = []
    bench.barrier(world, dev)
    got = bench.max_over_ranks(10.0 + 5.0 * rank, world, dev)
    if got != 10.0 + 5.0 * (world - 1):
        bad.append(f"max_over_ranks {got}")
    # Strong scaling: the whole problem's work over the slowest rank's time.
    if abs(bench.whole_job_value(4e9, 1, got, "GB/s") - 4.0 / (got * 1e-3)) > 1e-9:
        bad.append("whole_job_value")

    # Row shards (FALN-like): every rank draws the same problem, keeps rows.
    g = torch.Generator().manual_seed(1235)
    x = torch.randn(64, 32, generator=g)
    r = torch.randn(64, 32, generator=g)
    full_out = torch.nn.functional.layer_norm(x + r, (32,))
    mine = bench._rows_shard(2)((x, r), rank, world)
    outs = (torch.nn.functional.layer_norm(mine[0] + mine[1], (32,)),)
    bench.check_shard_shapes([tuple(o.shape) for o in outs], world, dev)
    fulls = bench.gather_outputs(outs, world, dev)
    if not torch.equal(fulls[0].view(64, 32), full_out):
        bad.append("row shards do not reassemble the full output")
    if world > 1 and bench._rows_shard(1)((x[:63],), rank, world) is not None:
        bad.append("uneven rows were accepted")

    # (batch, head) shards with heads split (batch 2 < world 4 when world=4;
    # batch split when world=2): outputs back in BTHD / (B, H) order.
    B, T, H, D = 2, 5, 8, 4
    q = torch.randn(B, T, H, D, generator=g)
    o_full, s_full = _stand_in_gdn(q, 0.5)
    bs, hs = bench.bh_split(B, H, rank, world)
    o, s = _stand_in_gdn(q[bs, :, hs].contiguous(), 0.5)
    flats = bench.gather_outputs((o, s), world, dev)
    o_back = bench.unshard_bthd(flats[0], B, T, H, D, world)
    if not torch.allclose(o_back, o_full) or not torch.allclose(flats[1].view(B, H, D, D),
                                                                s_full):
        bad.append("(batch, head) shards do not reassemble")
    bench.barrier(world, dev)
    return bad


def shape_mismatch(rank: int, world: int, dev) -> list[str]:
    shape = (8, 4) if rank == 0 else (8, 5)
    try:
        bench.check_shard_shapes([shape], world, dev)
    except RuntimeError as e:
        return [] if "shard shapes differ" in str(e) else [f"wrong error: {e}"]
    return ["mismatched shapes were not detected"]


def rank_exits(rank: int, world: int, dev) -> list[str]:
    bench.barrier(world, dev)  # step 1: everyone
    if rank == 1:
        sys.stdout.flush()
        os._exit(0)  # leaves between steps, nothing in flight
    time.sleep(0.5)
    t0 = time.monotonic()
    try:
        bench.max_over_ranks(1.0, world, dev)  # step 2: a peer is gone
    except Exception as e:  # gloo: connection closed, or the timeout
        took = time.monotonic() - t0
        return [] if took < 60 else [f"error after {took:.0f} s: {e}"]
    return ["a collective with a departed rank returned normally"]


def main() -> int:
    scenario = sys.argv[1] if len(sys.argv) > 1 else "pipeline"
    rank, _, world = bench.dist_env()
    timeout = datetime.timedelta(seconds=10 if scenario == "rank_exits" else 60)
    dist.init_process_group("gloo", timeout=timeout)
    dev = torch.device("cpu")
    bad = {"pipeline": pipeline, "shape_mismatch": shape_mismatch,
           "rank_exits": rank_exits}[scenario](rank, world, dev)
    print(f"rank {rank}/{world} {scenario} " + ("OK" if not bad else "FAIL " + "; ".join(bad)),
          flush=True)
    if scenario != "rank_exits":
        dist.destroy_process_group()
    return 0 if not bad else 1


if __name__ == "__main__":
    sys.exit(main())

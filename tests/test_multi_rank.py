"""The N > 1 path of bench.py on CPU ``gloo`` ranks, and its failure modes.

At N > 1 the bench splits one BASELINE problem across the ranks (rows,
batches or (batch, head) pairs), runs the op on each shard and reassembles
the outputs with ``all_gather_into_tensor``.  Here, without a GPU, two- and
four-rank ``gloo`` jobs check that host logic with stand-in torch ops (shards
reassemble to the whole-problem result; the max over ranks; the strong-scaling
value), and the failure modes the harness must survive without hanging: a
rank whose shard has another shape, a rank that leaves between steps, and a
rendezvous that a rank never joins.  The reference arm prints one line from
rank 0.
"""

import json
import os
import re
import socket
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _torchrun(script_args: list[str], nproc: int = 2, timeout: int = 240):
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={nproc}", "--master-addr", "127.0.0.1",
           "--master-port", str(_free_port())] + script_args
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="", OMP_NUM_THREADS="1")
    return subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True,
                          timeout=timeout)


def test_whole_job_value_is_strong_scaling():
    sys.path.insert(0, str(ROOT))
    import bench

    # The whole problem's work over the slowest rank's time, whatever N.
    assert bench.whole_job_value(2e9, 10, 20.0, "GB/s") == pytest.approx(1000.0)
    assert bench.whole_job_value(2e12, 1, 1000.0, "TFLOP/s") == pytest.approx(2.0)


def test_split_helpers():
    sys.path.insert(0, str(ROOT))
    import bench

    assert bench.split_range(8192, 3, 8) == slice(3072, 4096)
    assert bench.split_range(10, 0, 4) is None
    # GDN at 8 ranks: batch 4, 16 heads -> two head groups of 8 per batch.
    assert bench.bh_split(4, 16, 5, 8) == (slice(2, 3), slice(8, 16))
    assert bench.bh_split(4, 16, 1, 2) == (slice(2, 4), slice(0, 16))
    assert bench.bh_split(4, 5, 0, 8) is None  # 5 heads do not split into 2 groups
    assert bench.head_groups(4, 8) == 2 and bench.head_groups(8, 8) == 1


@pytest.mark.parametrize("nproc", [2, 4])
def test_gloo_shard_gather_pipeline(nproc):
    r = _torchrun(["tests/dist_worker.py", "pipeline"], nproc=nproc)
    assert r.returncode == 0, r.stdout + r.stderr
    found = re.findall(r"rank (\d)/\d pipeline (OK|FAIL.*)", r.stdout)
    assert sorted(f[0] for f in found) == [str(i) for i in range(nproc)], r.stdout
    assert all(f[1] == "OK" for f in found), r.stdout


def test_gloo_mismatched_shard_shapes_raise_on_every_rank():
    r = _torchrun(["tests/dist_worker.py", "shape_mismatch"])
    assert r.returncode == 0, r.stdout + r.stderr
    assert len(re.findall(r"rank \d/2 shape_mismatch OK", r.stdout)) == 2, r.stdout


def test_gloo_rank_that_leaves_ends_the_next_collective_with_an_error():
    r = _torchrun(["tests/dist_worker.py", "rank_exits"], timeout=180)
    assert "rank 0/2 rank_exits OK" in r.stdout, r.stdout + r.stderr


def test_rendezvous_a_rank_never_joins_times_out():
    """init_process_group with timeout= raises instead of waiting forever
    when a rank of the job never arrives."""
    code = (
        "import datetime, sys, torch.distributed as dist\n"
        "try:\n"
        f"    dist.init_process_group('gloo', init_method='tcp://127.0.0.1:{_free_port()}',\n"
        "                            world_size=2, rank=0,\n"
        "                            timeout=datetime.timedelta(seconds=3))\n"
        "except Exception as e:\n"
        "    print('raised', type(e).__name__); sys.exit(0)\n"
        "print('joined'); sys.exit(1)\n"
    )
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True,
                       timeout=120, env=dict(os.environ, CUDA_VISIBLE_DEVICES=""))
    assert r.returncode == 0 and "raised" in r.stdout, r.stdout + r.stderr


def test_reference_arm_prints_one_line_from_rank_zero():
    r = _torchrun(["bench.py", "--impl", "reference", "--gpus", "2", "--steps", "1",
                   "--warmup", "0"])
    assert r.returncode == 0, r.stdout + r.stderr
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, r.stdout
    line = json.loads(lines[0])
    assert line["impl"] == "reference"
    assert line["n_gpus"] == 2
    assert line["e2e"]["h2d_bytes_per_step"] == 0
    assert line["cpu_baseline"]["kind"] == "port"
    assert line["cpu_baseline"]["same_config"] is True  # the full FALN configuration
    assert line["value"] > 0

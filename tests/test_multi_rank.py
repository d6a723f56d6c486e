"""The N > 1 path of bench.py on CPU ``gloo`` ranks (world size 2).

The hot path shards into independent units (every rank runs its own batch,
no collective on the data path), so the multi-rank logic is host-side only:
rendezvous, barriers, max-over-ranks timing, the weak-scaling aggregate, and
rank 0 alone printing the result line.  These run here without a GPU.
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


def test_whole_job_value_is_weak_scaling():
    sys.path.insert(0, str(ROOT))
    import bench

    one = bench.whole_job_value(2e9, 10, 20.0, 1, "GB/s")
    assert one == pytest.approx(1000.0)
    # Two ranks, same per-rank work, the slower rank's time: twice the units.
    assert bench.whole_job_value(2e9, 10, 20.0, 2, "GB/s") == pytest.approx(2 * one)
    assert bench.whole_job_value(2e12, 1, 1000.0, 4, "TFLOP/s") == pytest.approx(8.0)


def test_gloo_two_ranks_barrier_and_max_over_ranks():
    r = _torchrun(["tests/dist_worker.py"])
    assert r.returncode == 0, r.stdout + r.stderr
    # The two ranks share one pipe, so their lines may interleave.
    found = re.findall(r"rank (\d)/2 local \d max ([\d.]+) value [\d.]+ (OK|MISMATCH)",
                       r.stdout)
    assert sorted(f[0] for f in found) == ["0", "1"], r.stdout
    assert all(f[1] == "15.0" and f[2] == "OK" for f in found), r.stdout


def test_reference_arm_prints_one_line_from_rank_zero():
    r = _torchrun(["bench.py", "--impl", "reference", "--gpus", "2", "--steps", "1",
                   "--warmup", "1", "--ref-rows", "8"])
    assert r.returncode == 0, r.stdout + r.stderr
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, r.stdout
    line = json.loads(lines[0])
    assert line["impl"] == "reference"
    assert line["n_gpus"] == 2
    assert line["e2e"]["h2d_bytes_per_step"] == 0
    assert line["cpu_baseline"]["kind"] == "port"
    assert line["value"] > 0

"""bench.py's multi-GPU bookkeeping on two CPU ranks (gloo): every rank ends
with the slowest rank's elapsed times, the whole-job rate counts every rank's
tokens over that time, and the reference arm does its work on rank 0 only."""
import json
import os
import socket
import subprocess
import sys

import pytest

from conftest import ROOT


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, out: str) -> None:
    import datetime

    import torch.distributed as dist

    sys.path.insert(0, ROOT)
    import bench

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    # rank r took (r + 1) * 10 ms for the timed steps and 5 ms end to end
    ms, e2e = bench.max_over_ranks([(rank + 1) * 10.0, 5.0], dist, "cpu")
    rate = bench.replica_rate(world, 64 * 8, ms)
    with open(os.path.join(out, f"rank{rank}.json"), "w") as f:
        json.dump({"ms": ms, "e2e": e2e, "rate": rate}, f)
    dist.destroy_process_group()


def test_max_over_ranks_and_rate_on_two_gloo_ranks(tmp_path):
    import torch.multiprocessing as mp

    port = _free_port()
    mp.start_processes(_rank_main, args=(2, port, str(tmp_path)), nprocs=2, start_method="spawn")
    res = [json.load(open(tmp_path / f"rank{r}.json")) for r in range(2)]
    for r in res:
        assert r["ms"] == 20.0 and r["e2e"] == 5.0  # the slowest rank's times on every rank
        assert r["rate"] == pytest.approx(2 * 64 * 8 / 0.020)


def test_reference_arm_works_on_rank_zero_only(tmp_path):
    """A rank other than 0 of `bench.py --impl reference` exits 0 without
    output (rank 0 alone times the CPU path and prints the line)."""
    env = dict(os.environ, RANK="1", WORLD_SIZE="2", LOCAL_RANK="1")
    p = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--gpus", "2"],
                       env=env, capture_output=True, text=True, timeout=120)
    assert p.returncode == 0, p.stderr
    assert p.stdout.strip() == ""


def test_bench_helpers_single_rank():
    sys.path.insert(0, ROOT)
    import bench

    assert bench.max_over_ranks([3.0, 4.0], None, "cpu") == [3.0, 4.0]
    assert bench.replica_rate(1, 128, 256.0) == pytest.approx(500.0)
    assert bench.expected_unique_experts(256, 8, 64) == pytest.approx(222.4, abs=0.1)

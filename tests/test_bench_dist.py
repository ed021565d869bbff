"""bench.py's multi-rank host logic with world_size 2 on the gloo backend (CPU):
the job time is the slowest rank's, the job value counts every rank's steps,
and the reference arm runs on rank 0 only."""
import os
import socket
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    import torch.distributed as dist
    sys.path.insert(0, ROOT)
    import bench
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    local = 1.0 + rank            # rank 1 is the slow one
    tmax = bench.max_over_ranks(local, dist)
    q.put((rank, tmax, bench.job_value(10, world, tmax)))
    dist.barrier()
    dist.destroy_process_group()


def test_two_rank_aggregation_gloo():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    got = sorted(q.get(timeout=10) for _ in range(2))
    for rank, tmax, value in got:
        assert tmax == 2.0                 # the slowest rank's time, on every rank
        assert value == pytest.approx(10.0)  # 2 ranks x 10 steps / 2 s


def test_single_process_aggregation():
    sys.path.insert(0, ROOT)
    import bench
    assert bench.max_over_ranks(1.5) == 1.5
    assert bench.job_value(30, 1, 1.5) == 20.0


def test_reference_arm_non_zero_rank_exits_quietly():
    env = dict(os.environ, RANK="1", LOCAL_RANK="1", WORLD_SIZE="2")
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "2"],
                       capture_output=True, text=True, env=env, timeout=120)
    assert r.returncode == 0 and r.stdout.strip() == ""

"""The bench's multi-rank plumbing on CPU: two gloo ranks (spawned processes,
rendezvous on 127.0.0.1) take the same barrier and max-over-ranks steps the
GPU runs take over NCCL, and the reference arm prints from rank 0 only."""
import argparse
import datetime
import os
import socket
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, times, q):
    import torch.distributed as dist
    sys.path.insert(0, ROOT)
    import bench
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        bench.barrier(world)
        got = bench.max_over_ranks(times[rank], world)
        bench.barrier(world)
        q.put((rank, got))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_max_over_ranks_gloo(world):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    times = [1.5 + 0.25 * r for r in range(world)][::-1]   # rank 0 is the slowest
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, times, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in range(world):
            rank, got = q.get(timeout=120)
            results[rank] = got
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert all(p.exitcode == 0 for p in procs)
    assert results == {r: max(times) for r in range(world)}


def test_single_rank_helpers_take_no_collective():
    sys.path.insert(0, ROOT)
    import bench
    bench.barrier(1)
    assert bench.max_over_ranks(3.25, 1) == 3.25


def test_reference_arm_prints_on_rank0_only(monkeypatch, capsys):
    sys.path.insert(0, ROOT)
    import bench
    monkeypatch.setenv("RANK", "1")
    bench.reference_arm(argparse.Namespace(steps=1, warmup=0, gpus=2))
    assert capsys.readouterr().out == ""

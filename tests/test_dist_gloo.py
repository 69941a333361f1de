"""Multi-rank host logic of bench.py on CPU with the gloo backend (2 ranks)."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    import bench
    ms = 10.0 + 5.0 * rank  # rank 1 is the slowest
    worst = bench.max_over_ranks(ms, torch.device("cpu"), world)
    rate = bench.job_rate(4, worst / 1e3, world)
    q.put((rank, worst, rate))
    dist.barrier()
    dist.destroy_process_group()


def test_max_over_ranks_and_weak_scaling_rate():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = sorted(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    import bench
    for rank, worst, rate in out:
        assert worst == 15.0  # every rank sees the slowest rank's time
        assert rate == pytest.approx(2 * 4 * bench.UPDATES / 0.015 / 1e9)


def test_reference_arm_other_ranks_exit_without_work(monkeypatch):
    import bench
    monkeypatch.setenv("RANK", "1")
    monkeypatch.setenv("WORLD_SIZE", "2")

    class A:
        steps, warmup, gpus = 1, 0, 2
    assert bench.run_reference(A()) == 0

"""The multi-process (data-parallel) bench path on CPU: two gloo ranks, each with its own
per-rank time; the job value uses the slowest rank and every rank agrees."""
import os
import socket
import sys

import pytest
import torch.multiprocessing as mp

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, out):
    import datetime

    import torch.distributed as dist

    sys.path.insert(0, REPO)
    import bench

    os.environ.update({"MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port)})
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        value, ms = bench.dp_value(10.0 + 5.0 * rank, steps=4, world=world, device="cpu")
        bench.barrier(world)
        out.put((rank, value, ms))
    finally:
        dist.destroy_process_group()


def test_dp_value_two_gloo_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    got = sorted(q.get(timeout=10) for _ in range(2))
    for rank, value, ms in got:
        assert ms == pytest.approx(15.0)
        assert value == pytest.approx(2 * 4 / 0.015)


def test_dp_value_single_rank_is_local():
    sys.path.insert(0, REPO)
    import bench

    value, ms = bench.dp_value(8.0, steps=16, world=1)
    assert ms == 8.0 and value == pytest.approx(2000.0)

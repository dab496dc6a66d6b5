"""The multi-process bench paths on CPU with two gloo ranks: the data-parallel and the
tensor-parallel job values use the slowest rank and every rank agrees; one rank's failed parity
check fails every rank's; and a rank that dies before a collective makes the others' next
collective end with an error at the process group's timeout instead of waiting for ever (how
the tensor-parallel bench and tests learn of a lost rank on the host)."""
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


def _tp_rank_main(rank: int, world: int, port: int, out):
    import datetime

    import torch.distributed as dist

    sys.path.insert(0, REPO)
    import bench

    os.environ.update({"MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port)})
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        value, ms = bench.tp_value(10.0 + 5.0 * rank, steps=4, world=world, device="cpu")
        all_ok = bench.parity_agreed(True, world, device="cpu")
        one_bad = bench.parity_agreed(rank != 1, world, device="cpu")
        out.put((rank, value, ms, all_ok, one_bad))
    finally:
        dist.destroy_process_group()


def _dying_rank_main(rank: int, world: int, port: int, out):
    import datetime

    import torch.distributed as dist

    sys.path.insert(0, REPO)
    import bench

    os.environ.update({"MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port)})
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=3))
    if rank == 1:
        os._exit(0)  # leaves between steps, before the next collective
    try:
        bench.tp_value(1.0, steps=4, world=world, device="cpu")
        out.put((rank, "returned"))
    except Exception as e:  # noqa: BLE001 - any error is what the test expects
        out.put((rank, "error: " + type(e).__name__))


def test_tp_value_and_parity_two_gloo_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_tp_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    got = sorted(q.get(timeout=10) for _ in range(2))
    for rank, value, ms, all_ok, one_bad in got:
        assert ms == pytest.approx(15.0)
        assert value == pytest.approx(4 / 0.015)  # one sequence: the steps, not world * steps
        assert all_ok is True and one_bad is False


def test_dead_rank_ends_the_next_collective_with_an_error():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_dying_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
    assert procs[1].exitcode == 0
    rank, what = q.get(timeout=30)
    assert rank == 0 and what.startswith("error"), what


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

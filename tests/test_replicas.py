"""Multi-process host logic of the request-replica path, with gloo ranks on CPU (world size 2):
rendezvous, disjoint request assignment and seeds, max-over-ranks timing, whole-job aggregation,
and failure detection (a rank that never joins a collective makes the survivor's collective fail
within the process-group timeout instead of hanging)."""

import os
import socket
import time

import pytest
import torch.multiprocessing as mp

from ppu_b200 import replicas as R


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _env(rank: int, world: int, port: int) -> None:
    os.environ.update({"RANK": str(rank), "WORLD_SIZE": str(world), "LOCAL_RANK": str(rank),
                       "MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port)})


def _worker_ok(rank: int, world: int, port: int, out) -> None:
    _env(rank, world, port)
    assert R.init("gloo", timeout_s=60)
    mine = R.requests_for_rank(10, world, rank)
    seeds = [R.request_seed(rank, i) for i in range(len(mine))]
    slowest = R.max_over_ranks(1.5 + rank)
    R.barrier()
    out.put((rank, mine, seeds, slowest))
    R.shutdown()


def _worker_dropout(rank: int, world: int, port: int, out) -> None:
    _env(rank, world, port)
    R.init("gloo", timeout_s=5)
    if rank == 1:  # leaves between steps: never enters the next collective
        R.barrier()
        out.put((rank, "left"))
        return
    R.barrier()
    t0 = time.time()
    try:
        R.max_over_ranks(1.0)
        out.put((rank, "no error"))
    except Exception as e:  # the survivor learns of the missing rank from the timeout
        out.put((rank, type(e).__name__, time.time() - t0))


def _run(target, world: int):
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=target, args=(r, world, port, out)) for r in range(world)]
    for p in procs:
        p.start()
    results = [out.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return sorted(results, key=lambda r: r[0])


def test_replica_host_logic_two_ranks():
    res = _run(_worker_ok, 2)
    (_, mine0, seeds0, slow0), (_, mine1, seeds1, slow1) = res
    assert sorted(mine0 + mine1) == list(range(10)) and not set(mine0) & set(mine1)
    assert not set(seeds0) & set(seeds1)
    assert slow0 == slow1 == 2.5


def test_missing_rank_fails_collective_instead_of_hanging():
    res = _run(_worker_dropout, 2)
    assert res[1][1] == "left"
    assert res[0][1] != "no error", res[0]
    assert res[0][2] < 60


def test_aggregation_and_seed_guards():
    assert R.aggregate_rate(32, 0.5, 4) == pytest.approx(256.0)
    with pytest.raises(ValueError):
        R.aggregate_rate(1, 0.0, 1)
    with pytest.raises(ValueError):
        R.request_seed(0, R.SEED_STRIDE)
    assert R.requests_for_rank(5, 1, 0) == [0, 1, 2, 3, 4]
    assert R.max_over_ranks(3.25) == 3.25  # single process: no group

"""Session sharding and the host-side collectives, on world-size-2 gloo process groups (CPU)."""
import os
import socket

import pytest
import torch.multiprocessing as mp

from loopfuse_b200.runtime.sharding import RankGroup, lpt_assign


def test_lpt_assign_balances_and_covers():
    work = [1024, 32768, 5000, 17000, 9000, 30000, 1500, 22000]
    parts = lpt_assign(work, 2)
    assert sorted(i for p in parts for i in p) == list(range(len(work)))
    loads = [sum(work[i] for i in p) for p in parts]
    assert max(loads) - min(loads) <= max(work)
    assert lpt_assign(work, 2) == parts                       # deterministic
    assert lpt_assign(work, 1) == [list(range(len(work)))]


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, work, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), WORLD_SIZE=str(world),
                      RANK=str(rank), LOCAL_RANK=str(rank))
    g = RankGroup(backend="gloo", timeout_s=30)
    mine = lpt_assign(work, world)[rank]
    local = float(sum(work[i] for i in mine))
    total = g.sum(local)
    worst = g.max(local)
    g.barrier()
    q.put((rank, mine, total, worst))
    g.close()


def test_two_gloo_ranks_agree_on_shards_and_reductions():
    work = [3000, 12000, 7000, 28000, 1100, 16000]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, work, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    (r0, m0, t0, w0), (r1, m1, t1, w1) = res
    assert sorted(m0 + m1) == list(range(len(work)))
    assert t0 == t1 == float(sum(work))
    assert w0 == w1 == max(float(sum(work[i] for i in m0)), float(sum(work[i] for i in m1)))


def _dropout_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), WORLD_SIZE=str(world),
                      RANK=str(rank), LOCAL_RANK=str(rank))
    g = RankGroup(backend="gloo", timeout_s=5)
    if rank == 1:
        raise SystemExit(3)              # a rank that leaves between steps
    try:
        g.barrier()
        q.put((rank, "no error"))
    except Exception as e:               # the survivor sees the loss at its next collective
        q.put((rank, type(e).__name__))


def test_surviving_rank_sees_a_dropped_rank_as_an_error():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_dropout_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    rank, outcome = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
    assert rank == 0 and outcome != "no error"

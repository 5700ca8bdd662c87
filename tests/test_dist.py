"""Multi-rank host logic on CPU (gloo, world size 2): stream partitioning and
the max-over-ranks job time, and a rank that fails before a collective is
seen by the other as an error, not a hang."""

import os
import socket

import pytest
import torch.multiprocessing as mp

from gorelaxor_b200.dist import max_over_ranks, owner, partition


def test_partition_is_contiguous_and_complete():
    for n in (1, 7, 256, 2048):
        for world in (1, 2, 3, 4, 8):
            got = [s for r in range(world) for s in partition(n, world, r)]
            assert got == list(range(n))
            for r in range(world):
                assert all(owner(s, n, world) == r for s in partition(n, world, r))
    assert len(partition(2048, 8, 3)) == 256


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q, fail_rank):
    import datetime

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=10))
    try:
        mine = list(partition(10, world, rank))
        t = max_over_ranks(1.0 + rank)
        if rank == fail_rank:
            raise RuntimeError("rank failed before its next collective")
        t2 = max_over_ranks(5.0 * (rank + 1))
        q.put((rank, mine, t, t2))
    except Exception as e:  # the surviving rank reports the error it saw
        q.put((rank, "error", type(e).__name__))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def _run(fail_rank):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, 2, port, q, fail_rank)) for r in range(2)]
    for p in ps:
        p.start()
    out = sorted(q.get(timeout=60) for _ in ps)
    for p in ps:
        p.join(timeout=30)
    return out


def test_two_ranks_gloo():
    out = _run(fail_rank=-1)
    assert out[0] == (0, [0, 1, 2, 3, 4], 2.0, 10.0)
    assert out[1] == (1, [5, 6, 7, 8, 9], 2.0, 10.0)


def test_failed_rank_is_an_error_not_a_hang():
    out = _run(fail_rank=1)
    assert out[1][:2] == (1, "error")
    assert out[0][:2] == (0, "error")  # the survivor's collective ends with an error

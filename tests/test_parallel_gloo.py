"""ParallelGroup on CPU ranks (gloo, world size 2 and 4), no GPU.

Mirrors the reference's group contract (moe_serving/gpt_oss_parallel.py:53-103
and tests/test_ep_moe.py): contiguous blocks of ``size`` ranks, the block-local
rank, and the four collectives the expert layer uses.
"""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, size: int, port: int, q):
    try:
        from datetime import timedelta

        from moe_serving_profile_b200.parallel import ParallelGroup

        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
        pg = ParallelGroup(size)
        assert pg.size == size and pg.rank == rank % size and pg.start_rank == rank - rank % size
        block = rank // size
        # reduce: SUM over the block only
        t = torch.full((3,), float(rank + 1))
        pg.reduce(t)
        expect = sum(r + 1 for r in range(block * size, block * size + size))
        assert torch.equal(t, torch.full((3,), float(expect)))
        # broadcast from the block's rank 1
        b = torch.full((2,), float(rank))
        pg.broadcast(b, owner=1)
        assert torch.equal(b, torch.full((2,), float(pg.start_rank + 1)))
        # gather along dim 1
        gth = pg.gather(torch.full((2, 1), float(rank)), dim=1)
        assert torch.equal(gth, torch.arange(pg.start_rank, pg.start_rank + size).float().expand(2, size))
        # all_to_all with uneven splits: rank r sends (r + j + 1) rows to block rank j
        me = pg.rank
        in_splits = [me + j + 1 for j in range(size)]
        out_splits = [j + me + 1 for j in range(size)]
        inp = torch.cat([torch.full((n, 4), float(100 * me + j)) for j, n in enumerate(in_splits)])
        out = torch.empty(sum(out_splits), 4)
        pg.all_to_all(out, inp, out_splits, in_splits)
        ref = torch.cat([torch.full((n, 4), float(100 * j + me)) for j, n in enumerate(out_splits)])
        assert torch.equal(out, ref)
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, "ok"))
    except Exception as exc:  # report to the parent instead of hanging it
        q.put((rank, repr(exc)))


@pytest.mark.parametrize("world,size", [(2, 2), (4, 2)])
def test_parallel_group_collectives(world, size):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, size, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
    assert results == {r: "ok" for r in range(world)}, results


def test_parallel_group_rejects_bad_size():
    from moe_serving_profile_b200.parallel import ParallelGroup

    with pytest.raises(ValueError):
        ParallelGroup(0)
    assert ParallelGroup(1).size == 1


def _exchange_worker(rank: int, world: int, port: int, q):
    try:
        from datetime import timedelta

        from moe_serving_profile_b200 import native

        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
        coll = native.ProcessGroupCollective()
        assert native.collective_for(world) is not None and coll.world_size == world
        send = [rank + d + 1 for d in range(world)]            # rows to destination d
        rows = torch.cat([torch.full((n, 3), float(10 * rank + d)) for d, n in enumerate(send)])
        got, recv = coll.exchange(rows, torch.tensor(send))    # reference path (count exchange)
        expect_counts = [s + rank + 1 for s in range(world)]
        assert recv.tolist() == expect_counts
        ref = torch.cat([torch.full((n, 3), float(10 * s + rank)) for s, n in enumerate(expect_counts)])
        assert torch.equal(got, ref)
        got2, recv2 = coll.exchange(rows, send, expect_counts)  # known splits: no count exchange
        assert torch.equal(got2, ref) and recv2 == expect_counts
        back, _ = coll.exchange(got2, expect_counts, send)      # return trip restores the rows
        assert torch.equal(back, rows)
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, "ok"))
    except Exception as exc:
        q.put((rank, repr(exc)))


def test_process_group_collective_exchange():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_exchange_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
    assert results == {0: "ok", 1: "ok"}, results

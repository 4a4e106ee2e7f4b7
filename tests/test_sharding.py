"""CPU: the multi-GPU batch sharding logic (torchsoftdtw_b200.sharding) with world_size 2 gloo ranks,
plus the failure path of a rank that never joins (a short process-group timeout ends with an error)."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from torchsoftdtw_b200 import sharding


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_shard_bounds_cover_batch_exactly():
    for B in (0, 1, 7, 256, 65536, 1001):
        for world in (1, 2, 3, 4, 8):
            spans = [sharding.shard_bounds(B, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == B
            for (b0, e0), (b1, e1) in zip(spans, spans[1:]):
                assert e0 == b1
            sizes = [e - b for b, e in spans]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        sharding.shard_bounds(10, 2, 2)


def _worker(rank, world, port, B, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = torch.Generator().manual_seed(0)
        global_costs = torch.rand(B, generator=g, dtype=torch.float64)
        local = sharding.shard(global_costs, world, rank)
        total = sharding.all_reduce_loss(local.sum())
        pending = sharding.all_reduce_loss(local.sum(), async_op=True)  # the overlapped form of the bench
        total_async = pending.wait()
        gathered = sharding.gather_costs(local, B)
        out[rank] = (float(total), torch.equal(gathered, global_costs), float(global_costs.sum()), float(total_async))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("B", [7, 256])
def test_two_rank_loss_and_gather(B):
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    out = manager.dict()
    port = free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, B, out)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for r in range(2):
        total, same, expected, total_async = out[r]
        assert same
        assert abs(total - expected) < 1e-12
        assert total_async == total


def _lonely(port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime

    try:
        dist.init_process_group("gloo", rank=0, world_size=2, timeout=datetime.timedelta(seconds=3))
        q.put("joined")
    except Exception as e:  # the second rank never joins: rendezvous must fail, not hang
        q.put(type(e).__name__)


def test_missing_rank_fails_with_timeout():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_lonely, args=(free_port(), q))
    p.start()
    p.join(timeout=60)
    assert p.exitcode == 0
    assert q.get(timeout=5) != "joined"

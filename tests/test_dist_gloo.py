"""The multi-GPU host path on CPU: two gloo ranks take their batch x head shards (no data-path
collective) and agree on the max-over-ranks timing reduction the benchmark uses."""

import os
import socket

import pytest
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    import torch
    import torch.distributed as dist

    from nanosaur2_web_b200 import sharding
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        units = [(b, h) for b0, bc, h0, hc in sharding.shard_batch_heads(2, 16, world, rank)
                 for b in range(b0, b0 + bc) for h in range(h0, h0 + hc)]
        gathered = [None] * world
        dist.all_gather_object(gathered, units)
        t = sharding.max_over_ranks(float(rank + 1) * 1.5)
        tot = sharding.sum_over_ranks(float(rank + 1))
        q.put((rank, gathered, t, tot))
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(120)
def test_two_rank_sharding_and_timing_reduction():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=100) for _ in procs]
    for p in procs:
        p.join(timeout=30)
        assert p.exitcode == 0
    for rank, gathered, t, tot in results:
        allu = sorted(u for part in gathered for u in part)
        assert allu == [(b, h) for b in range(2) for h in range(16)]
        assert set(gathered[0]).isdisjoint(gathered[1])
        assert t == 3.0
        assert tot == 3.0

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


def _packed_kv(qkv, L, kv_len, k_w, cos, sin, rows):
    """k'|v' rows (head-normed k, 2D RoPE on image rows; raw v) of the given key rows, through the
    oracle; rows at or past kv_len stay zero."""
    import numpy as np

    from oracle import attention_oracle as O
    C = 16 * 96
    out = np.zeros((len(rows), 2 * C), dtype=np.float32)
    for i, r in enumerate(rows):
        if r >= kv_len:
            continue
        k = qkv[r:r + 1, C:2 * C]
        rope = (cos[r:r + 1], sin[r:r + 1]) if r < L else (None, None)
        out[i, :C] = O.head_norm(k, k_w, 16, 96, *rope)
        out[i, C:] = qkv[r, 2 * C:]
    return out


def _seq_worker(rank, world, port, q):
    import numpy as np
    import torch
    import torch.distributed as dist

    from nanosaur2_web_b200.seqshard import gather_views, seq_shard_rows
    from oracle import attention_oracle as O
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        B, h, w, Lt, kv_rows = 2, 4, 8, 8, 48
        L = h * w
        g = np.random.default_rng(7)   # same inputs on every rank
        qkv = g.standard_normal((B, L + Lt, 3 * 16 * 96)).astype(np.float32)
        k_w = (1 + 0.1 * g.standard_normal(96)).astype(np.float32)
        kv_len = [L + 5, L + Lt]
        cos, sin = O.rope_2d(h, w)
        q0, qn = seq_shard_rows(L, world, rank)
        kv = torch.full((B, kv_rows, 2 * 16 * 96), float("nan"))
        for b in range(B):
            # what this rank's prologue writes: its own image rows, then every text / padding row
            kv[b, q0:q0 + qn] = torch.from_numpy(_packed_kv(qkv[b], L, kv_len[b], k_w, cos, sin, range(q0, q0 + qn)))
            kv[b, L:] = torch.from_numpy(_packed_kv(qkv[b], L, kv_len[b], k_w, cos, sin, range(L, kv_rows)))
            out, inp = gather_views(kv, b, L, q0, qn)
            dist.all_gather_into_tensor(out, inp.clone())
        full = [_packed_kv(qkv[b], L, kv_len[b], k_w, cos, sin, range(kv_rows)) for b in range(B)]
        err = max(float(np.abs(kv[b].numpy() - full[b]).max()) for b in range(B))
        q.put((rank, err))
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(120)
def test_two_rank_sequence_shard_gather_assembles_all_keys():
    """Each rank writes the k'|v' rows of its own image rows and of all text rows; the per-element
    all-gather over the views the CUDA path uses yields every rank the full key set."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_seq_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=100) for _ in procs]
    for p in procs:
        p.join(timeout=30)
        assert p.exitcode == 0
    for rank, err in results:
        assert err == 0.0, (rank, err)


def _gate_worker(rank, world, port, leave_after, q):
    """Ranks step through a StepGate; rank world-1 leaves between steps after ``leave_after`` steps
    (no collective in flight).  The others must see PeerTimeout at the next step's gate, naming it,
    before any collective of that step, and then abort the process group."""
    import torch
    import torch.distributed as dist

    from nanosaur2_web_b200 import health
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    health.init_process_group_bounded("gloo", rank, world, timeout_s=20)
    gate = health.StepGate(health.default_store(), rank, world, timeout_s=1.5)
    steps_done, result = 0, None
    try:
        for step in range(4):
            if rank == world - 1 and step == leave_after:
                result = ("left", step)
                break
            gate.enter(step)
            t = torch.tensor([float(rank)])
            dist.all_reduce(t)   # the step's collective: only reached when every rank is present
            assert t.item() == sum(range(world))
            steps_done += 1
        else:
            result = ("done", steps_done)
    except health.PeerTimeout as e:
        result = ("timeout", e.step, e.missing, steps_done)
    if result[0] == "left":
        q.put((rank, result))
        q.close()
        q.join_thread()   # the result must reach the parent before the hard exit
        os._exit(0)   # leave without a goodbye, as a crashed rank would
    health.abort_process_group()
    q.put((rank, result))


@pytest.mark.timeout(120)
def test_step_gate_detects_a_rank_that_left():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    world = 3
    procs = [ctx.Process(target=_gate_worker, args=(r, world, port, 2, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=100) for _ in procs)
    for p in procs:
        p.join(timeout=30)
        assert p.exitcode == 0
    assert results[2] == ("left", 2)
    for r in (0, 1):
        assert results[r] == ("timeout", 2, [2], 2), results[r]


@pytest.mark.timeout(120)
def test_step_gate_passes_when_every_rank_arrives():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gate_worker, args=(r, 2, port, 99, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=100) for _ in procs)
    for p in procs:
        p.join(timeout=30)
        assert p.exitcode == 0
    assert results == {0: ("done", 4), 1: ("done", 4)}

"""Batch sharding without a GPU: bucketing, LPT balance, pass planning, and the gather that restores
the original order, the last over a world-size-2 gloo process group on the CPU."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest


@pytest.fixture(scope="module")
def shard():
    from conftest import load_e2c

    load_e2c()
    import e2c_b200.shard as s

    return s


def test_log_uniform_lengths_and_buckets(shard):
    rng = np.random.default_rng(0)
    lens = shard.log_uniform_lengths(rng, 65536)
    assert lens.min() >= 32 and lens.max() <= 2048
    assert 400 < lens.mean() < 560                  # mean of floor(exp(U[ln 32, ln 2048])) ~ 485
    pad = shard.bucket_length(lens, 64)
    assert np.all(pad % 64 == 0) and np.all(pad >= lens) and np.all(pad - lens < 64)


def test_lpt_covers_every_sequence_once_and_balances(shard):
    rng = np.random.default_rng(1)
    lens = shard.bucket_length(shard.log_uniform_lengths(rng, 4096), 64)
    cost = shard.sequence_cost(lens)
    for world in (1, 2, 4, 8):
        parts = shard.lpt_assign(cost, world)
        allidx = np.concatenate(parts)
        assert np.array_equal(np.sort(allidx), np.arange(len(lens)))
        loads = np.array([cost[p].sum() for p in parts])
        # LPT: the spread of the loads is at most one sequence's cost
        assert loads.max() - loads.min() <= cost.max() + 1e-6


def test_passes_respect_the_token_budget(shard):
    rng = np.random.default_rng(2)
    lens = shard.log_uniform_lengths(rng, 1000)
    pad = shard.bucket_length(lens, 64)
    passes = shard.plan_passes(np.arange(1000), pad, max_tokens=32768)
    seen = np.concatenate([p.seqs for p in passes])
    assert np.array_equal(np.sort(seen), np.arange(1000))
    for p in passes:
        assert np.all(pad[p.seqs] == p.length)
        assert len(p.seqs) * p.length <= max(32768, p.length)
    ids, valid = shard.pack_batch(lambda i: np.full(int(lens[i]), i + 2, np.int32), lens, passes[0])
    for r, i in enumerate(passes[0].seqs):
        assert valid[r].sum() == lens[i] and np.all(ids[r, : lens[i]] == i + 2) and np.all(ids[r, lens[i]:] == 0)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gather_worker(rank: int, world: int, port: int, n: int, q):
    import torch
    import torch.distributed as dist

    from conftest import load_e2c

    load_e2c()
    import e2c_b200.shard as shard

    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rng = np.random.default_rng(5)  # the same plan on every rank
        lens = shard.bucket_length(shard.log_uniform_lengths(rng, n), 64)
        shares = shard.lpt_assign(shard.sequence_cost(lens), world)
        mine = shares[rank]
        # stand-in embeddings: row i is a function of the sequence index only
        emb = torch.stack([torch.full((8,), float(i)) + torch.arange(8.0) for i in mine]) if len(mine) else \
            torch.zeros((0, 8))
        out = shard.gather_embeddings(dist, shares, emb, n)
        want = torch.arange(n, dtype=torch.float32)[:, None] + torch.arange(8.0)[None, :]
        q.put((rank, bool(torch.equal(out, want)), len(mine)))
    finally:
        dist.destroy_process_group()


def test_gather_restores_order_over_two_gloo_ranks():
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port, n, world = _free_port(), 333, 2
    procs = [ctx.Process(target=_gather_worker, args=(r, world, port, n, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert all(ok for _, ok, _ in res), res
    assert sum(c for _, _, c in res) == n

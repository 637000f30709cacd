"""Request sharding across GPUs (host logic, CPU): the greedy assignment, the
packing, the config-4 length generator, and the N > 1 bookkeeping on a
world-size-2 gloo process group."""
import os
import socket

import numpy as np
import pytest

from tokenvector.inference_b200 import sharding as S


def test_shard_covers_every_request_once_and_balances():
    lengths = S.ragged_lengths(256, 131072, 32, 1024, seed=4)
    for world in (1, 2, 4, 8):
        shards = S.shard_requests(lengths, world)
        flat = sorted(i for s in shards for i in s)
        assert flat == list(range(256))
        loads = [sum(lengths[i] for i in s) for s in shards]
        assert sum(loads) == 131072
        # LPT bound: max load <= ideal + longest request
        assert max(loads) <= 131072 / world + max(lengths)
        assert all(s == sorted(s) for s in shards)


def test_shard_is_deterministic_and_ties_go_to_lower_rank():
    assert S.shard_requests([5, 5, 5, 5], 2) == [[0, 2], [1, 3]]
    assert S.shard_requests([1], 3) == [[0], [], []]
    assert S.shard_requests([3, 9, 3], 2) == [[1], [0, 2]]
    with pytest.raises(ValueError):
        S.shard_requests([0, 3], 2)
    with pytest.raises(ValueError):
        S.shard_requests([3], 0)


def test_pack_segments():
    assert S.pack_segments([3, 1, 4]).tolist() == [0, 3, 4, 8]
    assert S.pack_segments([]).tolist() == [0]


def test_ragged_lengths_config4():
    x = S.ragged_lengths(256, 131072, 32, 1024, seed=0)
    assert len(x) == 256 and sum(x) == 131072
    assert min(x) >= 32 and max(x) <= 1024
    assert x == S.ragged_lengths(256, 131072, 32, 1024, seed=0)
    with pytest.raises(ValueError):
        S.ragged_lengths(4, 10, 32, 1024, seed=0)


def test_plan_per_rank():
    lengths = [100, 37, 64, 1, 900, 5]
    plans = [S.plan(lengths, 2, r) for r in range(2)]
    assert sorted(plans[0].requests + plans[1].requests) == list(range(6))
    for p in plans:
        assert p.seg[0] == 0 and p.tokens == sum(p.lengths)
        assert p.lengths == [lengths[i] for i in p.requests]


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, lengths, q):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        p = S.plan(lengths, world, rank)
        counts = S.gather_counts(p.tokens)
        # a per-rank "step time" that differs by rank: the max is the slowest
        t = S.max_over_ranks(1.0 + rank * 0.5)
        q.put((rank, p.requests, counts, t))
    finally:
        dist.destroy_process_group()


def test_two_rank_gloo_bookkeeping():
    import torch.multiprocessing as mp
    lengths = S.ragged_lengths(32, 8000, 32, 1024, seed=7)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, lengths, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(2)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    res.sort()
    shards = S.shard_requests(lengths, 2)
    for rank, req, counts, t in res:
        assert req == shards[rank]
        assert counts == [sum(lengths[i] for i in shards[r]) for r in range(2)]
        assert t == 1.5

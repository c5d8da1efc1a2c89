"""Multi-rank host logic on CPU: world_size 2 over gloo (127.0.0.1).

The path shards requests across ranks with no data-path collective; the
search results are all-gathered once and the step time is the max over ranks.
"""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, q) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime

    from kadllm_b200.shard import all_ranks, gather_beams, max_over_ranks, rank_prompts

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        B, W, D, L, V = 3, 4, 2, 16, 1000
        ids = rank_prompts(rank, B, L, V)
        # a stand-in search result that encodes the rank and the prompts
        tokens = torch.from_numpy(ids[:, :W * D].reshape(B, W, D).copy()) + rank * V
        scores = torch.full((B, W), -float(rank), dtype=torch.float32) - torch.arange(W, dtype=torch.float32)
        all_t, all_s = gather_beams(tokens, scores)
        slow = max_over_ranks(10.0 + rank)
        every = all_ranks(10.0 + rank)
        q.put((rank, ids, all_t.numpy(), all_s.numpy(), slow, every))
    finally:
        dist.destroy_process_group()


def test_two_rank_shards_gather_and_max():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = {}
    for _ in range(world):
        rank, ids, all_t, all_s, slow, every = q.get(timeout=120)
        got[rank] = (ids, all_t, all_s, slow, every)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    ids0, ids1 = got[0][0], got[1][0]
    assert not np.array_equal(ids0, ids1)  # each rank serves its own requests
    B, W, D, V = 3, 4, 2, 1000
    want_t = np.concatenate([ids0[:, :W * D].reshape(B, W, D), ids1[:, :W * D].reshape(B, W, D) + V])
    for r in range(world):
        _, all_t, all_s, slow, every = got[r]
        np.testing.assert_array_equal(all_t, want_t)  # rank order, identical on every rank
        assert all_s.shape == (world * B, W)
        np.testing.assert_array_equal(all_s[:B, 0], 0.0)
        np.testing.assert_array_equal(all_s[B:, 0], -1.0)
        assert slow == 11.0  # max over ranks
        assert every == [10.0, 11.0]  # every rank's value, in rank order


def test_single_process_identity():
    from kadllm_b200.shard import all_ranks, gather_beams, max_over_ranks

    t = torch.arange(6).reshape(1, 3, 2)
    s = torch.zeros(1, 3)
    a, b = gather_beams(t, s)
    assert a is t and b is s
    assert max_over_ranks(2.5) == 2.5
    assert all_ranks(2.5) == [2.5]

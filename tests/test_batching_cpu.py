"""Request partitioning across ranks (one process per GPU, no data-path
collective) and the timing / result gathering that is the only traffic
between ranks: checked on CPU with world_size 2 over the ``gloo`` backend."""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from soraku_tts_b200.batching import gather_codes, max_over_ranks, split_requests


def test_split_covers_every_request_once_and_balances():
    rng = np.random.default_rng(3)
    costs = (rng.integers(16, 97, 64) + rng.integers(24, 145, 64) + 250).tolist()
    for world in (1, 2, 3, 4, 8):
        parts = split_requests(costs, world)
        assert len(parts) == world
        flat = sorted(i for p in parts for i in p)
        assert flat == list(range(64))
        loads = [sum(costs[i] for i in p) for p in parts]
        # greedy longest-first: no rank exceeds the mean by more than the largest request
        assert max(loads) - sum(loads) / world <= max(costs)
        assert max(len(p) for p in parts) - min(len(p) for p in parts) <= 2


def test_split_edge_cases():
    assert split_requests([], 4) == [[], [], [], []]
    assert split_requests([5], 3) == [[0], [], []]
    # equal costs: round robin over ranks, deterministic
    assert split_requests([1, 1, 1, 1], 2) == [[0, 2], [1, 3]]
    with pytest.raises(ValueError):
        split_requests([1], 0)


def test_single_process_helpers_without_group():
    assert max_over_ranks(2.5) == 2.5
    codes = {3: np.zeros((2, 16), np.int64)}
    assert gather_codes(codes).keys() == {3}


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, q):
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        costs = [100 + 7 * i for i in range(10)]
        mine = split_requests(costs, world)[rank]
        # stand-in for this rank's decode: codes that name their request
        local = {i: np.full((4, 16), i, np.int64) for i in mine}
        slowest = max_over_ranks(1.0 + rank)
        merged = gather_codes(local)
        if rank == 0:
            q.put((slowest, sorted(merged), all(int(v[0, 0]) == k for k, v in merged.items())))
        else:
            q.put((slowest, merged, None))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_two_rank_partition_and_gather_over_gloo():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    slowest = {r[0] for r in results}
    assert slowest == {2.0}  # both ranks see the max over ranks
    root = [r for r in results if r[2] is not None]
    others = [r for r in results if r[2] is None]
    assert len(root) == 1 and len(others) == 1
    assert root[0][1] == list(range(10)) and root[0][2]
    assert others[0][1] is None

"""Multi-request decode across GPUs: requests are partitioned by rank (one
process per GPU, no collective on the data path) and only timing and the
generated codes travel over ``torch.distributed`` afterwards.

The reference serves one utterance per generator call
(``fast_generate.py`` ``FastGenerator.generate``); a batch of requests is a
list of such calls.  Here each rank decodes its share of the list as one
batched engine step (2 CFG rows per request), so ranks never exchange
activations.
"""

from __future__ import annotations

from typing import Sequence

import numpy as np


def split_requests(costs: Sequence[int], world: int) -> list[list[int]]:
    """Static partition of request indices over ``world`` ranks, balanced on
    ``costs`` (e.g. prompt length + frames to generate, the KV positions a
    request keeps): longest first, each to the least-loaded rank (ties: the
    lowest rank).  Every index appears exactly once; each part is sorted."""
    if world < 1:
        raise ValueError(f"world must be >= 1, got {world}")
    order = sorted(range(len(costs)), key=lambda i: (-int(costs[i]), i))
    load = [0] * world
    parts: list[list[int]] = [[] for _ in range(world)]
    for i in order:
        w = min(range(world), key=lambda k: (load[k], k))
        parts[w].append(i)
        load[w] += int(costs[i])
    return [sorted(p) for p in parts]


def max_over_ranks(value: float, device=None) -> float:
    """The largest ``value`` over all ranks (the job's time is its slowest
    rank's); the value itself without an initialised process group."""
    import torch
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()):
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def gather_codes(local: dict[int, np.ndarray], dst: int = 0) -> dict[int, np.ndarray] | None:
    """Collects every rank's {request index: codes [frames, Q]} on rank
    ``dst`` (None elsewhere).  Raises if two ranks report the same request."""
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()):
        return dict(local)
    world = dist.get_world_size()
    rank = dist.get_rank()
    payload = {int(k): np.asarray(v) for k, v in local.items()}
    box = [None] * world if rank == dst else None
    dist.gather_object(payload, box, dst=dst)
    if rank != dst:
        return None
    merged: dict[int, np.ndarray] = {}
    for part in box:
        for k, v in part.items():
            if k in merged:
                raise RuntimeError(f"request {k} decoded on two ranks")
            merged[k] = v
    return merged

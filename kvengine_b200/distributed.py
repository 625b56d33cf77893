"""Data-parallel request sharding across GPUs (one process per GPU).

Greedy speculative output for a request depends only on that request, so the
requests of a job are split across ranks with no exchange during decoding.
Each rank holds a full draft + target replica and its own KV pools; the only
collective is `gather_tokens`, run once after decoding to collect every
request's tokens on every rank (NCCL on GPUs, gloo in CPU tests).
"""

from __future__ import annotations

import torch
import torch.distributed as dist


def shard_requests(costs: list[int], world: int) -> list[list[int]]:
    """Longest-processing-time assignment of request indices to ranks.

    `costs` estimates each request's work (e.g. prompt + output length). Requests
    are taken longest first (ties by index) and each goes to the rank with the
    least work so far (ties by rank), so the split is deterministic.
    """
    if world < 1:
        raise ValueError("world must be >= 1")
    order = sorted(range(len(costs)), key=lambda i: (-costs[i], i))
    load = [0] * world
    shards: list[list[int]] = [[] for _ in range(world)]
    for i in order:
        r = min(range(world), key=lambda j: (load[j], j))
        shards[r].append(i)
        load[r] += costs[i]
    for s in shards:
        s.sort()
    return shards


def contiguous_shards(n: int, world: int) -> list[list[int]]:
    """Rank r gets requests [r*n/world, (r+1)*n/world)."""
    return [list(range(r * n // world, (r + 1) * n // world)) for r in range(world)]


def gather_tokens(local: dict[int, list[int]], device: torch.device | str = "cpu",
                  group=None) -> dict[int, list[int]]:
    """All-gather {request index: token list} from every rank (untimed, after decoding).

    Sizes are exchanged first, then one padded int32 tensor per rank
    ([n_local, 2 + max_len]: index, length, tokens).
    """
    world = dist.get_world_size(group)
    device = torch.device(device)
    max_len = max((len(v) for v in local.values()), default=0)
    meta = torch.tensor([len(local), max_len], dtype=torch.int64, device=device)
    metas = [torch.zeros_like(meta) for _ in range(world)]
    dist.all_gather(metas, meta, group=group)
    rows = max(int(m[0]) for m in metas)
    width = 2 + max(int(m[1]) for m in metas)
    buf = torch.full((max(rows, 1), width), -1, dtype=torch.int32, device=device)
    for r, (idx, toks) in enumerate(sorted(local.items())):
        buf[r, 0] = idx
        buf[r, 1] = len(toks)
        if toks:
            buf[r, 2:2 + len(toks)] = torch.tensor(toks, dtype=torch.int32, device=device)
    bufs = [torch.empty_like(buf) for _ in range(world)]
    dist.all_gather(bufs, buf, group=group)
    out: dict[int, list[int]] = {}
    for b, m in zip(bufs, metas):
        b = b.cpu()
        for r in range(int(m[0])):
            idx, n = int(b[r, 0]), int(b[r, 1])
            out[idx] = b[r, 2:2 + n].tolist()
    return out

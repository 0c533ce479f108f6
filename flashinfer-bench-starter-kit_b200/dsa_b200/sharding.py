"""Request sharding for data-parallel DSA decode on one node.

Decode requests are independent, so a batch is split by request across the
GPUs; each GPU holds its own page pools (FP8 index cache, ckv, kpe) and block
table for its requests, and no collective runs on the hot path.  The split
balances context tokens (the indexer's work is 132 B per token, attention's
is fixed per request): requests are assigned longest-first to the rank with
the fewest tokens so far (LPT), ties to the lower rank, and each rank keeps
its requests in their original order.
"""

from __future__ import annotations


def shard_requests(seq_lens: list, world: int) -> list:
    """Returns one list of request indices per rank."""
    if world < 1:
        raise ValueError("world must be >= 1")
    load = [0] * world
    count = [0] * world
    shards = [[] for _ in range(world)]
    order = sorted(range(len(seq_lens)), key=lambda i: (-int(seq_lens[i]), i))
    for i in order:
        # token load, then request count (attention work), then rank id
        r = min(range(world), key=lambda k: (load[k], count[k], k))
        shards[r].append(i)
        load[r] += max(0, int(seq_lens[i]))
        count[r] += 1
    return [sorted(s) for s in shards]


def shard_imbalance(seq_lens: list, shards: list) -> float:
    """max rank tokens / mean rank tokens (1.0 = perfect)."""
    loads = [sum(max(0, int(seq_lens[i])) for i in s) for s in shards]
    mean = sum(loads) / max(1, len(loads))
    return max(loads) / mean if mean > 0 else 1.0


def reduce_step_stats(ms_total: float, rank_bytes: float, rank_requests: float, world: int) -> tuple:
    """Whole-job step statistics from every rank's: time is the MAX over ranks
    (the job is done when its slowest rank is), bytes and requests are SUMS.
    Uses torch.distributed when world > 1 (NCCL on GPUs, gloo on CPU); every
    rank must call it, in the same order as its other collectives."""
    import torch

    if world <= 1:
        return float(ms_total), float(rank_bytes), float(rank_requests)
    import torch.distributed as dist

    backend = dist.get_backend()
    dev = torch.device("cuda", torch.cuda.current_device()) if backend == "nccl" else torch.device("cpu")
    stats = torch.tensor([ms_total, rank_bytes, rank_requests], dtype=torch.float64, device=dev)
    mx = stats.clone()
    dist.all_reduce(mx, op=dist.ReduceOp.MAX)
    sm = stats.clone()
    dist.all_reduce(sm, op=dist.ReduceOp.SUM)
    return float(mx[0]), float(sm[1]), float(sm[2])


def gather_outputs(tensors: list, world: int) -> list:
    """All-gathers one decode shard's output tensors -- e.g. (topk_indices,
    output, lse), each with the rank's requests as dimension 0 -- from every
    rank, padded to the largest shard so one collective per tensor suffices.
    Returns, per rank, the list of its tensors trimmed to its own request
    count.  Every rank must call it (NCCL on GPUs, gloo on CPU); it is meant
    for verification outside the timed region, never the hot path."""
    import torch

    if world <= 1:
        return [list(tensors)]
    import torch.distributed as dist

    dev = tensors[0].device
    n = torch.tensor([tensors[0].shape[0]], dtype=torch.int64, device=dev)
    counts = [torch.zeros_like(n) for _ in range(world)]
    dist.all_gather(counts, n)
    counts = [int(c) for c in counts]
    bmax = max(counts)
    per_rank = [[] for _ in range(world)]
    for t in tensors:
        pad = torch.zeros((bmax,) + tuple(t.shape[1:]), dtype=t.dtype, device=t.device)
        pad[: t.shape[0]] = t
        parts = [torch.empty_like(pad) for _ in range(world)]
        dist.all_gather(parts, pad)
        for r in range(world):
            per_rank[r].append(parts[r][: counts[r]])
    return per_rank

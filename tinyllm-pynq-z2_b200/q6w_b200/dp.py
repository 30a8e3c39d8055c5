"""Data-parallel request sharding across GPUs (host side, no collectives on the data path).

Requests are independent and the model is replicated per GPU, so a run is
split on the host before any GPU work: each rank takes its share of the
requests, runs them alone, and results are gathered after timing.  For
ragged prompts the split balances prompt tokens (the prefill work), not
request counts.  A rank that fails leaves its share to be re-queued over the
survivors.
"""

import heapq


def shard_range(n_total, rank, world):
    """Contiguous, balanced [lo, hi) slice of n_total items for ``rank``."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("need 0 <= rank < world")
    base, extra = divmod(n_total, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def balance_by_tokens(lengths, world):
    """Assign item indices to ``world`` ranks, longest first, each to the rank
    with the fewest tokens so far (greedy LPT).  Returns a list of index lists
    (each sorted); the heaviest rank exceeds the lightest by at most the
    longest single item."""
    if world < 1:
        raise ValueError("world must be >= 1")
    heap = [(0, r) for r in range(world)]
    out = [[] for _ in range(world)]
    for i in sorted(range(len(lengths)), key=lambda i: (-lengths[i], i)):
        load, r = heapq.heappop(heap)
        out[r].append(i)
        heapq.heappush(heap, (load + int(lengths[i]), r))
    return [sorted(x) for x in out]


def requeue(assignments, failed, lengths=None):
    """Redistribute the items of ``failed`` ranks over the surviving ranks.

    ``assignments``: list of index lists per rank.  Returns a new list where
    failed ranks hold nothing and survivors additionally hold the orphaned
    items (balanced by ``lengths`` when given, else by count).
    """
    failed = set(failed)
    alive = [r for r in range(len(assignments)) if r not in failed]
    if not alive:
        raise RuntimeError("no surviving rank to take the work")
    orphans = [i for r in failed for i in assignments[r]]
    w = [1] * (max(orphans) + 1 if orphans else 0) if lengths is None else lengths
    extra = balance_by_tokens([w[i] for i in orphans], len(alive))
    out = [list(a) if r not in failed else [] for r, a in enumerate(assignments)]
    for k, r in enumerate(alive):
        out[r] = sorted(out[r] + [orphans[j] for j in extra[k]])
    return out


def gather_to_rank0(obj, world):
    """Gather one picklable object per rank to rank 0 (call outside timed regions)."""
    import torch.distributed as dist

    if world == 1:
        return [obj]
    buf = [None] * world if dist.get_rank() == 0 else None
    dist.gather_object(obj, buf, dst=0)
    return buf

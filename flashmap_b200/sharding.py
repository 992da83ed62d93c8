"""Request sharding of drafting across GPUs: one process per GPU, each with a
full weight replica, drafting its own requests.  No collective is on the
drafting path: every rank derives its share from the same inputs.

A request's cost is modelled as ``a + b * C`` (C = its context length): the
GEMM work of a draft is the same for every request, the cross-attention work
grows with the context.  Requests are assigned by longest-processing-time
first (Graham's LPT rule): in decreasing cost order, each goes to the rank
with the smallest load so far (lowest rank on ties), which keeps the slowest
rank within one request of the mean.  With a ``capacity`` (requests per rank)
only ranks below it take requests: ``balanced_capacity`` gives every rank the
same count to within one, so that no rank drafts one short extra batch (a
batch of a few requests costs almost a full weight pass).  Large shares are
then drafted in chunks of at most ``chunk`` requests (the context cache of 64
long requests already holds tens of GB).
"""

from __future__ import annotations

from typing import List, Optional, Sequence

# cost of one draft in units of one context position.  Drafting many requests
# per GPU runs the GEMMs tensor-bound: one request's share of them (about 40
# GFLOP at the config-2/5 sizes, ~25-30 us) costs about what streaming the
# cross-attention keys and values of 2000 context positions (64-100 KB each)
# costs, so a request weighs 2000 + C.
DEFAULT_FIXED_COST = 2000.0
DEFAULT_PER_POSITION = 1.0


def request_costs(context_lengths: Sequence[int], fixed: float = DEFAULT_FIXED_COST,
                  per_position: float = DEFAULT_PER_POSITION) -> List[float]:
    return [fixed + per_position * float(c) for c in context_lengths]


def balanced_capacity(n_requests: int, world_size: int) -> int:
    """Requests per rank when every rank drafts the same count to within one."""
    if world_size < 1:
        raise ValueError("world_size must be at least 1")
    return -(-n_requests // world_size)


def lpt_assign(costs: Sequence[float], world_size: int, capacity: Optional[int] = None) -> List[List[int]]:
    """Request indices per rank, longest-processing-time first.  Deterministic:
    ties in cost keep request order, ties in load go to the lower rank.  With
    ``capacity``, a rank holding that many requests takes no more."""
    if world_size < 1:
        raise ValueError("world_size must be at least 1")
    if capacity is not None and capacity * world_size < len(costs):
        raise ValueError(f"capacity {capacity} x {world_size} ranks holds fewer than {len(costs)} requests")
    order = sorted(range(len(costs)), key=lambda i: (-costs[i], i))
    loads = [0.0] * world_size
    shares: List[List[int]] = [[] for _ in range(world_size)]
    for i in order:
        open_ranks = [k for k in range(world_size) if capacity is None or len(shares[k]) < capacity]
        r = min(open_ranks, key=lambda k: (loads[k], k))
        shares[r].append(i)
        loads[r] += costs[i]
    return [sorted(s) for s in shares]


def shard_requests(context_lengths: Sequence[int], world_size: int, rank: int, capacity: Optional[int] = None,
                   **cost_kw) -> List[int]:
    """This rank's request indices."""
    if not 0 <= rank < world_size:
        raise ValueError(f"rank {rank} outside world of {world_size}")
    return lpt_assign(request_costs(context_lengths, **cost_kw), world_size, capacity)[rank]


def chunks(indices: Sequence[int], chunk: int = 64) -> List[List[int]]:
    """A rank's share in drafting batches of at most `chunk` requests."""
    if chunk < 1:
        raise ValueError("chunk must be at least 1")
    return [list(indices[i:i + chunk]) for i in range(0, len(indices), chunk)]


def shard_loads(context_lengths: Sequence[int], world_size: int, capacity: Optional[int] = None,
                **cost_kw) -> List[float]:
    costs = request_costs(context_lengths, **cost_kw)
    return [sum(costs[i] for i in s) for s in lpt_assign(costs, world_size, capacity)]


__all__ = ["balanced_capacity", "chunks", "lpt_assign", "request_costs", "shard_loads", "shard_requests"]

"""Host request router for data-parallel serving: one process, pool and
allocator per GPU, and nothing on the data path crosses GPUs.

The reference serves from one process (``AsyncEngine`` over one
``BlockAllocator``, engine/serving/async_engine.py); scaling it out to N GPUs
means N such engines and a router in front of them. Two rules decide the rank
of a request:

* least outstanding tokens: the rank with the fewest prompt + output tokens
  admitted and not yet released takes the request (ties go to the lowest
  rank);
* prefix-group affinity: requests that share a prefix key (the shared-prefix
  groups of a prefix-cache workload) go to the rank that served the group
  first, so its cached blocks are hit, unless that rank's load exceeds the
  least loaded rank's by more than ``affinity_slack`` tokens.

``RequestRouter`` is the live form (``release`` as requests finish).
``route_trace`` replays a whole trace with the tokens a request holds counted
until the end of the trace: a pure function of the trace, so every rank can
compute the same assignment and keep its own share without any exchange.
"""
from __future__ import annotations

from typing import Dict, Hashable, List, Optional, Sequence


class RequestRouter:
    def __init__(self, num_ranks: int, affinity_slack: int = 16384):
        if num_ranks < 1:
            raise ValueError("num_ranks must be >= 1")
        self.num_ranks = num_ranks
        self.affinity_slack = affinity_slack
        self.load: List[int] = [0] * num_ranks
        self.prefix_rank: Dict[Hashable, int] = {}

    def least_loaded(self) -> int:
        return min(range(self.num_ranks), key=lambda r: (self.load[r], r))

    def assign(self, tokens: int, prefix_key: Optional[Hashable] = None) -> int:
        """Rank for a request holding ``tokens`` (prompt + output) tokens."""
        if tokens < 0:
            raise ValueError("tokens must be >= 0")
        best = self.least_loaded()
        rank = best
        if prefix_key is not None:
            home = self.prefix_rank.get(prefix_key)
            if home is None:
                self.prefix_rank[prefix_key] = best
            elif self.load[home] - self.load[best] <= self.affinity_slack:
                rank = home
        self.load[rank] += tokens
        return rank

    def release(self, rank: int, tokens: int) -> None:
        """A request of ``tokens`` tokens on ``rank`` finished."""
        if not 0 <= rank < self.num_ranks:
            raise ValueError(f"rank {rank} out of range")
        if tokens > self.load[rank]:
            raise ValueError(f"rank {rank} releases {tokens} tokens but holds {self.load[rank]}")
        self.load[rank] -= tokens


def route_trace(tokens: Sequence[int], num_ranks: int, prefix_keys: Optional[Sequence[Hashable]] = None,
                affinity_slack: int = 16384) -> List[int]:
    """Rank of every request of a trace, in arrival order (see the module
    docstring); identical on every process that calls it with the same trace."""
    router = RequestRouter(num_ranks, affinity_slack)
    keys = prefix_keys if prefix_keys is not None else [None] * len(tokens)
    if len(keys) != len(tokens):
        raise ValueError("prefix_keys and tokens differ in length")
    return [router.assign(int(t), k) for t, k in zip(tokens, keys)]

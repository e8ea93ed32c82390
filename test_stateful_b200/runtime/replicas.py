"""Request-sharded replicas across the GPUs of one box.

The reference serves one GPU per process and scales by running more
processes (engine/server.py:995 ``--device``); nothing crosses between
streams except the per-process prefix cache.  The B200 build keeps that:
one process per GPU, each with its own weights, paged pool and prefix cache,
and a host router that places a new session on a replica.  No collective runs
on the decode path; ``torch.distributed`` is used only to agree on the routing
table and to report timings (max over ranks).
"""

from __future__ import annotations

from typing import Dict, List, Optional, Sequence, Tuple


class ReplicaRouter:
    """Least-loaded placement with prefix-key affinity.

    A session whose prefix key was placed before goes to the same replica
    while it has room (its prefix blocks are cached there); otherwise the
    replica with the fewest active sessions (lowest index on ties).
    """

    def __init__(self, n_replicas: int, capacity: int):
        if n_replicas < 1 or capacity < 1:
            raise ValueError("need at least one replica and capacity >= 1")
        self.n = n_replicas
        self.capacity = capacity
        self.load: List[int] = [0] * n_replicas
        self.where: Dict[str, int] = {}
        self.prefix_home: Dict[str, int] = {}

    def route(self, session_id: str, prefix_key: Optional[str] = None) -> int:
        if session_id in self.where:
            return self.where[session_id]
        home = self.prefix_home.get(prefix_key) if prefix_key is not None else None
        if home is not None and self.load[home] < self.capacity:
            r = home
        else:
            r = min(range(self.n), key=lambda i: (self.load[i], i))
            if self.load[r] >= self.capacity:
                raise RuntimeError("all replicas are full")
            if prefix_key is not None and prefix_key not in self.prefix_home:
                self.prefix_home[prefix_key] = r
        self.where[session_id] = r
        self.load[r] += 1
        return r

    def release(self, session_id: str) -> None:
        r = self.where.pop(session_id, None)
        if r is not None:
            self.load[r] -= 1


def assign_sessions(sessions: Sequence[Tuple[str, Optional[str]]], world: int, capacity: int) -> List[int]:
    """Route a batch of (session_id, prefix_key) in arrival order."""
    router = ReplicaRouter(world, capacity)
    return [router.route(s, k) for s, k in sessions]


def share_routing(sessions, rank: int, world: int, capacity: int):
    """Rank 0 routes; every rank receives the table and keeps its own sessions."""
    import torch.distributed as dist
    table = [assign_sessions(sessions, world, capacity) if rank == 0 else None]
    if world > 1:
        dist.broadcast_object_list(table, src=0)
    return [s for s, r in zip(sessions, table[0]) if r == rank], table[0]


def max_over_ranks(value: float, world: int, device=None) -> float:
    """Max of a per-rank measurement (timings are reported as the slowest rank)."""
    if world <= 1:
        return float(value)
    import torch
    import torch.distributed as dist
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())

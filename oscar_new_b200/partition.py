"""Split of one attention workload over the GPUs of a box: KV heads x requests.

Decode and verify attention need no collective: a (request, KV head) pair reads only
its own cache pages and writes only its own query heads' outputs.  The split follows
the reference deployment: tensor parallelism over KV heads first (each rank holds
``num_kv_heads / tp`` heads and their ``group`` query heads; the reference's target is
TP4 with one KV head per rank, ``oscar_ascend/backend.py:92-93``), then the requests
are divided among the ``world / tp`` request groups, balanced by total context length
(the work of a request is proportional to its context).

Every rank computes the same plan from the same host inputs (no communication); a
rank's cache holds only its heads, and its batch only its requests, in the order of
``Shard.requests``.
"""

from __future__ import annotations

import math
from dataclasses import dataclass


@dataclass(frozen=True)
class Shard:
    rank: int
    head_begin: int  # KV heads [head_begin, head_end) of this rank
    head_end: int
    requests: tuple  # request ids (ascending) of this rank's batch

    @property
    def kv_heads(self) -> int:
        return self.head_end - self.head_begin

    def query_heads(self, group: int) -> range:
        """Query heads of the rank's KV heads (head h serves h*group .. h*group + group - 1)."""
        return range(self.head_begin * group, self.head_end * group)


def head_split(kv_heads: int, world: int, min_heads_per_rank: int = 1) -> int:
    """Tensor-parallel degree over KV heads: the largest common divisor of both that
    leaves every rank at least `min_heads_per_rank` KV heads (1: the model's TP split)."""
    if kv_heads <= 0 or world <= 0 or min_heads_per_rank <= 0:
        raise ValueError("kv_heads, world and min_heads_per_rank must be positive")
    g = math.gcd(kv_heads, world)
    while g > 1 and kv_heads // g < min_heads_per_rank:
        g -= 1
        while g > 1 and (kv_heads % g or world % g):
            g -= 1
    return g


def balance_requests(context_lens, groups: int) -> list:
    """Requests into `groups` lists of nearly equal total context: longest first, each to
    the group with the least context so far (ties: the lower group).  Deterministic; each
    list ascending.  The largest group exceeds the mean by less than one request's
    context."""
    if groups <= 0:
        raise ValueError("groups must be positive")
    order = sorted(range(len(context_lens)), key=lambda r: (-int(context_lens[r]), r))
    load = [0] * groups
    members = [[] for _ in range(groups)]
    for r in order:
        g = min(range(groups), key=lambda i: (load[i], i))
        load[g] += int(context_lens[r])
        members[g].append(r)
    return [sorted(m) for m in members]


def partition(context_lens, kv_heads: int, world: int, min_heads_per_rank: int = 1) -> list:
    """The shard of every rank: rank = request_group * tp + head_group."""
    tp = head_split(kv_heads, world, min_heads_per_rank)
    per = kv_heads // tp
    groups = balance_requests(context_lens, world // tp)
    return [Shard(rank=g * tp + h, head_begin=h * per, head_end=(h + 1) * per, requests=tuple(groups[g]))
            for g in range(world // tp) for h in range(tp)]


def shard_of(rank: int, context_lens, kv_heads: int, world: int, min_heads_per_rank: int = 1) -> Shard:
    if not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world {world}")
    return partition(context_lens, kv_heads, world, min_heads_per_rank)[rank]
